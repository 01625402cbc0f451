// On-device k-means for the int4w attractor branch (replaces the host
// MiniBatchKMeans of kvr_retrieval.py:234-246).
//
// Lloyd iterations over n points of d = 128 fp32 values, k <= 256 clusters:
//   init      centroid j = point floor(j * n / k)            (deterministic)
//   assign    label(x) = argmin_j ||c_j||^2 - 2 x.c_j (lowest j on ties)
//   update    c_j = mean of the points labelled j (unchanged if none)
// The update is deterministic: every CTA sums its block of points per
// cluster in point order (one thread per dimension), and one pass adds the
// CTA partials in CTA order.  After `iters` updates a last assignment gives
// the labels.  Spec: oracle/int4w_ref.py kmeans_lloyd.
#include "kvr_common.cuh"

namespace kvr {

constexpr int kKmD = 128;
constexpr int kKmMaxK = 256;
constexpr int kKmBlock = 256;  // points per CTA in the assignment and partial-sum kernels

__global__ void km_init_kernel(const float *__restrict__ x, int64_t n, int k, float *__restrict__ c) {
  const int j = blockIdx.x, t = threadIdx.x;  // 128 threads
  const int64_t src = (int64_t)j * n / k;
  c[(int64_t)j * kKmD + t] = x[src * kKmD + t];
}

// One thread per point; the k centroids (and their squared norms) in shared memory.
__global__ void __launch_bounds__(kKmBlock) km_assign_kernel(const float *__restrict__ x, int64_t n, int k,
                                                             const float *__restrict__ c, int32_t *__restrict__ lab) {
  extern __shared__ __align__(16) float cs[];  // [k][128] then norms[k]
  float *cn = cs + (int64_t)k * kKmD;
  for (int i = threadIdx.x; i < k * kKmD / 4; i += blockDim.x)
    reinterpret_cast<float4 *>(cs)[i] = __ldg(reinterpret_cast<const float4 *>(c) + i);
  __syncthreads();
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    float s = 0.0f;
    for (int e = 0; e < kKmD; ++e) s = fmaf(cs[j * kKmD + e], cs[j * kKmD + e], s);
    cn[j] = s;
  }
  __syncthreads();
  const int64_t p = (int64_t)blockIdx.x * kKmBlock + threadIdx.x;
  if (p >= n) return;
  float xv[kKmD];
  const float4 *xp = reinterpret_cast<const float4 *>(x + p * kKmD);
#pragma unroll
  for (int e = 0; e < kKmD / 4; ++e) {
    const float4 v = __ldg(xp + e);
    xv[4 * e] = v.x; xv[4 * e + 1] = v.y; xv[4 * e + 2] = v.z; xv[4 * e + 3] = v.w;
  }
  float best = INFINITY;
  int arg = 0;
  for (int j = 0; j < k; ++j) {
    const float4 *cj = reinterpret_cast<const float4 *>(cs + j * kKmD);
    float acc = 0.0f;
#pragma unroll
    for (int e = 0; e < kKmD / 4; ++e) {
      const float4 v = cj[e];
      acc = fmaf(xv[4 * e], v.x, acc);
      acc = fmaf(xv[4 * e + 1], v.y, acc);
      acc = fmaf(xv[4 * e + 2], v.z, acc);
      acc = fmaf(xv[4 * e + 3], v.w, acc);
    }
    const float dist = fmaf(-2.0f, acc, cn[j]);
    if (dist < best) {
      best = dist;
      arg = j;
    }
  }
  lab[p] = arg;
}

// Per-CTA cluster sums over the CTA's block of points, in point order: thread
// t owns dimension t of every cluster.  part: [ctas][k][128], cnt: [ctas][k].
__global__ void __launch_bounds__(kKmD) km_partial_kernel(const float *__restrict__ x, int64_t n, int k,
                                                          const int32_t *__restrict__ lab, float *__restrict__ part,
                                                          int32_t *__restrict__ cnt) {
  extern __shared__ __align__(16) float ps[];  // [k][128]
  int32_t *pc = reinterpret_cast<int32_t *>(ps + (int64_t)k * kKmD);
  const int t = threadIdx.x;
  for (int j = 0; j < k; ++j) ps[j * kKmD + t] = 0.0f;
  for (int j = t; j < k; j += blockDim.x) pc[j] = 0;
  __syncthreads();
  const int64_t p0 = (int64_t)blockIdx.x * kKmBlock;
  const int64_t p1 = p0 + kKmBlock < n ? p0 + kKmBlock : n;
  for (int64_t p = p0; p < p1; ++p) {
    const int l = __ldg(lab + p);
    ps[l * kKmD + t] += __ldg(x + p * kKmD + t);
    if (t == 0) pc[l] += 1;
  }
  __syncthreads();
  float *dst = part + (int64_t)blockIdx.x * k * kKmD;
  for (int j = 0; j < k; ++j) dst[j * kKmD + t] = ps[j * kKmD + t];
  for (int j = t; j < k; j += blockDim.x) cnt[(int64_t)blockIdx.x * k + j] = pc[j];
}

// c_j = (sum over CTAs, in CTA order) / count; unchanged when the count is 0.
__global__ void km_update_kernel(const float *__restrict__ part, const int32_t *__restrict__ cnt, int nctas, int k,
                                 float *__restrict__ c) {
  const int j = blockIdx.x, t = threadIdx.x;  // 128 threads
  float s = 0.0f;
  int64_t m = 0;
  for (int b = 0; b < nctas; ++b) {
    s += part[((int64_t)b * k + j) * kKmD + t];
    m += cnt[(int64_t)b * k + j];
  }
  if (m > 0) c[(int64_t)j * kKmD + t] = s / (float)m;
}

// Basin of tokens appended after clustering: head-0 K of tokens [t0, t1)
// dequantised from the packed int4 codes (code * 2*s/16, as the clustering
// input was formed) and assigned with the same rule as km_assign_kernel.
__global__ void __launch_bounds__(kKmBlock) km_assign_packed_kernel(const uint8_t *__restrict__ kp, int n_kv,
                                                                    const float *__restrict__ ks, int64_t t0,
                                                                    int64_t t1, int k, const float *__restrict__ c,
                                                                    int32_t *__restrict__ lab) {
  extern __shared__ __align__(16) float cs[];  // [k][128] then norms[k]
  float *cn = cs + (int64_t)k * kKmD;
  for (int i = threadIdx.x; i < k * kKmD / 4; i += blockDim.x)
    reinterpret_cast<float4 *>(cs)[i] = __ldg(reinterpret_cast<const float4 *>(c) + i);
  __syncthreads();
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    float s = 0.0f;
    for (int e = 0; e < kKmD; ++e) s = fmaf(cs[j * kKmD + e], cs[j * kKmD + e], s);
    cn[j] = s;
  }
  __syncthreads();
  const int64_t p = t0 + (int64_t)blockIdx.x * kKmBlock + threadIdx.x;
  if (p >= t1) return;
  float xv[kKmD];
  const uint8_t *row = kp + p * (int64_t)n_kv * (kKmD / 2);  // head 0
#pragma unroll
  for (int e = 0; e < kKmD / 2; ++e) {
    const uint32_t byte = __ldg(row + e);
    xv[2 * e] = __fmul_rn((float)((int)(byte >> 4) - 8), __fdiv_rn(__fmul_rn(2.0f, __ldg(ks + 2 * e)), 16.0f));
    xv[2 * e + 1] = __fmul_rn((float)((int)(byte & 15u) - 8), __fdiv_rn(__fmul_rn(2.0f, __ldg(ks + 2 * e + 1)), 16.0f));
  }
  float best = INFINITY;
  int arg = 0;
  for (int j = 0; j < k; ++j) {
    const float4 *cj = reinterpret_cast<const float4 *>(cs + j * kKmD);
    float acc = 0.0f;
#pragma unroll
    for (int e = 0; e < kKmD / 4; ++e) {
      const float4 v = cj[e];
      acc = fmaf(xv[4 * e], v.x, acc);
      acc = fmaf(xv[4 * e + 1], v.y, acc);
      acc = fmaf(xv[4 * e + 2], v.z, acc);
      acc = fmaf(xv[4 * e + 3], v.w, acc);
    }
    const float dist = fmaf(-2.0f, acc, cn[j]);
    if (dist < best) {
      best = dist;
      arg = j;
    }
  }
  lab[p] = arg;
}

}  // namespace kvr

using namespace kvr;

extern "C" int kvr_int4w_assign_basins(const uint8_t *k_packed, const float *k_scales, int n_kv, int64_t t0,
                                       int64_t t1, const float *centroids, int k, int32_t *labels,
                                       kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(k_packed && k_scales && centroids && labels, "kvr_int4w_assign_basins: null pointer");
  KVR_REQUIRE(n_kv > 0 && k >= 1 && k <= kKmMaxK && t0 >= 0 && t1 >= t0, "kvr_int4w_assign_basins: bad sizes");
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(centroids) & 15) == 0, "kvr_int4w_assign_basins: centroids alignment");
  if (t1 == t0) return KVR_OK;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaFuncSetAttribute(km_assign_packed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kKmMaxK * (kKmD + 1) * 4);
    set_dev = dev;
  }
  const int64_t blocks = (t1 - t0 + kKmBlock - 1) / kKmBlock;
  km_assign_packed_kernel<<<(unsigned)blocks, kKmBlock, (size_t)k * (kKmD + 1) * 4, as_cuda(stream)>>>(
      k_packed, n_kv, k_scales, t0, t1, k, centroids, labels);
  return check_launch("kvr_int4w_assign_basins");
}

static int64_t km_ctas(int64_t n) { return (n + kKmBlock - 1) / kKmBlock; }

extern "C" size_t kvr_kmeans_workspace_bytes(int64_t n, int k) {
  const int64_t b = km_ctas(n);
  return align_up((size_t)b * k * kKmD * 4, 256) + align_up((size_t)b * k * 4, 256);
}

extern "C" int kvr_kmeans(const float *x, int64_t n, int d, int k, int iters, float *centroids, int32_t *labels,
                          void *workspace, size_t workspace_bytes, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(x && centroids && labels && workspace, "kvr_kmeans: null pointer");
  KVR_REQUIRE(d == kKmD, "kvr_kmeans: d must be 128");
  KVR_REQUIRE(k >= 1 && k <= kKmMaxK, "kvr_kmeans: k must be in [1, %d]", kKmMaxK);
  KVR_REQUIRE(n >= k, "kvr_kmeans: need at least k points");
  KVR_REQUIRE(iters >= 0, "kvr_kmeans: negative iteration count");
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(centroids) & 15) == 0,
              "kvr_kmeans: x and centroids must be 16-byte aligned");
  KVR_REQUIRE(workspace_bytes >= kvr_kmeans_workspace_bytes(n, k), "kvr_kmeans: workspace too small");
  cudaStream_t st = as_cuda(stream);
  const int64_t b = km_ctas(n);
  float *part = reinterpret_cast<float *>(workspace);
  int32_t *cnt = reinterpret_cast<int32_t *>(reinterpret_cast<char *>(workspace) +
                                             align_up((size_t)b * k * kKmD * 4, 256));
  const size_t smem_assign = (size_t)k * (kKmD + 1) * 4;
  const size_t smem_part = (size_t)k * kKmD * 4 + (size_t)k * 4;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaFuncSetAttribute(km_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kKmMaxK * (kKmD + 1) * 4);
    cudaFuncSetAttribute(km_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kKmMaxK * kKmD * 4 + kKmMaxK * 4);
    set_dev = dev;
  }
  km_init_kernel<<<k, kKmD, 0, st>>>(x, n, k, centroids);
  for (int it = 0; it < iters; ++it) {
    km_assign_kernel<<<(unsigned)b, kKmBlock, smem_assign, st>>>(x, n, k, centroids, labels);
    km_partial_kernel<<<(unsigned)b, kKmD, smem_part, st>>>(x, n, k, labels, part, cnt);
    km_update_kernel<<<k, kKmD, 0, st>>>(part, cnt, (int)b, k, centroids);
  }
  km_assign_kernel<<<(unsigned)b, kKmBlock, smem_assign, st>>>(x, n, k, centroids, labels);
  return check_launch("kvr_kmeans");
}
