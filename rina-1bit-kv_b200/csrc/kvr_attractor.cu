// int4w attractor branch of retrieve_topk on the device (sm_100a).
//
// Reference: modules/kvr_retrieval.py:248-263 (compute_attractor_scores) and
// :332-367 (the branch taken after build_attractors): cosine of the head-0
// group-mean query against the 128 basin centroids, the top 48 basins, the
// top 16 tokens of each basin by head-0 cosine of the re-rotated dequantised
// K, the sorted union, the exclusion range; the same token list serves every
// head.  The reference does this in a Python loop with a boolean mask,
// .nonzero() and an argsort per basin (one host sync each).  Here it is three
// launches with no host sync:
//   1. attractor_basins_kernel (1 CTA): centroid cosines, top basins;
//   2. attractor_tokens_kernel (one CTA per chosen basin): the basin's tokens
//      are gathered in ascending order from the label array (every labelled
//      token, including tokens appended after the clustering); each warp
//      scores tokens, then a block top-16;
//   3. attractor_merge_kernel (1 CTA): drop empty slots and excluded tokens,
//      sort ascending (basins are disjoint, so there are no duplicates), write
//      the (rows, n_kv) index list and the device-side row count.
// Ties are broken by index ascending (score descending first); torch's
// argsort/topk leave tie order unspecified.
#include "kvr_common.cuh"
#include "kvr_topk.cuh"

namespace kvr {

namespace attr {
constexpr int kD = 128;
constexpr int kPerBasin = 16;
constexpr int kMaxBasins = 1024;
constexpr int kMaxTopA = 64;
}  // namespace attr

// group-mean of query heads [0, g) of head 0 into qa[128]; returns ||qa|| + 1e-8
__device__ float stage_qavg0(const float *__restrict__ q, int g, float *qa, float *red) {
  const int tid = threadIdx.x;
  if (tid < attr::kD) {
    float s = 0.0f;
    for (int j = 0; j < g; ++j) s += q[j * attr::kD + tid];
    qa[tid] = s / (float)g;
  }
  __syncthreads();
  if (tid < 32) {
    float s = 0.0f;
    for (int c = tid; c < attr::kD; c += 32) s = fmaf(qa[c], qa[c], s);
    s = warp_sum(s);
    if (tid == 0) red[0] = sqrtf(s) + 1e-8f;
  }
  __syncthreads();
  return red[0];
}

__global__ void __launch_bounds__(256) attractor_basins_kernel(const float *__restrict__ q, int g,
                                                               const float *__restrict__ cent, int na, int top_a,
                                                               int32_t *__restrict__ basins) {
  __shared__ float qa[attr::kD];
  __shared__ float red[1];
  __shared__ float sc[attr::kMaxBasins];
  const float qn = stage_qavg0(q, g, qa, red);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int a = warp; a < na; a += 8) {
    const float *cr = cent + (int64_t)a * attr::kD;
    float dot = 0.0f, nn = 0.0f;
    for (int c = lane; c < attr::kD; c += 32) {
      dot = fmaf(qa[c], cr[c], dot);
      nn = fmaf(cr[c], cr[c], nn);
    }
    dot = warp_sum(dot);
    nn = warp_sum(nn);
    if (lane == 0) {
      float s = dot / (qn * (sqrtf(nn) + 1e-8f));
      sc[a] = (s != s) ? -INFINITY : s;
    }
  }
  __syncthreads();
  // rank = number of basins ahead under (score desc, index asc)
  for (int a = threadIdx.x; a < na; a += blockDim.x) {
    const unsigned long long ka = make_key(sc[a], a);
    int rank = 0;
    for (int b = 0; b < na; ++b) rank += make_key(sc[b], b) > ka;
    if (rank < top_a) basins[rank] = a;
  }
}

// head-0 cosine of token t: warp-wide, lane owns dims 4l..4l+3
__device__ __forceinline__ float token_cosine_h0(const uint8_t *__restrict__ kp, int64_t row_bytes,
                                                 const float *step4, const float *qa, float qn,
                                                 const float *__restrict__ cs, const float *__restrict__ sn,
                                                 int64_t rope_stride, int64_t t, int lane) {
  const uint16_t two = __ldg(reinterpret_cast<const uint16_t *>(kp + t * row_bytes + lane * 2));
  const int codes[4] = {(int)((two >> 4) & 15) - 8, (int)(two & 15) - 8, (int)((two >> 12) & 15) - 8,
                        (int)((two >> 8) & 15) - 8};
  float dot = 0.0f, nk = 0.0f;
  const float4 c4 = __ldg(reinterpret_cast<const float4 *>(cs + t * rope_stride + lane * 4));
  const float4 s4 = __ldg(reinterpret_cast<const float4 *>(sn + t * rope_stride + lane * 4));
  const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float kx = __fmul_rn((float)codes[r], step4[r]);
    const float partner = __shfl_xor_sync(0xffffffffu, kx, 16);
    const float rh = lane < 16 ? -partner : partner;
    const float kr = __fadd_rn(__fmul_rn(kx, cv[r]), __fmul_rn(rh, sv[r]));
    dot = fmaf(qa[lane * 4 + r], kr, dot);
    nk = fmaf(kr, kr, nk);
  }
  dot = warp_sum(dot);
  nk = warp_sum(nk);
  float s = dot / (qn * (sqrtf(nk) + 1e-8f));
  return (s != s) ? -INFINITY : s;
}

__global__ void __launch_bounds__(256) attractor_tokens_kernel(
    const float *__restrict__ q, int g, const uint8_t *__restrict__ kp, int n_kv, const float *__restrict__ ks,
    const float *__restrict__ cs, const float *__restrict__ sn, int64_t rope_stride, const int32_t *__restrict__ labels,
    int64_t n_lab, const int32_t *__restrict__ basins, int32_t *__restrict__ scratch_tok,
    float *__restrict__ scratch_sc, int32_t *__restrict__ sel_tok) {
  __shared__ float qa[attr::kD];
  __shared__ float red[1];
  __shared__ __align__(16) unsigned char tsm_raw[sizeof(TopkSmem)];
  __shared__ unsigned long long cand[attr::kPerBasin];
  __shared__ int wcount[8];
  TopkSmem &tsm = *reinterpret_cast<TopkSmem *>(tsm_raw);
  const float qn = stage_qavg0(q, g, qa, red);
  const int b = basins[blockIdx.x];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t *toks = scratch_tok + (int64_t)blockIdx.x * n_lab;
  float *scs = scratch_sc + (int64_t)blockIdx.x * n_lab;
  // the basin's tokens, ascending: ordered compaction of labels == b
  int64_t n = 0;
  for (int64_t r0 = 0; r0 < n_lab; r0 += blockDim.x) {
    const int64_t i = r0 + threadIdx.x;
    const bool m = i < n_lab && __ldg(labels + i) == b;
    const unsigned bal = __ballot_sync(0xffffffffu, m);
    if (lane == 0) wcount[warp] = __popc(bal);
    __syncthreads();
    int64_t before = n, total = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      if (w < warp) before += wcount[w];
      total += wcount[w];
    }
    if (m) toks[before + __popc(bal & ((1u << lane) - 1u))] = (int32_t)i;
    n += total;
    __syncthreads();
  }
  int32_t *out = sel_tok + blockIdx.x * attr::kPerBasin;
  if (n <= attr::kPerBasin) {  // the whole basin (kvr_retrieval.py:345-346)
    for (int r = threadIdx.x; r < attr::kPerBasin; r += blockDim.x) out[r] = r < n ? toks[r] : -1;
    return;
  }
  float step4[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) step4[r] = __fdiv_rn(__fmul_rn(2.0f, __ldg(ks + lane * 4 + r)), 16.0f);
  const int64_t row_bytes = (int64_t)n_kv * (attr::kD / 2);
  for (int64_t p = warp; p < n; p += 8) {
    const int64_t t = toks[p];
    const float s = token_cosine_h0(kp, row_bytes, step4, qa, qn, cs, sn, rope_stride, t, lane);
    if (lane == 0) scs[p] = s;
  }
  __syncthreads();
  block_topk<256>([&](int64_t i) -> float { return __ldcg(scs + i); }, n, attr::kPerBasin, cand, tsm);
  for (int r = threadIdx.x; r < attr::kPerBasin; r += blockDim.x) out[r] = toks[key_index(cand[r])];
}

__global__ void __launch_bounds__(1024) attractor_merge_kernel(const int32_t *__restrict__ sel_tok, int n_slots,
                                                               int64_t ex0, int64_t ex1, int n_kv, int rows_cap,
                                                               int64_t *__restrict__ top,
                                                               int32_t *__restrict__ count) {
  __shared__ int32_t toks[attr::kMaxTopA * attr::kPerBasin];
  __shared__ int n_ok;
  __shared__ int32_t first;
  if (threadIdx.x == 0) {
    n_ok = 0;
    first = 0x7fffffff;
  }
  __syncthreads();
  const bool excl = ex1 > ex0;
  for (int i = threadIdx.x; i < n_slots; i += blockDim.x) {
    int32_t t = sel_tok[i];
    if (t >= 0 && excl && t >= ex0 && t < ex1) t = -1;
    toks[i] = t;
    if (t >= 0) {
      atomicAdd(&n_ok, 1);
      atomicMin(&first, t);
    }
  }
  __syncthreads();
  const int nv = n_ok;
  for (int i = threadIdx.x; i < n_slots; i += blockDim.x) {
    const int32_t t = toks[i];
    if (t < 0) continue;
    int rank = 0;
    for (int j = 0; j < n_slots; ++j) {
      const int32_t u = toks[j];
      rank += (u >= 0 && u < t);
    }
    for (int h = 0; h < n_kv; ++h) top[(int64_t)rank * n_kv + h] = t;
  }
  // rows past the count keep a valid token index (never attended)
  const int32_t fill = nv > 0 ? first : 0;
  for (int i = nv + (int)threadIdx.x; i < rows_cap; i += blockDim.x)
    for (int h = 0; h < n_kv; ++h) top[(int64_t)i * n_kv + h] = fill;
  if (threadIdx.x == 0) *count = nv;
}

}  // namespace kvr

using namespace kvr;

extern "C" size_t kvr_int4w_attractor_workspace_bytes(int64_t n_labelled, int top_a) {
  const size_t ta = (size_t)(top_a > 0 ? top_a : 1);
  const size_t nl = (size_t)(n_labelled > 0 ? n_labelled : 1);
  return align_up((size_t)attr::kMaxTopA * 4, 256) + align_up(ta * attr::kPerBasin * 4, 256) +
         2 * align_up(ta * nl * 4, 256);
}

extern "C" int kvr_int4w_attractor_select(const float *q, int n_q, int n_kv, const uint8_t *k_packed,
                                          const float *k_scales, const float *cos_tbl, const float *sin_tbl,
                                          int64_t rope_stride, const float *centroids, int n_attractors,
                                          const int32_t *labels, int64_t n_labelled, int top_a, int64_t ex_start,
                                          int64_t ex_end, int64_t *top, int32_t *count, void *workspace,
                                          size_t workspace_bytes, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(q && k_packed && k_scales && cos_tbl && sin_tbl && centroids && labels && top && count && workspace,
              "kvr_int4w_attractor_select: null pointer");
  KVR_REQUIRE(n_kv > 0 && n_q % n_kv == 0 && n_q >= n_kv, "kvr_int4w_attractor_select: bad head counts");
  KVR_REQUIRE(n_attractors > 0 && n_attractors <= attr::kMaxBasins, "kvr_int4w_attractor_select: 1..%d basins",
              attr::kMaxBasins);
  KVR_REQUIRE(top_a > 0 && top_a <= n_attractors && top_a <= attr::kMaxTopA, "kvr_int4w_attractor_select: bad top_a");
  KVR_REQUIRE(n_labelled > 0 && n_labelled < 0x7fffffffll, "kvr_int4w_attractor_select: bad n_labelled");
  KVR_REQUIRE(rope_stride >= attr::kD, "kvr_int4w_attractor_select: rope tables need full rows");
  KVR_REQUIRE(workspace_bytes >= kvr_int4w_attractor_workspace_bytes(n_labelled, top_a),
              "kvr_int4w_attractor_select: workspace too small");
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "kvr_int4w_attractor_select: workspace alignment");
  char *p = reinterpret_cast<char *>(workspace);
  int32_t *basins = reinterpret_cast<int32_t *>(p);
  p += align_up((size_t)attr::kMaxTopA * 4, 256);
  int32_t *sel_tok = reinterpret_cast<int32_t *>(p);
  p += align_up((size_t)top_a * attr::kPerBasin * 4, 256);
  int32_t *scratch_tok = reinterpret_cast<int32_t *>(p);
  p += align_up((size_t)top_a * n_labelled * 4, 256);
  float *scratch_sc = reinterpret_cast<float *>(p);
  cudaStream_t st = as_cuda(stream);
  const int g = n_q / n_kv;
  attractor_basins_kernel<<<1, 256, 0, st>>>(q, g, centroids, n_attractors, top_a, basins);
  attractor_tokens_kernel<<<top_a, 256, 0, st>>>(q, g, k_packed, n_kv, k_scales, cos_tbl, sin_tbl, rope_stride,
                                                 labels, n_labelled, basins, scratch_tok, scratch_sc, sel_tok);
  attractor_merge_kernel<<<1, 1024, 0, st>>>(sel_tok, top_a * attr::kPerBasin, ex_start, ex_end, n_kv,
                                             top_a * attr::kPerBasin, top, count);
  return check_launch("kvr_int4w_attractor_select");
}
