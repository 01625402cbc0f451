// int4w V reconstruction of the selected tokens (sm_100a):
//   v[i, h, c] = fp16( W[h*d + c, :] . (deq K[t] - K_mean) + V_mean[h*d + c]
//                      + int2 residual[t, h, c] * step_h ),   t = top[i, h]
// (modules/kvr_retrieval.py:131-134, 394-402: the V-predict GEMM over the
// unique selected tokens, the residual add and the .half() of ret_v).
//
// The contraction runs on the tensor cores straight from the packed int4
// codes.  Since deq K[t, j] = code[t, j] * step[j], the prediction is
//   sum_j (W[r, j] * step[j]) * code[t, j] + (V_mean[r] - sum_j W[r, j] K_mean[j])
// with codes in [-8, 7], which are exact fp16 operands.  W' = W * diag(step)
// is prepared once per calibration (kvr_int4w_vpredict_prepare): each output
// row r is scaled by a power of two 2^e_r that puts its largest |W'| in
// [2^13, 2^14), then split into fp16 hi + lo parts; the two MMAs (codes x hi,
// codes x lo) accumulate in fp32 into the same registers and the epilogue
// multiplies by 2^-e_r (exact).  The representation error of W' is 2^-22
// relative (or 2^-25 of the row's largest entry), i.e. fp32-level: the
// result differs from the reference's fp32 GEMM only by summation order.
//
// Work split: a CTA owns M (64, or 32 when that leaves SMs idle) selected
// tokens of one KV head and all 128 output channels; its 8 warps tile
// (M/16 token slabs) x (128 channels), mma.sync m16n8k16 (fp16 in, fp32
// accumulate).  The contraction dimension (n_kv * d) advances in chunks of
// 64: the codes of the CTA's tokens are gathered from their packed rows and widened to
// fp16 in registers, W' hi/lo chunks (32 KB) arrive by cp.async; both are
// double-buffered so the next chunk loads while the current one multiplies.
#include "kvr_common.cuh"

namespace kvr {

namespace vp {
constexpr int kD = 128;
constexpr int kK = 64;          // contraction chunk
constexpr int kPitch = kK + 8;  // smem row pitch in halves (144 B: conflict-free ldmatrix)
constexpr int kBHalves = 2 * kD * kPitch;  // hi and lo parts
template <int M>
struct Cfg {
  static constexpr int kAHalves = M * kPitch;
  static constexpr int kStageHalves = kAHalves + kBHalves;
  static constexpr size_t kSmem = 2 * kStageHalves * 2;  // two stages, bytes
  static constexpr int kWarpsM = M / 16;                  // 16-row slabs
  static constexpr int kWarpsN = 8 / kWarpsM;             // column groups
  static constexpr int kColsW = kD / kWarpsN;             // columns per warp
  static constexpr int kNT = kColsW / 8;                  // n8 tiles per warp
  static constexpr int kABytesT = M * (kK / 2) / 256;     // packed code bytes per thread per chunk
};
}  // namespace vp

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2*NW int4 codes (NW packed words, even element in each byte's high nibble)
// -> fp16 values in element order, as half2 words.
template <int NW>
__device__ __forceinline__ void codes_to_half(const uint32_t (&w)[NW], uint32_t (&h)[4 * NW]) {
#pragma unroll
  for (int b = 0; b < 4 * NW; ++b) {
    const uint32_t byte = (w[b >> 2] >> (8 * (b & 3))) & 0xffu;
    const __half e = __int2half_rn((int)(byte >> 4) - 8), o = __int2half_rn((int)(byte & 15u) - 8);
    h[b] = (uint32_t)__half_as_ushort(e) | ((uint32_t)__half_as_ushort(o) << 16);
  }
}

template <int M>
__global__ void __launch_bounds__(256) vpredict_kernel(const uint8_t *__restrict__ kp, const int64_t *__restrict__ top,
                                                       const int32_t *__restrict__ count, int k, int n_kv,
                                                       const __half *__restrict__ w3, const float *__restrict__ unscale,
                                                       const float *__restrict__ bias, const uint8_t *__restrict__ vr,
                                                       const float *__restrict__ vrs, __half *__restrict__ out) {
  using namespace vp;
  using C = Cfg<M>;
  constexpr int NWORD = C::kABytesT / 4;  // 32-bit code words per thread per chunk (2 or 1)
  extern __shared__ __align__(16) unsigned char smraw[];
  __half *sm = reinterpret_cast<__half *>(smraw);
  const int h = blockIdx.y;
  const int i0 = blockIdx.x * M;
  const int n_valid = count ? min(k, __ldg(count)) : k;
  if (i0 >= n_valid) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int KD = n_kv * kD;
  const int64_t row_bytes = (int64_t)n_kv * (kD / 2);
  const int nch = KD / kK;
  // A producer: thread -> (token row, piece of C::kABytesT bytes of the chunk's 32 code bytes)
  constexpr int PPR = (kK / 2) / C::kABytesT;  // pieces per row
  const int ar = tid / PPR, ap = tid % PPR;
  const bool a_ok = i0 + ar < n_valid;
  const int64_t tok = a_ok ? __ldg(top + (int64_t)(i0 + ar) * n_kv + h) : 0;
  const uint8_t *arow = kp + tok * row_bytes;
  const __half *wh = w3 + (int64_t)h * 2 * kD * KD;  // [part][c][j]

  auto issue_b = [&](int c, int stage) {
    __half *Bs = sm + stage * C::kStageHalves + C::kAHalves;
    const int j0 = c * kK;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int idx = tid + it * 256;          // 2048 pieces of 16 B
      const int rr = idx >> 3, seg = idx & 7;  // rr in [0, 256): part * 128 + c
      cp_async16(Bs + rr * kPitch + seg * 8, wh + (int64_t)rr * KD + j0 + seg * 8);
    }
    cp_async_commit();
  };
  auto load_a = [&](int c, uint32_t (&w)[NWORD]) {
#pragma unroll
    for (int q = 0; q < NWORD; ++q) w[q] = 0x88888888u;  // codes 0
    if (!a_ok) return;
    if constexpr (NWORD == 2) {
      const uint2 v = __ldg(reinterpret_cast<const uint2 *>(arow + c * (kK / 2) + ap * 8));
      w[0] = v.x;
      w[NWORD - 1] = v.y;
    } else {
      w[0] = __ldg(reinterpret_cast<const uint32_t *>(arow + c * (kK / 2) + ap * 4));
    }
  };
  auto store_a = [&](const uint32_t (&w)[NWORD], int stage) {
    uint32_t hv[4 * NWORD];
    codes_to_half<NWORD>(w, hv);
    __half *As = sm + stage * C::kStageHalves;
    uint4 *dst = reinterpret_cast<uint4 *>(As + ar * kPitch + ap * (8 * NWORD));
#pragma unroll
    for (int q = 0; q < NWORD; ++q) dst[q] = make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]);
  };

  float acc[C::kNT][4];
#pragma unroll
  for (int n = 0; n < C::kNT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
  const int wm = (warp % C::kWarpsM) * 16, wn = (warp / C::kWarpsM) * C::kColsW;

  issue_b(0, 0);
  {
    uint32_t w0[NWORD];
    load_a(0, w0);
    store_a(w0, 0);
  }
  for (int c = 0; c < nch; ++c) {
    const int st = c & 1;
    uint32_t nxt[NWORD];
    if (c + 1 < nch) {
      issue_b(c + 1, st ^ 1);
      load_a(c + 1, nxt);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __half *As = sm + st * C::kStageHalves;
    const __half *Bs = As + C::kAHalves;
#pragma unroll
    for (int kk = 0; kk < kK; kk += 16) {
      uint32_t a[4];
      ldsm_x4(a, As + (wm + (lane & 7) + ((lane >> 3) & 1) * 8) * kPitch + kk + (lane >> 4) * 8);
#pragma unroll
      for (int part = 0; part < 2; ++part) {
#pragma unroll
        for (int np = 0; np < C::kNT / 2; ++np) {  // pairs of n8 tiles
          uint32_t b[4];
          const int nrow = part * kD + wn + np * 16 + (lane & 7) + (lane >> 4) * 8;
          ldsm_x4(b, Bs + nrow * kPitch + kk + ((lane >> 3) & 1) * 8);
          mma16816(acc[2 * np], a, b[0], b[1]);
          mma16816(acc[2 * np + 1], a, b[2], b[3]);
        }
      }
    }
    if (c + 1 < nch) store_a(nxt, st ^ 1);
    __syncthreads();
  }

  // epilogue: unscale, bias, int2 residual, fp16
  const float step = __fdiv_rn(__fmul_rn(2.0f, __ldg(vrs + h)), 4.0f);
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int half_ = 0; half_ < 2; ++half_) {
    const int i = i0 + wm + g + half_ * 8;
    if (i >= n_valid) continue;
    const int64_t t = __ldg(top + (int64_t)i * n_kv + h);
    const uint8_t *rrow = vr + (t * n_kv + h) * (kD / 4);
#pragma unroll
    for (int n = 0; n < C::kNT; ++n) {
      const int col = wn + n * 8 + 2 * t4;
      const int r = h * kD + col;
      float v2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float pred = __fadd_rn(__fmul_rn(acc[n][half_ * 2 + e], __ldg(unscale + r + e)), __ldg(bias + r + e));
        const uint32_t byte = __ldg(rrow + (col + e) / 4);
        const int code = (int)((byte >> (6 - 2 * ((col + e) & 3))) & 3u) - 2;
        v2[e] = __fadd_rn(pred, __fmul_rn((float)code, step));
      }
      *reinterpret_cast<__half2 *>(out + ((int64_t)i * n_kv + h) * kD + col) = __floats2half2_rn(v2[0], v2[1]);
    }
  }
}

// One CTA per output row r: W'[r, j] = W[r, j] * step[j], the row's power-of-two
// scale, the fp16 hi/lo split and the bias V_mean[r] - sum_j W[r, j] K_mean[j]
// (accumulated in fp64).
__global__ void __launch_bounds__(256) vpredict_prepare_kernel(const float *__restrict__ W,
                                                               const float *__restrict__ kmean,
                                                               const float *__restrict__ vmean,
                                                               const float *__restrict__ kscales, int n_kv,
                                                               __half *__restrict__ w3, float *__restrict__ unscale,
                                                               float *__restrict__ bias) {
  constexpr int kD = vp::kD;
  __shared__ float red[8];
  __shared__ double redd[8];
  const int KD = n_kv * kD;
  const int r = blockIdx.x;
  const int h = r / kD, c = r - h * kD;
  const float *wr = W + (int64_t)r * KD;
  float mx = 0.0f;
  double bs = 0.0;
  for (int j = threadIdx.x; j < KD; j += blockDim.x) {
    const float step = __fdiv_rn(__fmul_rn(2.0f, __ldg(kscales + j)), 16.0f);
    mx = fmaxf(mx, fabsf(__fmul_rn(__ldg(wr + j), step)));
    bs += (double)__ldg(wr + j) * (double)__ldg(kmean + j);
  }
  mx = warp_max(mx);
  for (int o = 16; o > 0; o >>= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o);
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = mx;
    redd[threadIdx.x >> 5] = bs;
  }
  __syncthreads();
  mx = 0.0f;
  bs = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    mx = fmaxf(mx, red[w]);
    bs += redd[w];
  }
  int e = 0;
  if (mx > 0.0f) {
    int ex;
    frexpf(mx, &ex);  // mx in [2^(ex-1), 2^ex)
    e = 14 - ex;      // scaled max in [2^13, 2^14)
  }
  const float sc = ldexpf(1.0f, e);
  if (threadIdx.x == 0) {
    unscale[r] = ldexpf(1.0f, -e);
    bias[r] = (float)((double)__ldg(vmean + r) - bs);
  }
  __half *hi = w3 + ((int64_t)(h * 2 + 0) * kD + c) * KD;
  __half *lo = w3 + ((int64_t)(h * 2 + 1) * kD + c) * KD;
  for (int j = threadIdx.x; j < KD; j += blockDim.x) {
    const float step = __fdiv_rn(__fmul_rn(2.0f, __ldg(kscales + j)), 16.0f);
    const float x = __fmul_rn(__fmul_rn(__ldg(wr + j), step), sc);
    const __half xh = __float2half_rn(x);
    hi[j] = xh;
    lo[j] = __float2half_rn(__fsub_rn(x, __half2float(xh)));
  }
}

}  // namespace kvr

using namespace kvr;

extern "C" size_t kvr_int4w_vpredict_weights_bytes(int n_kv, int d) {
  if (n_kv <= 0 || d != vp::kD) return 0;
  const size_t KD = (size_t)n_kv * d;
  return KD * 2 * KD * 2;  // (n_kv, 2, d, KD) fp16
}

extern "C" int kvr_int4w_vpredict_prepare(const float *W, const float *k_mean, const float *v_mean,
                                          const float *k_scales, int n_kv, int d, void *w3, float *unscale,
                                          float *bias, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == vp::kD, "kvr_int4w_vpredict_prepare: head_dim must be 128");
  KVR_REQUIRE(n_kv > 0 && n_kv <= 64, "kvr_int4w_vpredict_prepare: bad n_kv %d", n_kv);
  KVR_REQUIRE(W && k_mean && v_mean && k_scales && w3 && unscale && bias, "kvr_int4w_vpredict_prepare: null pointer");
  vpredict_prepare_kernel<<<n_kv * d, 256, 0, as_cuda(stream)>>>(W, k_mean, v_mean, k_scales, n_kv,
                                                                reinterpret_cast<__half *>(w3), unscale, bias);
  return check_launch("kvr_int4w_vpredict_prepare");
}

extern "C" int kvr_int4w_vpredict(const uint8_t *k_packed, const int64_t *top, const int32_t *count, int k, int n_kv,
                                  int d, const void *w3, const float *unscale, const float *bias,
                                  const uint8_t *vr_packed, const float *vr_scales, uint16_t *ret_v,
                                  kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == vp::kD, "kvr_int4w_vpredict: head_dim must be 128");
  KVR_REQUIRE(n_kv > 0 && n_kv <= 64 && k >= 0, "kvr_int4w_vpredict: bad sizes");
  KVR_REQUIRE(k_packed && top && w3 && unscale && bias && vr_packed && vr_scales && ret_v,
              "kvr_int4w_vpredict: null pointer");
  auto al = [](const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  KVR_REQUIRE(al(k_packed, 8) && al(w3, 16) && al(ret_v, 4), "kvr_int4w_vpredict: misaligned buffers");
  if (k == 0) return KVR_OK;
  // 32-token tiles (more CTAs in flight) unless the selection is large enough
  // to fill the GPU with 64-token tiles
  const bool small_m = (int64_t)((k + 63) / 64) * n_kv < 2 * 148;
  static thread_local int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaFuncSetAttribute(vpredict_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vp::Cfg<64>::kSmem);
    cudaFuncSetAttribute(vpredict_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vp::Cfg<32>::kSmem);
    attr_dev = dev;
  }
  if (small_m) {
    dim3 grid((unsigned)((k + 31) / 32), (unsigned)n_kv);
    vpredict_kernel<32><<<grid, 256, vp::Cfg<32>::kSmem, as_cuda(stream)>>>(
        k_packed, top, count, k, n_kv, reinterpret_cast<const __half *>(w3), unscale, bias, vr_packed, vr_scales,
        reinterpret_cast<__half *>(ret_v));
  } else {
    dim3 grid((unsigned)((k + 63) / 64), (unsigned)n_kv);
    vpredict_kernel<64><<<grid, 256, vp::Cfg<64>::kSmem, as_cuda(stream)>>>(
        k_packed, top, count, k, n_kv, reinterpret_cast<const __half *>(w3), unscale, bias, vr_packed, vr_scales,
        reinterpret_cast<__half *>(ret_v));
  }
  return check_launch("kvr_int4w_vpredict");
}
