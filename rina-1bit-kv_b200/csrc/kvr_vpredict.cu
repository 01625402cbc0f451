// int4w V reconstruction of the selected tokens (sm_100a, tcgen05):
//   v[i, h, c] = fp16( W[h*d + c, :] . (deq K[t] - K_mean) + V_mean[h*d + c]
//                      + int2 residual[t, h, c] * step_h ),   t = top[i, h]
// (modules/kvr_retrieval.py:131-134, 394-402: the V-predict GEMM over the
// unique selected tokens, the residual add and the .half() of ret_v).
//
// The contraction runs on the 5th-generation tensor cores straight from the
// packed int4 codes.  Since deq K[t, j] = code[t, j] * step[j], the
// prediction is
//   sum_j (W[r, j] * step[j]) * code[t, j] + (V_mean[r] - sum_j W[r, j] K_mean[j])
// with codes in [-8, 7], which are exact fp16 operands.  W' = W * diag(step)
// is prepared once per calibration (kvr_int4w_vpredict_prepare): each output
// row r is scaled by a power of two 2^e_r that puts its largest |W'| in
// [2^13, 2^14), then split into fp16 hi + lo parts; the MMAs of both parts
// accumulate in fp32 into the same tensor-memory accumulator and the
// epilogue multiplies by 2^-e_r (exact).  The representation error of W' is
// 2^-22 relative (or 2^-25 of the row's largest entry), i.e. fp32-level: the
// result differs from the reference's fp32 GEMM only by summation order.
//
// Work split: a CTA owns 128 selected tokens of one KV head (MMA M = 128)
// and half of its 128 output channels (N = 64: twice the CTAs and half the
// W' bytes each, since the bytes in flight per SM bound the W' stream); the
// contraction (n_kv * d) advances in chunks of 64.  Roles: warps 0-7 (two
// threads per token row) copy their packed rows into shared memory once
// (cp.async), then widen each chunk's codes to fp16 into the A stage and
// finally run the epilogue from tensor memory (32 channels each); warp 8
// streams the W' chunks (hi + lo, 16 KB, laid out by the prepare kernel as
// the MMA's shared-memory image) with one bulk copy each; warp 9 issues
// tcgen05.mma (8 per chunk: 4 K-steps x 2 parts).  Operands are K-major, no
// swizzle: 8-row x 16-byte core matrices, SBO = 128 B between 8-row groups,
// LBO = (rows / 8) * 128 B between 8-element K chunks.  Every wait is
// bounded; a timeout sets the error word read by kvr_int4w_vpredict_status,
// lets copies and MMAs in flight finish and frees the tensor memory.
#include "kvr_common.cuh"

namespace kvr {

namespace vp {
constexpr int kD = 128;
constexpr int kK = 64;                          // contraction chunk
constexpr int kM = 128;                         // tokens per CTA (MMA M)
constexpr int kN = 64;                          // output channels per CTA (MMA N): half a head
constexpr int kStages = 4;
constexpr uint32_t kLboA = (kM / 8) * 128;      // 2048 B between 8-element K chunks of A (128 rows)
constexpr uint32_t kLboB = (kN / 8) * 128;      // 1024 B between 8-element K chunks of B (64 rows)
constexpr int kABytes = kM * kK * 2;            // 16 KB
constexpr int kPartBytes = kN * kK * 2;         // 8 KB
constexpr int kBBytes = 2 * kPartBytes;         // hi + lo
constexpr int kStageBytes = kABytes + kBBytes;  // 32 KB
constexpr int kRawPitch = 8 * 64 + 16;          // packed row (n_kv <= 8) + 16 B: conflict-free 16-byte reads
constexpr int kOffRaw = kStages * kStageBytes;
constexpr int kOffConst = kOffRaw + kM * kRawPitch;  // unscale, bias of the head: 2 x 128 fp32
constexpr int kOffBar = kOffConst + 2 * kN * 4;
constexpr int kSmem = kOffBar + 8 * (3 * kStages + 1) + 16;
constexpr int kThreads = 320;  // warps 0-7 A + epilogue, warp 8 W' copies, warp 9 MMA
constexpr uint32_t kTmemCols = kN;
// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, N, M.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
}  // namespace vp

__device__ unsigned g_vp_err;  // bounded waits that gave up (kvr_int4w_vpredict_status)

// sm100 shared-memory matrix descriptor, K-major, no swizzle
__device__ __forceinline__ uint64_t vp_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)((lbo >> 4) & 0x3fffu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fffu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
  return d;
}

__device__ __forceinline__ bool vp_wait(uint64_t *bar, unsigned phase, volatile int *abort_s) {
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    if (mbar_try_wait(bar, phase)) return true;
    if (abort_s != nullptr && (it & 255u) == 255u && *abort_s) return false;
  }
  return false;
}

// 8 int4 codes (one 32-bit word, even element in each byte's high nibble) ->
// 8 fp16 values in element order: fp16(1024 + nibble) has the nibble as its
// mantissa, and subtracting 1032 leaves nibble - 8 exactly.  Byte q's two
// nibbles are placed by one byte permute into the low bytes of the halves.
__device__ __forceinline__ uint4 vp_codes8(uint32_t w) {
  const uint32_t hi = (w >> 4) & 0x0f0f0f0fu, lo = w & 0x0f0f0f0fu;
  const __half2 off = __halves2half2(__ushort_as_half(0x6408u), __ushort_as_half(0x6408u));  // 1032
  uint32_t r[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t x = (__byte_perm(hi, lo, (uint32_t)(q | ((q + 4) << 8) | (q << 16) | ((q + 4) << 24))) &
                        0x00ff00ffu) | 0x64006400u;
    const __half2 v = __hsub2(*reinterpret_cast<const __half2 *>(&x), off);
    r[q] = *reinterpret_cast<const uint32_t *>(&v);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

__global__ void __launch_bounds__(vp::kThreads, 1) vpredict_kernel(
    const uint8_t *__restrict__ kp, const int64_t *__restrict__ top, const int32_t *__restrict__ count, int k,
    int n_kv, const unsigned char *__restrict__ w3, const float *__restrict__ unscale, const float *__restrict__ bias,
    const uint8_t *__restrict__ vr, const float *__restrict__ vrs, __half *__restrict__ out) {
  using namespace vp;
  extern __shared__ __align__(1024) unsigned char sm[];
  uint64_t *full_a = reinterpret_cast<uint64_t *>(sm + kOffBar);
  uint64_t *full_b = full_a + kStages;
  uint64_t *empty = full_b + kStages;
  uint64_t *done = empty + kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float *us_s = reinterpret_cast<float *>(sm + kOffConst);
  float *bs_s = us_s + kN;
  const int h = blockIdx.y >> 1, ch0 = (blockIdx.y & 1) * kN, i0 = blockIdx.x * kM;
  const int n_valid = count ? min(k, __ldg(count)) : k;
  if (i0 >= n_valid) return;  // uniform: before any allocation or barrier
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = n_kv * kD / kK;
  const int row_bytes = n_kv * (kD / 2);

  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 8 * 32) {
    *abort_s = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_a[s], 8);  // one arrive per producer warp
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
  }
  if (tid < kN) {
    us_s[tid] = __ldg(unscale + h * kD + ch0 + tid);
    bs_s[tid] = __ldg(bias + h * kD + ch0 + tid);
  }
  // warps 0-7: thread (m, hf) = (token row i0 + m, half hf of each chunk's
  // 32 code bytes); it copies the 16-byte pieces of the packed row (all
  // heads) that it widens later into shared memory
  const int m = tid & (kM - 1), hf = (tid >> 7) & 1;
  const bool row_ok = warp < 8 && i0 + m < n_valid;
  int64_t t = 0;
  unsigned char *raw = sm + kOffRaw + m * kRawPitch;
  if (row_ok) {
    t = __ldg(top + (int64_t)(i0 + m) * n_kv + h);
    const uint8_t *src = kp + t * row_bytes;
    for (int o = 16 * hf; o < row_bytes; o += 32) cp_async16(raw + o, src + o);
  }
  cp_async_commit();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp < 8) {
    // ---- A: half hf of chunk c's 64 codes of row m widened to fp16 in the MMA layout
    cp_async_wait<0>();
    bool stop = false;
    for (int c = 0; c < nch; ++c) {
      const int s = c % kStages;
      if (c >= kStages && !__all_sync(0xffffffffu, vp_wait(&empty[s], (unsigned)((c / kStages - 1) & 1), abort_s))) {
        if (lane == 0) {
          atomicOr(&g_vp_err, 1u);
          *abort_s = 1;
        }
        stop = true;
        break;
      }
      // rows past the selection: any codes (their output is not stored)
      const uint4 w4 = *reinterpret_cast<const uint4 *>(raw + c * (kK / 2) + 16 * hf);
      const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
      unsigned char *As = sm + s * kStageBytes + 4 * hf * kLboA + (m >> 3) * 128 + (m & 7) * 16;
#pragma unroll
      for (int kc = 0; kc < 4; ++kc) *reinterpret_cast<uint4 *>(As + kc * kLboA) = vp_codes8(ww[kc]);
      // generic-proxy writes -> visible to the tensor core (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&full_a[s])) : "memory");
    }
    // ---- epilogue: row m of the accumulator (TMEM lane m), channels ch0 + [32 hf, 32 hf + 32)
    bool ok = !stop && __all_sync(0xffffffffu, vp_wait(done, 0u, abort_s));
    if (!stop && !ok && lane == 0) {
      atomicOr(&g_vp_err, 1u);
      *abort_s = 1;
    }
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const float step = __fdiv_rn(__fmul_rn(2.0f, __ldg(vrs + h)), 4.0f);
      uint4 rc[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
      if (row_ok) {
        const uint4 *rr = reinterpret_cast<const uint4 *>(vr + (t * n_kv + h) * (kD / 4));
        rc[0] = __ldg(rr);
        rc[1] = __ldg(rr + 1);
      }
      const uint32_t rcw[8] = {rc[0].x, rc[0].y, rc[0].z, rc[0].w, rc[1].x, rc[1].y, rc[1].z, rc[1].w};
#pragma unroll
      for (int cb = hf; cb < hf + 1; ++cb) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(cb * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
              "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
              "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
              "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row_ok) {
          uint32_t packed[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float v2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int col = cb * 32 + e + u;
              const float pred = __fadd_rn(__fmul_rn(__uint_as_float(r[e + u]), us_s[col]), bs_s[col]);
              const int gc = ch0 + col;  // channel of the head
              const uint32_t byte = (rcw[gc >> 4] >> (8 * ((gc >> 2) & 3))) & 0xffu;
              const int code = (int)((byte >> (6 - 2 * (gc & 3))) & 3u) - 2;
              v2[u] = __fadd_rn(pred, __fmul_rn((float)code, step));
            }
            const __half2 hv = __floats2half2_rn(v2[0], v2[1]);
            packed[e / 2] = *reinterpret_cast<const uint32_t *>(&hv);
          }
          uint4 *dst = reinterpret_cast<uint4 *>(out + ((int64_t)(i0 + m) * n_kv + h) * kD + ch0 + cb * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  } else if (warp == 8) {
    // ---- W' chunks of head h (hi + lo, the MMA's shared-memory image)
    int last[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) last[s] = -1;
    if (lane == 0) {
      const unsigned char *wh = w3 + (int64_t)(2 * h + ch0 / kN) * nch * kBBytes;
      for (int c = 0; c < nch; ++c) {
        const int s = c % kStages;
        if (c >= kStages && !vp_wait(&empty[s], (unsigned)((c / kStages - 1) & 1), abort_s)) {
          atomicOr(&g_vp_err, 1u);
          *abort_s = 1;
          break;
        }
        mbar_expect_tx(&full_b[s], kBBytes);
        bulk_g2s(sm + s * kStageBytes + kABytes, wh + (int64_t)c * kBBytes, kBBytes, &full_b[s]);
        last[s] = c;
      }
      // copies in flight land before the CTA exits (normally all consumed)
      if (*abort_s)
        for (int s = 0; s < kStages; ++s)
          if (last[s] >= 0) vp_wait(&full_b[s], (unsigned)((last[s] / kStages) & 1), nullptr);
    }
    __syncwarp();
  } else {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t base = smem_u32(sm);
      int issued = 0;
      for (int c = 0; c < nch; ++c) {
        const int s = c % kStages;
        const unsigned ph = (unsigned)((c / kStages) & 1);
        if (!vp_wait(&full_a[s], ph, abort_s) || !vp_wait(&full_b[s], ph, abort_s)) {
          atomicOr(&g_vp_err, 1u);
          *abort_s = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_base = base + s * kStageBytes, b_base = a_base + kABytes;
#pragma unroll
        for (int ks = 0; ks < kK / 16; ++ks) {
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            const uint64_t da = vp_desc(a_base + ks * 2 * kLboA, kLboA, 128);
            const uint64_t db = vp_desc(b_base + part * kPartBytes + ks * 2 * kLboB, kLboB, 128);
            const uint32_t acc = (c > 0 || ks > 0 || part > 0) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
                "l"(da), "l"(db), "r"(kIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
                : "memory");
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&empty[s]))
                     : "memory");
        issued = c + 1;
      }
      // every MMA issued completes before `done` (also on an abort, so the
      // tensor memory is not freed under them)
      if (issued > 0)
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(done))
                     : "memory");
      if (*abort_s && issued > 0) vp_wait(done, 0u, nullptr);
    }
    __syncwarp();
  }
  __syncthreads();
  if (warp == 9) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// One CTA per output row r: W'[r, j] = W[r, j] * step[j], the row's power-of-two
// scale, the fp16 hi/lo split and the bias V_mean[r] - sum_j W[r, j] K_mean[j]
// (accumulated in fp64).  hi/lo are stored as the V-predict kernel's shared-
// memory image: per (head h, channel half, 64-wide chunk c) 16 KB =
// [part][8-element K chunk kc][channel n 0..63][8 halves].
__global__ void __launch_bounds__(256) vpredict_prepare_kernel(const float *__restrict__ W,
                                                               const float *__restrict__ kmean,
                                                               const float *__restrict__ vmean,
                                                               const float *__restrict__ kscales, int n_kv,
                                                               __half *__restrict__ w3, float *__restrict__ unscale,
                                                               float *__restrict__ bias) {
  constexpr int kD = vp::kD;
  __shared__ float red[8];
  __shared__ double redd[8];
  const int KD = n_kv * kD, nch = KD / vp::kK;
  const int r = blockIdx.x;
  const int h = r / kD, n = r - h * kD;
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
  for (int j = threadIdx.x; j < KD; j += blockDim.x) {
    const float step = __fdiv_rn(__fmul_rn(2.0f, __ldg(kscales + j)), 16.0f);
    const float x = __fmul_rn(__fmul_rn(__ldg(wr + j), step), sc);
    const __half xh = __float2half_rn(x);
    const int c = j / vp::kK, kc = (j % vp::kK) / 8, el = j % 8;
    const int nh = n / vp::kN, nl = n % vp::kN;
    const int64_t base = (((int64_t)((h * 2 + nh) * nch + c) * 2 * 8 + kc) * vp::kN + nl) * 8 + el;  // part 0
    w3[base] = xh;
    w3[base + 8 * vp::kN * 8] = __float2half_rn(__fsub_rn(x, __half2float(xh)));  // part 1
  }
}

}  // namespace kvr

using namespace kvr;

extern "C" size_t kvr_int4w_vpredict_weights_bytes(int n_kv, int d) {
  if (n_kv <= 0 || d != vp::kD) return 0;
  const size_t KD = (size_t)n_kv * d;
  return KD * 2 * KD * 2;  // hi + lo fp16 for every (output row, input) pair
}

extern "C" int kvr_int4w_vpredict_prepare(const float *W, const float *k_mean, const float *v_mean,
                                          const float *k_scales, int n_kv, int d, void *w3, float *unscale,
                                          float *bias, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == vp::kD, "kvr_int4w_vpredict_prepare: head_dim must be 128");
  KVR_REQUIRE(n_kv > 0 && n_kv <= 8, "kvr_int4w_vpredict_prepare: bad n_kv %d (1..8)", n_kv);
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
  KVR_REQUIRE(n_kv > 0 && n_kv <= 8 && k >= 0, "kvr_int4w_vpredict: bad sizes (n_kv 1..8)");
  KVR_REQUIRE(k_packed && top && w3 && unscale && bias && vr_packed && vr_scales && ret_v,
              "kvr_int4w_vpredict: null pointer");
  auto al = [](const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  KVR_REQUIRE(al(k_packed, 16) && al(w3, 16) && al(ret_v, 16) && al(vr_packed, 16),
              "kvr_int4w_vpredict: k_packed, w3, vr_packed and ret_v must be 16-byte aligned");
  if (k == 0) return KVR_OK;
  static thread_local int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaFuncSetAttribute(vpredict_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, vp::kSmem);
    attr_dev = dev;
  }
  dim3 grid((unsigned)((k + vp::kM - 1) / vp::kM), (unsigned)(2 * n_kv));
  vpredict_kernel<<<grid, vp::kThreads, vp::kSmem, as_cuda(stream)>>>(
      k_packed, top, count, k, n_kv, reinterpret_cast<const unsigned char *>(w3), unscale, bias, vr_packed,
      vr_scales, reinterpret_cast<__half *>(ret_v));
  return check_launch("kvr_int4w_vpredict");
}

extern "C" int kvr_int4w_vpredict_status(kvr_stream_t stream) {
  clear_error();
  unsigned flag = 0;
  cudaStream_t st = as_cuda(stream);
  if (cudaMemcpyFromSymbolAsync(&flag, g_vp_err, 4, 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return check_launch("kvr_int4w_vpredict_status");
  if (flag) {
    const unsigned zero = 0;
    cudaMemcpyToSymbolAsync(g_vp_err, &zero, 4, 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
    return set_error(KVR_ETIMEOUT, "kvr_int4w_vpredict: a bounded device-side wait gave up");
  }
  return KVR_OK;
}
