// Prefill-sized tile scoring on the 5th-generation tensor cores (tcgen05).
//
// For a block of prefill query positions (chunked prefill / multi-token
// decode over an existing sd1 store) every query must score every stored
// tile: S = Q' Khat^T with Q' the transformed GQA-group-mean queries and
// Khat the decoded keys s_c (2 bit - 1) in the transformed domain.  That is a
// dense contraction (M = 128 queries, N = 256 tokens, K = 128 channels per
// CTA), so it runs as tcgen05.mma (kind::f16: fp16 operands, fp32 accumulate
// in tensor memory).  Khat is exact in fp16 (the scales are fp16 and the
// signs are exact); Q' is rounded to fp16 once.  The epilogue reads the
// accumulator back with tcgen05.ld and reduces each query's row to the max
// over each 64-token tile.  Spec: oracle/sd1_ref.py prefill_tile_scores.
//
// Operands sit in shared memory in the K-major, no-swizzle canonical layout:
// 8-row x 16-byte core matrices; SBO = 128 B between 8-row groups, LBO =
// (rows/8) * 128 B between 8-element K chunks; one MMA consumes K = 16 (two
// chunks), so K = 128 takes 8 MMAs issued by one thread.  This file is used by
// single-GPU calls only and its copies read local memory (no multicast).
#include "kvr_common.cuh"
#include "kvr_transform.cuh"

namespace kvr {

constexpr int kPfM = 128;       // queries per CTA (MMA M)
constexpr int kPfN = 256;       // tokens per CTA (MMA N) = 4 tiles of 64
constexpr int kPfTile = 64;
constexpr int kPfThreads = 128;  // 4 warps: one per TMEM lane quarter
constexpr uint32_t kPfLboA = (kPfM / 8) * 128;  // 2048 B
constexpr uint32_t kPfLboB = (kPfN / 8) * 128;  // 4096 B
constexpr int kPfSmemA = kPfM * kD * 2;         // 32 KB
constexpr int kPfSmemB = kPfN * kD * 2;         // 64 KB

// sm100 shared-memory matrix descriptor, K-major, no swizzle
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)((lbo >> 4) & 0x3fffu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fffu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
  return d;                // base offset 0, legacy LBO mode, layout type 0 (no swizzle)
}

// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, N, M.
constexpr uint32_t kPfIdesc = (1u << 4)                      // D format: F32
                              | (0u << 7) | (0u << 10)         // A, B: F16
                              | ((uint32_t)(kPfN >> 3) << 17)  // N / 8
                              | ((uint32_t)(kPfM >> 4) << 24); // M / 16

// q (Nq, n_q, d) -> qp16 (Nq, n_kv, d) fp16: group mean, transform, round.
template <int DTQ>
__global__ void __launch_bounds__(256) prefill_qprep_kernel(const void *__restrict__ q, int64_t nq, int n_q,
                                                            int n_kv, int kind, __half *__restrict__ qp16) {
  __shared__ float lee_s[kD];
  __shared__ __align__(16) float buf_s[8][2 * kD];
  load_lee(lee_s);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = n_q / n_kv;
  const int64_t rows = nq * n_kv;
  for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < rows; r += (int64_t)gridDim.x * 8) {
    const int64_t i = r / n_kv;
    const int h = (int)(r - i * n_kv);
    const int64_t qb = (i * n_q + (int64_t)h * g) * kD + lane * 4;
    float acc[4];
    load4<DTQ>(q, qb, acc);
    for (int k = 1; k < g; ++k) {
      float t[4];
      load4<DTQ>(q, qb + (int64_t)k * kD, t);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = __fadd_rn(acc[e], t[e]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = __fdiv_rn(acc[e], (float)g);
    transform128(acc, lane, kind, false, buf_s[warp], lee_s);
    __half2 *dst = reinterpret_cast<__half2 *>(qp16 + r * kD + lane * 4);
    dst[0] = __floats2half2_rn(acc[0], acc[1]);
    dst[1] = __floats2half2_rn(acc[2], acc[3]);
  }
}

struct PrefillArgs {
  const __half *qp16;  // (Nq, n_kv, d)
  int64_t nq;
  int n_kv;
  const uint32_t *kbits;
  const uint16_t *kscale;
  int64_t nt_cap, n_tiles;
  float *out;  // (Nq, n_kv, n_tiles)
  unsigned *err;
};

__global__ void __launch_bounds__(kPfThreads, 1) prefill_scores_kernel(PrefillArgs a) {
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char *As = sm;                 // [16 kc][16 mg][8 r][16 B]
  unsigned char *Bs = sm + kPfSmemA;      // [16 kc][32 ng][8 r][16 B]
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm + kPfSmemA + kPfSmemB);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kPfSmemA + kPfSmemB + 16);
  int *ok_s = reinterpret_cast<int *>(sm + kPfSmemA + kPfSmemB + 32);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.z;
  const int64_t q0 = (int64_t)blockIdx.y * kPfM;
  const int64_t t0 = (int64_t)blockIdx.x * (kPfN / kPfTile);  // first tile of this CTA
  const int64_t row = h;                                      // batch 1: store row = head

  // ---- TMEM accumulator: 256 fp32 columns x 128 lanes
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kPfN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    ok_s[0] = 1;
    mbar_init(bar, 1);
  }

  // ---- A: 128 queries x 128 channels fp16 (rows past nq are zero)
  for (int i = tid; i < kPfM * (kD / 8); i += kPfThreads) {
    const int m = i >> 4, kc = i & 15;  // 16-byte chunk (8 channels) of query m
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (q0 + m < a.nq) v = __ldg(reinterpret_cast<const uint4 *>(a.qp16 + ((q0 + m) * a.n_kv + h) * kD + kc * 8));
    *reinterpret_cast<uint4 *>(As + kc * kPfLboA + (m >> 3) * 128 + (m & 7) * 16) = v;
  }
  // ---- B: 256 tokens x 128 channels, k_hat = +-s (fp16, exact)
  for (int i = tid; i < kPfN * (kD / 8); i += kPfThreads) {
    const int n = i >> 4, kc = i & 15;
    const int64_t tile = t0 + n / kPfTile;
    const int j = n % kPfTile;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (tile < a.n_tiles) {
      const int64_t tix = row * a.nt_cap + tile;
      const uint32_t w = __ldg(a.kbits + (tix * kPfTile + j) * 4 + (kc >> 2));
      const uint4 s = __ldg(reinterpret_cast<const uint4 *>(a.kscale + tix * kD + kc * 8));
      const uint32_t sw[4] = {s.x, s.y, s.z, s.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c0 = kc * 8 + 2 * e;  // channels c0, c0 + 1
        uint32_t lo = sw[e] & 0xffffu, hi = sw[e] >> 16;
        if (!((w >> (c0 & 31)) & 1u)) lo ^= 0x8000u;        // sign bit 0 -> -s
        if (!((w >> ((c0 + 1) & 31)) & 1u)) hi ^= 0x8000u;
        o[e] = lo | (hi << 16);
      }
      v = make_uint4(o[0], o[1], o[2], o[3]);
    }
    *reinterpret_cast<uint4 *>(Bs + kc * kPfLboB + (n >> 3) * 128 + (n & 7) * 16) = v;
  }
  // generic-proxy smem writes -> visible to the tensor core (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // ---- 8 MMAs over K = 128, issued by one thread
  if (tid == 0) {
    const uint32_t a_base = smem_u32(As), b_base = smem_u32(Bs);
#pragma unroll
    for (int s = 0; s < kD / 16; ++s) {
      const uint64_t da = umma_desc(a_base + s * 2 * kPfLboA, kPfLboA, 128);
      const uint64_t db = umma_desc(b_base + s * 2 * kPfLboB, kPfLboB, 128);
      const uint32_t acc = s > 0 ? 1u : 0u;
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
          "l"(da), "l"(db), "r"(kPfIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
          : "memory");
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
  }
  if (!mbar_wait_bounded(bar, 0)) {
    atomicOr(a.err, 1u);
    ok_s[0] = 0;
    mbar_wait_bounded(bar, 0);  // let MMAs in flight finish before TMEM is freed
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();

  // ---- epilogue: warp w reads TMEM lanes 32w..32w+31 (its queries)
  const int64_t qi = q0 + warp * 32 + lane;
  if (ok_s[0]) {
    float best[kPfN / kPfTile];
#pragma unroll
    for (int t = 0; t < kPfN / kPfTile; ++t) best[t] = -INFINITY;
#pragma unroll
    for (int c0 = 0; c0 < kPfN; c0 += 16) {
      uint32_t r[16];
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
          "%15}, [%16];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
            "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int e = 0; e < 16; ++e) best[c0 / kPfTile] = fmaxf(best[c0 / kPfTile], __uint_as_float(r[e]));
    }
    if (qi < a.nq) {
#pragma unroll
      for (int t = 0; t < kPfN / kPfTile; ++t)
        if (t0 + t < a.n_tiles) a.out[(qi * a.n_kv + h) * a.n_tiles + t0 + t] = best[t];
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfN));
}

}  // namespace kvr

using namespace kvr;

extern "C" size_t kvr_sd1_prefill_workspace_bytes(int64_t nq, int n_kv) {
  return kWsHeader + align_up((size_t)nq * n_kv * kD * 2, 256);
}

extern "C" int kvr_sd1_prefill_scores(const void *q, int q_dtype, int64_t nq, int n_q, int n_kv,
                                      const uint32_t *kbits, const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles,
                                      int tile, int kind, float *scores, void *workspace, size_t workspace_bytes,
                                      kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(q && kbits && kscale && scores && workspace, "kvr_sd1_prefill_scores: null pointer");
  KVR_REQUIRE(valid_dtype(q_dtype), "kvr_sd1_prefill_scores: bad dtype");
  KVR_REQUIRE(nq >= 0 && n_kv > 0 && n_q > 0 && n_q % n_kv == 0, "kvr_sd1_prefill_scores: bad head counts");
  KVR_REQUIRE(tile == kPfTile, "kvr_sd1_prefill_scores: tile must be 64");
  KVR_REQUIRE(kind == KVR_HADAMARD || kind == KVR_DCT, "kvr_sd1_prefill_scores: unknown transform");
  KVR_REQUIRE(n_tiles >= 0 && n_tiles <= nt_cap, "kvr_sd1_prefill_scores: n_tiles > nt_cap");
  const size_t need = kvr_sd1_prefill_workspace_bytes(nq, n_kv);
  KVR_REQUIRE(workspace_bytes >= need, "kvr_sd1_prefill_scores: workspace %zu < %zu bytes", workspace_bytes, need);
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "kvr_sd1_prefill_scores: workspace alignment");
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(kscale) & 15) == 0, "kvr_sd1_prefill_scores: kscale must be 16-byte aligned");
  if (nq == 0 || n_tiles == 0) return KVR_OK;
  cudaStream_t st = as_cuda(stream);
  char *p = reinterpret_cast<char *>(workspace);
  __half *qp16 = reinterpret_cast<__half *>(p + kWsHeader);
  const int64_t rows = nq * n_kv;
  const int qb = (int)((rows + 7) / 8 < 148 * 16 ? (rows + 7) / 8 : 148 * 16);
  if (q_dtype == KVR_F32) prefill_qprep_kernel<KVR_F32><<<qb, 256, 0, st>>>(q, nq, n_q, n_kv, kind, qp16);
  else if (q_dtype == KVR_F16) prefill_qprep_kernel<KVR_F16><<<qb, 256, 0, st>>>(q, nq, n_q, n_kv, kind, qp16);
  else prefill_qprep_kernel<KVR_BF16><<<qb, 256, 0, st>>>(q, nq, n_q, n_kv, kind, qp16);
  int rc = check_launch("kvr_sd1_prefill_scores (q prep)");
  if (rc) return rc;
  PrefillArgs a{qp16, nq, n_kv, kbits, kscale, nt_cap, n_tiles, scores, reinterpret_cast<unsigned *>(p)};
  const size_t smem = kPfSmemA + kPfSmemB + 64;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaFuncSetAttribute(prefill_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    set_dev = dev;
  }
  dim3 grid((unsigned)((n_tiles + 3) / 4), (unsigned)((nq + kPfM - 1) / kPfM), n_kv);
  prefill_scores_kernel<<<grid, kPfThreads, smem, st>>>(a);
  return check_launch("kvr_sd1_prefill_scores");
}
