// Prefill-sized tile scoring on the 5th-generation tensor cores (tcgen05).
//
// For a block of prefill query positions (chunked prefill / multi-token
// decode over an existing sd1 store) every query must score every stored
// tile: S = Q' Khat^T with Q' the transformed GQA-group-mean queries and
// Khat the decoded keys s_c (2 bit - 1) in the transformed domain.  That is a
// dense contraction, so it runs as tcgen05.mma (kind::f16: fp16 operands,
// fp32 accumulate in tensor memory).  Khat is exact in fp16 (the scales are
// fp16 and the signs are exact); Q' is rounded to fp16 once.  Spec:
// oracle/sd1_ref.py prefill_tile_scores.
//
// Work split: a CTA owns 256 stored tokens (4 tiles of 64) of one KV head.
// It decodes them once into shared memory (B, 64 KB) and keeps them there
// while it walks over 128-query blocks of Q' (A, 32 KB each).  The prep
// kernel writes Q' already in the MMA's shared-memory layout, so each A block
// is ONE contiguous bulk copy (cp.async.bulk, local memory, no multicast)
// into a 4-deep ring.  Per block one thread issues 8 MMAs (M 128, N 256,
// K 16 each) into one of two 256-column TMEM accumulators; while the tensor
// core works on block i+1, the 8 warps read block i's accumulator back with
// tcgen05.ld and reduce every query row to the max over each 64-token tile.
//
// Operands sit in shared memory in the K-major, no-swizzle canonical layout:
// 8-row x 16-byte core matrices; SBO = 128 B between 8-row groups, LBO =
// (rows/8) * 128 B between 8-element K chunks; one MMA consumes K = 16 (two
// chunks).  Every wait is bounded; a timeout sets the error word, lets the
// copies and MMAs in flight drain and frees the tensor memory.
#include "kvr_common.cuh"
#include "kvr_transform.cuh"

namespace kvr {

constexpr int kPfM = 128;        // queries per block (MMA M)
constexpr int kPfN = 256;        // tokens per CTA (MMA N) = 4 tiles of 64
constexpr int kPfTile = 64;
constexpr int kPfThreads = 320;  // 8 reader warps + MMA warp + copy warp
constexpr uint32_t kPfLboA = (kPfM / 8) * 128;  // 2048 B
constexpr uint32_t kPfLboB = (kPfN / 8) * 128;  // 4096 B
constexpr int kPfSmemA = kPfM * kD * 2;         // 32 KB per A block
constexpr int kPfSmemB = kPfN * kD * 2;         // 64 KB
constexpr int kPfStages = 3;                    // A ring depth
constexpr int kPfOffA = 2 * kPfSmemB;           // two B buffers, then the A ring
constexpr int kPfOffLut = kPfOffA + kPfStages * kPfSmemA;
constexpr int kPfOffBar = kPfOffLut + 16 * 8;
constexpr int kPfSmem = kPfOffBar + 8 * (2 * kPfStages + 6) + 16;
constexpr uint32_t kPfTmemCols = 2 * kPfN;      // double-buffered accumulator

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

// Byte offset of (query m, 8-channel chunk kc) inside one A block.
__device__ __forceinline__ uint32_t pf_a_off(int m, int kc) {
  return (uint32_t)kc * kPfLboA + (uint32_t)(m >> 3) * 128 + (uint32_t)(m & 7) * 16;
}

// q (Nq, n_q, d) -> Q' fp16 in A-block layout: block (h, qb) is 32 KB at
// ((h * nqb + qb) * 32 KB); query rows past nq are zero.  A quad of lanes per
// row (lane t: elements 32t .. 32t+31): group mean in head order, then the
// transform in registers (quad DCT / 32-lane Hadamard), fp16 out.
template <int DTQ>
__global__ void __launch_bounds__(256) prefill_qprep_kernel(const void *__restrict__ q, int64_t nq, int n_q,
                                                            int n_kv, int kind, int64_t nqb,
                                                            unsigned char *__restrict__ qa) {
  __shared__ __align__(16) float qscr[8][8 * kD];  // quad scratch per warp
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = n_q / n_kv;
  const int64_t rows = nqb * kPfM * n_kv;
  if (kind == KVR_DCT) {
    const int t = lane & 3;
    for (int64_t r0 = ((int64_t)blockIdx.x * 8 + warp) * 8; r0 < rows; r0 += (int64_t)gridDim.x * 64) {
      const int64_t r = r0 + (lane >> 2);
      const int64_t i = r / n_kv;
      const int h = (int)(r - i * n_kv);
      float v[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = 0.0f;
      if (r < rows && i < nq) {
        const int64_t qb = (i * n_q + (int64_t)h * g) * kD + 32 * t;
#pragma unroll
        for (int c = 0; c < 8; ++c) load4<DTQ>(q, qb + 4 * c, *reinterpret_cast<float(*)[4]>(v + 4 * c));
        for (int k = 1; k < g; ++k) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float x4[4];
            load4<DTQ>(q, qb + (int64_t)k * kD + 4 * c, x4);
#pragma unroll
            for (int e = 0; e < 4; ++e) v[4 * c + e] = __fadd_rn(v[4 * c + e], x4[e]);
          }
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __fdiv_rn(v[e], (float)g);
      }
      dct128_fwd_quad(v, lane, qscr[warp]);  // all lanes (rows past the end carry zeros)
      if (r < rows) {
        const int64_t blk = (int64_t)h * nqb + i / kPfM;
        const int m = (int)(i % kPfM);
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 8-channel chunks 4t .. 4t+3
          __half2 hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) hv[e] = __floats2half2_rn(v[8 * c + 2 * e], v[8 * c + 2 * e + 1]);
          *reinterpret_cast<uint4 *>(qa + blk * kPfSmemA + pf_a_off(m, 4 * t + c)) = *reinterpret_cast<uint4 *>(hv);
        }
      }
    }
    return;
  }
  for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < rows; r += (int64_t)gridDim.x * 8) {
    const int64_t i = r / n_kv;
    const int h = (int)(r - i * n_kv);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (i < nq) {  // warp-uniform
      const int64_t qb = (i * n_q + (int64_t)h * g) * kD + lane * 4;
      load4<DTQ>(q, qb, acc);
      for (int k = 1; k < g; ++k) {
        float t[4];
        load4<DTQ>(q, qb + (int64_t)k * kD, t);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = __fadd_rn(acc[e], t[e]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = __fdiv_rn(acc[e], (float)g);
      wht128(acc, lane);
    }
    const int64_t blk = (int64_t)h * nqb + i / kPfM;
    const int m = (int)(i % kPfM);
    __half2 *dst = reinterpret_cast<__half2 *>(qa + blk * kPfSmemA + pf_a_off(m, lane >> 1) + (lane & 1) * 8);
    dst[0] = __floats2half2_rn(acc[0], acc[1]);
    dst[1] = __floats2half2_rn(acc[2], acc[3]);
  }
}

struct PrefillArgs {
  const unsigned char *qa;  // A blocks, (n_kv, nqb) x 32 KB
  int64_t nq, nqb;
  int n_kv;
  int64_t ntg, qsplit, items;  // token groups of 256, query splits, work items
  const uint32_t *kbits;
  const uint16_t *kscale;
  int64_t nt_cap, n_tiles;
  float *out;  // (Nq, n_kv, n_tiles)
  unsigned *err;
};

__device__ __forceinline__ bool pf_wait(uint64_t *bar, unsigned phase) {
  for (uint32_t it = 0; it < kSpinLimit; ++it)
    if (mbar_try_wait(bar, phase)) return true;
  return false;
}
// Same, but also gives up once another role has aborted.
__device__ __forceinline__ bool pf_wait_or_abort(uint64_t *bar, unsigned phase, volatile int *abort_s) {
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((it & 255u) == 255u && *abort_s) return false;
  }
  return false;
}

__device__ __forceinline__ void pf_mma_block(uint32_t tmem_d, uint32_t a_base, uint32_t b_base) {
#pragma unroll
  for (int s = 0; s < kD / 16; ++s) {
    const uint64_t da = umma_desc(a_base + s * 2 * kPfLboA, kPfLboA, 128);
    const uint64_t db = umma_desc(b_base + s * 2 * kPfLboB, kPfLboB, 128);
    const uint32_t acc = s > 0 ? 1u : 0u;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kPfIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
  }
}

__device__ __forceinline__ void pf_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void pf_tmem_ld32(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// max of 64 fp32 bit patterns (tree, exact)
__device__ __forceinline__ float pf_max64(const uint32_t *r) {
  float m[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) m[e] = __uint_as_float(r[e]);
#pragma unroll
  for (int e = 8; e < 64; ++e) m[e & 7] = fmaxf(m[e & 7], __uint_as_float(r[e]));
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

// Work item w = (head h, token group tg, query split y): the 256 stored
// tokens [256 tg, 256 tg + 256) of head h against query blocks y, y + qsplit,
// ...  A persistent grid (one CTA per SM) walks items w = blockIdx.x,
// blockIdx.x + gridDim.x, ...
struct PfItem {
  int h;
  int64_t t0, qb0, nblk;  // first tile, first query block, query blocks
};
__device__ __forceinline__ PfItem pf_item(const PrefillArgs &a, int64_t w) {
  PfItem it;
  const int64_t y = w % a.qsplit, r = w / a.qsplit;
  const int64_t tg = r % a.ntg;
  it.h = (int)(r / a.ntg);
  it.t0 = tg * (kPfN / kPfTile);
  it.qb0 = y;
  it.nblk = y < a.nqb ? (a.nqb - y + a.qsplit - 1) / a.qsplit : 0;
  return it;
}

// Decodes the 256 tokens of an item into B (fp16 +-s in the MMA layout); one
// token per reader thread (256 threads).
__device__ __forceinline__ void pf_decode_b(const PrefillArgs &a, const PfItem &it, unsigned char *Bs,
                                            const uint2 *lut, int tid) {
  const int n = tid;
  const int64_t tile = it.t0 + n / kPfTile;
  const int j = n % kPfTile;
  if (tile < a.n_tiles) {
    const int64_t tix = (int64_t)it.h * a.nt_cap + tile;  // batch 1: store row = head
    const uint4 w4 = __ldg(reinterpret_cast<const uint4 *>(a.kbits + (tix * kPfTile + j) * 4));
    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
    const uint4 *sc = reinterpret_cast<const uint4 *>(a.kscale + tix * kD);
#pragma unroll
    for (int kc = 0; kc < 16; ++kc) {
      const uint32_t byte = (ww[kc >> 2] >> ((kc & 3) * 8)) & 0xffu;
      const uint2 lo = lut[byte & 15u], hi = lut[byte >> 4];
      const uint4 sv = __ldg(sc + kc);
      *reinterpret_cast<uint4 *>(Bs + kc * kPfLboB + (n >> 3) * 128 + (n & 7) * 16) =
          make_uint4(sv.x ^ lo.x, sv.y ^ lo.y, sv.z ^ hi.x, sv.w ^ hi.y);
    }
  } else {
#pragma unroll
    for (int kc = 0; kc < 16; ++kc)
      *reinterpret_cast<uint4 *>(Bs + kc * kPfLboB + (n >> 3) * 128 + (n & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  // generic-proxy writes -> visible to the tensor core (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Roles: warps 0-7 decode B operands and read accumulators back (warp w: TMEM
// lanes 32(w%4).., columns 128(w/4)..); warp 8 lane 0 issues the MMAs; warp 9
// lane 0 streams the A blocks.  A stages and accumulators are used round-
// robin by a block counter that runs on across the CTA's items.  Barriers:
// afull[s] (copy landed), aempty[s] (MMAs reading stage s done, via
// tcgen05.commit), done[b] (accumulator b ready), tfree[b] (the 8 reader warps
// are through with accumulator b), bfull[k] (B buffer k decoded; count 8).
// A B buffer is rewritten only after the readers have seen every MMA of the
// item that used it complete.
__global__ void __launch_bounds__(kPfThreads, 1) prefill_scores_kernel(PrefillArgs a) {
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char *As = sm + kPfOffA;
  uint2 *lut = reinterpret_cast<uint2 *>(sm + kPfOffLut);  // nibble -> fp16 sign-flip masks
  uint64_t *afull = reinterpret_cast<uint64_t *>(sm + kPfOffBar);
  uint64_t *aempty = afull + kPfStages;
  uint64_t *done = aempty + kPfStages;
  uint64_t *tfree = done + 2;
  uint64_t *bfull = tfree + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bfull + 2);
  volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n_items = a.items;
  const int64_t w0 = blockIdx.x, wstep = gridDim.x;

  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kPfTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid < 16) {  // channel pair e of a nibble: bits 2e, 2e+1 -> halves 0/1 of word e
    const uint32_t nb = ~(uint32_t)tid;
    lut[tid] = make_uint2(((nb & 1u) << 15) | ((nb & 2u) << 30), ((nb & 4u) << 13) | ((nb & 8u) << 28));
  }
  if (tid == 9 * 32) {
    *abort_s = 0;
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&done[b], 1);
      mbar_init(&tfree[b], 8);
      mbar_init(&bfull[b], 8);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ---- producer: the A blocks of every item through the ring
    int64_t last[kPfStages];
#pragma unroll
    for (int s = 0; s < kPfStages; ++s) last[s] = -1;
    if (lane == 0) {
      int64_t j = 0;
      for (int64_t w = w0; w < n_items && !*abort_s; w += wstep) {
        const PfItem it = pf_item(a, w);
        const unsigned char *qa_h = a.qa + (int64_t)it.h * a.nqb * kPfSmemA;
        for (int64_t i = 0; i < it.nblk; ++i, ++j) {
          if (*abort_s) break;
          const int s = (int)(j % kPfStages);
          if (j >= kPfStages && !pf_wait_or_abort(&aempty[s], (unsigned)((j / kPfStages - 1) & 1), abort_s)) {
            atomicOr(a.err, 1u);
            *abort_s = 1;
            break;
          }
          mbar_expect_tx(&afull[s], kPfSmemA);
          bulk_g2s(As + s * kPfSmemA, qa_h + (it.qb0 + i * a.qsplit) * kPfSmemA, kPfSmemA, &afull[s]);
          last[s] = j;
        }
      }
    }
    __syncwarp();
    __syncthreads();  // end of work
    if (lane == 0 && *abort_s)  // copies in flight must land before the CTA exits
      for (int s = 0; s < kPfStages; ++s)
        if (last[s] >= 0) pf_wait(&afull[s], (unsigned)((last[s] / kPfStages) & 1));
  } else if (warp == 8) {
    // ---- MMA issuer
    int64_t issued = 0;
    if (lane == 0) {
      const uint32_t a_base = smem_u32(As), b_base0 = smem_u32(sm);
      int64_t i = 0;  // block counter across items
      int64_t k = 0;  // item counter of this CTA
      for (int64_t w = w0; w < n_items && !*abort_s; w += wstep, ++k) {
        const PfItem it = pf_item(a, w);
        const int bb = (int)(k & 1);
        if (!pf_wait_or_abort(&bfull[bb], (unsigned)((k >> 1) & 1), abort_s)) {
          atomicOr(a.err, 1u);
          *abort_s = 1;
          break;
        }
        const uint32_t b_base = b_base0 + bb * kPfSmemB;
        for (int64_t q = 0; q < it.nblk; ++q, ++i) {
          const int s = (int)(i % kPfStages), b = (int)(i & 1);
          bool ok = pf_wait_or_abort(&afull[s], (unsigned)((i / kPfStages) & 1), abort_s);
          if (ok && i >= 2) ok = pf_wait_or_abort(&tfree[b], (unsigned)((i / 2 - 1) & 1), abort_s);
          if (!ok) {
            atomicOr(a.err, 1u);
            *abort_s = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          pf_mma_block(tmem + (uint32_t)(b * kPfN), a_base + s * kPfSmemA, b_base);
          pf_commit(&done[b]);
          pf_commit(&aempty[s]);
          issued = i + 1;
        }
      }
      if (*abort_s && issued > 0)  // MMAs in flight must finish before TMEM is freed
        pf_wait(&done[(issued - 1) & 1], (unsigned)(((issued - 1) / 2) & 1));
    }
    __syncwarp();
    __syncthreads();
  } else {
    // ---- readers: decode B of item k+1 ahead, then read back item k
    const int quarter = warp & 3, half = warp >> 2;
    int64_t i = 0, k = 0;
    bool stop = false;
    if (w0 < n_items) {
      pf_decode_b(a, pf_item(a, w0), sm, lut, tid);
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bfull[0])) : "memory");
    }
    for (int64_t w = w0; w < n_items && !stop; w += wstep, ++k) {
      const PfItem it = pf_item(a, w);
      if (w + wstep < n_items) {  // next item's B into the other buffer: its last reader was item k-1
        pf_decode_b(a, pf_item(a, w + wstep), sm + ((k + 1) & 1) * kPfSmemB, lut, tid);
        __syncwarp();
        if (lane == 0)
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bfull[(k + 1) & 1])) : "memory");
      }
      const int nt_here = (int)(a.n_tiles - it.t0 < 4 ? a.n_tiles - it.t0 : 4);
      for (int64_t q = 0; q < it.nblk; ++q, ++i) {
        if (__shfl_sync(~0u, *abort_s, 0)) {
          stop = true;
          break;
        }
        const int b = (int)(i & 1);
        if (!__all_sync(~0u, pf_wait_or_abort(&done[b], (unsigned)((i >> 1) & 1), abort_s))) {
          if (lane == 0) atomicOr(a.err, 1u);
          *abort_s = 1;
          stop = true;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint32_t r[128];
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * kPfN + half * 128);
        pf_tmem_ld32(taddr, r);
        pf_tmem_ld32(taddr + 32, r + 32);
        pf_tmem_ld32(taddr + 64, r + 64);
        pf_tmem_ld32(taddr + 96, r + 96);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&tfree[b])) : "memory");
        const float best0 = pf_max64(r), best1 = pf_max64(r + 64);
        const int64_t qi = (it.qb0 + q * a.qsplit) * kPfM + quarter * 32 + lane;
        if (qi < a.nq) {
          float *o = a.out + (qi * a.n_kv + it.h) * a.n_tiles + it.t0 + half * 2;
          if (half * 2 < nt_here) o[0] = best0;
          if (half * 2 + 1 < nt_here) o[1] = best1;
        }
      }
    }
    __syncthreads();
  }

  // every role is past its last TMEM access (or drained after an abort)
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 8)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols));
}

}  // namespace kvr

using namespace kvr;

static int64_t pf_qblocks(int64_t nq) { return (nq + kPfM - 1) / kPfM; }

extern "C" size_t kvr_sd1_prefill_workspace_bytes(int64_t nq, int n_kv) {
  return kWsHeader + (size_t)pf_qblocks(nq) * n_kv * kPfSmemA;
}

extern "C" int kvr_sd1_prefill_scores(const void *q, int q_dtype, int64_t nq, int n_q, int n_kv,
                                      const uint32_t *kbits, const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles,
                                      int tile, int kind, float *scores, void *workspace, size_t workspace_bytes,
                                      kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(q && kbits && kscale && scores && workspace, "kvr_sd1_prefill_scores: null pointer");
  KVR_REQUIRE(valid_dtype(q_dtype), "kvr_sd1_prefill_scores: bad dtype");
  KVR_REQUIRE(nq >= 0 && n_kv > 0 && n_q > 0 && n_q % n_kv == 0, "kvr_sd1_prefill_scores: bad head counts");
  KVR_REQUIRE(n_kv <= 65535, "kvr_sd1_prefill_scores: too many KV heads");
  KVR_REQUIRE(tile == kPfTile, "kvr_sd1_prefill_scores: tile must be 64");
  KVR_REQUIRE(kind == KVR_HADAMARD || kind == KVR_DCT, "kvr_sd1_prefill_scores: unknown transform");
  KVR_REQUIRE(n_tiles >= 0 && n_tiles <= nt_cap, "kvr_sd1_prefill_scores: n_tiles > nt_cap");
  const size_t need = kvr_sd1_prefill_workspace_bytes(nq, n_kv);
  KVR_REQUIRE(workspace_bytes >= need, "kvr_sd1_prefill_scores: workspace %zu < %zu bytes", workspace_bytes, need);
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "kvr_sd1_prefill_scores: workspace alignment");
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(kscale) & 15) == 0 && (reinterpret_cast<uintptr_t>(kbits) & 15) == 0,
              "kvr_sd1_prefill_scores: kbits/kscale must be 16-byte aligned");
  if (nq == 0 || n_tiles == 0) return KVR_OK;
  cudaStream_t st = as_cuda(stream);
  char *p = reinterpret_cast<char *>(workspace);
  unsigned char *qa = reinterpret_cast<unsigned char *>(p + kWsHeader);
  const int64_t nqb = pf_qblocks(nq);
  const int64_t rows = nqb * kPfM * n_kv;
  const int64_t per_cta = kind == KVR_DCT ? 64 : 8;  // rows per CTA per pass
  const int qgrid = (int)((rows + per_cta - 1) / per_cta < 148 * 8 ? (rows + per_cta - 1) / per_cta : 148 * 8);
  if (q_dtype == KVR_F32) prefill_qprep_kernel<KVR_F32><<<qgrid, 256, 0, st>>>(q, nq, n_q, n_kv, kind, nqb, qa);
  else if (q_dtype == KVR_F16) prefill_qprep_kernel<KVR_F16><<<qgrid, 256, 0, st>>>(q, nq, n_q, n_kv, kind, nqb, qa);
  else prefill_qprep_kernel<KVR_BF16><<<qgrid, 256, 0, st>>>(q, nq, n_q, n_kv, kind, nqb, qa);
  int rc = check_launch("kvr_sd1_prefill_scores (q prep)");
  if (rc) return rc;
  // work items: (head, 256-token group, query split); query blocks are split
  // only when the items alone would leave SMs idle (each split re-decodes B)
  const int64_t ntg = (n_tiles + 3) / 4;
  int64_t qsplit = (148 + ntg * n_kv - 1) / (ntg * n_kv);
  qsplit = qsplit < 1 ? 1 : (qsplit > nqb ? nqb : qsplit);
  const int64_t items = ntg * n_kv * qsplit;
  PrefillArgs a{qa, nq, nqb, n_kv, ntg, qsplit, items, kbits, kscale, nt_cap, n_tiles, scores,
                reinterpret_cast<unsigned *>(p)};
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaFuncSetAttribute(prefill_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
    set_dev = dev;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ctas = items < sms ? items : sms;  // persistent: one CTA per SM
  prefill_scores_kernel<<<(unsigned)ctas, kPfThreads, kPfSmem, st>>>(a);
  return check_launch("kvr_sd1_prefill_scores");
}
