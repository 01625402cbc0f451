// sd1 1-bit codec: encoder, tile scoring + selection, tile decode (sm_100a).
//
// The codec has no counterpart in the reference (which stores int4 K and int2
// V residuals, modules/kvr_retrieval.py:2-4); its specification is the CPU
// statement in oracle/sd1_ref.py, which these kernels match bit for bit for
// the packed bits, the fp16 scales and the tile scores.  Selection follows the
// reference's design: the GQA-group mean of the post-RoPE query scores fixed
// tiles (modules/kvr_retrieval.py:270, 291-315) and a per-KV-head top-k keeps
// the best ones (modules/kvr_retrieval.py:370-392).
#include <cstdlib>
#include <cstring>
#include <utility>
#include <vector>

#include "kvr_common.cuh"
#include "kvr_sd1_score.cuh"
#include "kvr_topk.cuh"
#include "kvr_transform.cuh"

namespace kvr {

// ------------------------------------------------------------ transform ----
__global__ void __launch_bounds__(256) transform_kernel(const float *x, float *y, int64_t rows, int kind,
                                                        int inverse) {
  __shared__ float lee_s[kD];
  __shared__ __align__(16) float buf_s[8][2 * kD];
  load_lee(lee_s);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (kind == KVR_DCT) {
    // quad form: each warp transforms 8 rows at a time
    __shared__ __align__(16) float qscr[8][8 * kD];
    for (int64_t r0 = ((int64_t)blockIdx.x * 8 + warp) * 8; r0 < rows; r0 += (int64_t)gridDim.x * 64) {
      const int64_t r = r0 + (lane >> 2);
      const int t = lane & 3;
      float v[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 a = r < rows ? reinterpret_cast<const float4 *>(x + r * kD + 32 * t)[i]
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
      }
      if (inverse) dct128_inv_quad(v, lane, qscr[warp]);
      else dct128_fwd_quad(v, lane, qscr[warp]);
      if (r < rows)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          reinterpret_cast<float4 *>(y + r * kD + 32 * t)[i] =
              make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    return;
  }
  for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < rows; r += (int64_t)gridDim.x * 8) {
    float v[4];
    float4 t = reinterpret_cast<const float4 *>(x + r * kD)[lane];
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    transform128(v, lane, kind, inverse != 0, buf_s[warp], lee_s);
    reinterpret_cast<float4 *>(y + r * kD)[lane] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// -------------------------------------------------------------- encoder ----
// One CTA of 2*TILE threads per (tile, kv head, batch).  Phase 1: each
// thread owns one token vector (threads < TILE: K, the rest: V), holds all
// 128 elements in registers, applies RoPE to K when tables are given, runs
// the transform with compile-time indices (no shuffles, no shared memory),
// and writes the result channel-major into X[kv][c][j].  Phase 2: one thread
// per (kv, channel) chain reads its channel's TILE values as float4 runs,
// forms the fp16 scale and runs the sigma-delta scan; a token's bits come out
// of a warp ballot (a warp covers channels 32w'..32w'+31 = one word).
template <int DT, int TILE>
__global__ void __launch_bounds__(2 * TILE) sd1_encode_kernel(
    const void *__restrict__ k, const void *__restrict__ v, int n_kv, int64_t batch_stride,
    int64_t tok_stride, const float *__restrict__ cos_tbl, const float *__restrict__ sin_tbl,
    int64_t rope_stride, int64_t pos0, int kind, uint32_t *__restrict__ kbits, uint16_t *__restrict__ kscale,
    uint32_t *__restrict__ vbits, uint16_t *__restrict__ vscale, int64_t nt_cap, int64_t tile0, int vec16) {
  constexpr int NT = 2 * TILE;    // one thread per token vector (K: tid < TILE, V: tid >= TILE)
  constexpr int LD = TILE + 4;    // channel-major row stride: conflict-free both ways
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float *X = reinterpret_cast<float *>(smem_raw);  // [2][128][LD]: X[kv][c][j]
  __shared__ __align__(16) uint32_t bits_s[2 * TILE * 4];

  const int tid = threadIdx.x, lane = tid & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t tile_in = blockIdx.x;
  const int kv = tid / TILE, j = tid % TILE;  // warp-uniform kv (TILE is a multiple of 32)
  const int64_t tok = tile_in * TILE + j;

  // ---- phase 1a: stage the tile's 2*TILE rows (and the RoPE rows) into
  // shared memory with coalesced asynchronous copies; the staging area
  // aliases X and is released by the barrier before X is written
  constexpr int ES = DT == KVR_F32 ? 4 : 2;
  constexpr int RB = kD * ES;          // row bytes
  constexpr int RS = RB + 16;          // padded row stride: conflict-free row reads
  constexpr int CS = kD * 4 + 16;      // RoPE row stride
  unsigned char *raw = smem_raw;                      // [2*TILE][RS]
  unsigned char *cs_s = smem_raw + 2 * TILE * RS;     // [2][TILE][CS] cos, sin
  const bool rope = cos_tbl != nullptr;
  {
    const int64_t base = (int64_t)b * batch_stride + (int64_t)h * kD + tile_in * TILE * tok_stride;
    const unsigned char *kp = reinterpret_cast<const unsigned char *>(k) + base * ES;
    const unsigned char *vp = reinterpret_cast<const unsigned char *>(v) + base * ES;
    const int64_t tsb = tok_stride * ES;
    if (vec16) {
      constexpr int CPR = RB / 16;
      for (int i = tid; i < 2 * TILE * CPR; i += NT) {
        const int r = i / CPR, c = i % CPR;
        const unsigned char *src = (r < TILE ? kp + r * tsb : vp + (r - TILE) * tsb) + c * 16;
        cp_async16(raw + r * RS + c * 16, src);
      }
      if (rope) {
        constexpr int CPC = kD * 4 / 16;
        for (int i = tid; i < 2 * TILE * CPC; i += NT) {
          const int r = i / CPC, c = i % CPC;
          const int jj = r % TILE;
          const float *tbl = r < TILE ? cos_tbl : sin_tbl;
          cp_async16(cs_s + r * CS + c * 16, tbl + (pos0 + tile_in * TILE + jj) * rope_stride + c * 4);
        }
      }
    } else {
      constexpr int CPR = RB / 8;
      for (int i = tid; i < 2 * TILE * CPR; i += NT) {
        const int r = i / CPR, c = i % CPR;
        const unsigned char *src = (r < TILE ? kp + r * tsb : vp + (r - TILE) * tsb) + c * 8;
        cp_async8(raw + r * RS + c * 8, src);
      }
      if (rope) {
        constexpr int CPC = kD * 4 / 8;
        for (int i = tid; i < 2 * TILE * CPC; i += NT) {
          const int r = i / CPC, c = i % CPC;
          const int jj = r % TILE;
          const float *tbl = r < TILE ? cos_tbl : sin_tbl;
          cp_async8(cs_s + r * CS + c * 8, tbl + (pos0 + tile_in * TILE + jj) * rope_stride + c * 2);
        }
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
  }
  __syncthreads();

  // ---- phase 1b: this thread's vector from shared memory, RoPE (K), transform
  {
    float x[kD];
    const uint4 *row = reinterpret_cast<const uint4 *>(raw + tid * RS);
#pragma unroll
    for (int q = 0; q < RB / 16; ++q) {
      const uint4 u = row[q];
      if constexpr (DT == KVR_F32) {
        x[4 * q] = __uint_as_float(u.x); x[4 * q + 1] = __uint_as_float(u.y);
        x[4 * q + 2] = __uint_as_float(u.z); x[4 * q + 3] = __uint_as_float(u.w);
      } else {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint16_t lo = w[e] & 0xffffu, hi = w[e] >> 16;
          if constexpr (DT == KVR_F16) {
            x[8 * q + 2 * e] = __half2float(__ushort_as_half(lo));
            x[8 * q + 2 * e + 1] = __half2float(__ushort_as_half(hi));
          } else {
            x[8 * q + 2 * e] = __bfloat162float(__ushort_as_bfloat16(lo));
            x[8 * q + 2 * e + 1] = __bfloat162float(__ushort_as_bfloat16(hi));
          }
        }
      }
    }
    if (rope && kv == 0) {
      // (x * cos) + (rotate_half(x) * sin), rotate_half(x)_i = -x_{i+64} (i < 64), x_{i-64}
      const float4 *cr = reinterpret_cast<const float4 *>(cs_s + j * CS);
      const float4 *sr = reinterpret_cast<const float4 *>(cs_s + (TILE + j) * CS);
      float y[kD];
#pragma unroll
      for (int q = 0; q < kD / 4; ++q) {
        const float4 c4 = cr[q], s4 = sr[q];
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 4 * q + e;
          const float rh = i < kD / 2 ? -x[i + kD / 2] : x[i - kD / 2];
          y[i] = __fadd_rn(__fmul_rn(x[i], cc[e]), __fmul_rn(rh, ss[e]));
        }
      }
#pragma unroll
      for (int i = 0; i < kD; ++i) x[i] = y[i];
    }
    __syncthreads();  // staging area is read: X may overwrite it
    if (kind == KVR_HADAMARD) wht128_reg(x);
    else dct128_fwd_reg(x);
    float *xo = X + (kv * kD) * LD + j;
#pragma unroll
    for (int c = 0; c < kD; ++c) xo[c * LD] = x[c];
  }
  __syncthreads();

  // ---- phase 2: per channel chain (kv, c): scale = fp16(mean |x|), sigma-delta bits.
  // A thread's CPT chains (tid + i * NT) are independent: they advance together,
  // so their dependent sigma-delta steps overlap.
  const int64_t out_tile = ((int64_t)b * n_kv + h) * nt_cap + tile0 + tile_in;
  constexpr int CPT = 2 * kD / NT;  // chains per thread: 4, 2, 1 for tiles of 32, 64, 128
  const float4 *Xc[CPT];
  uint32_t *bs[CPT];
  float s_[CPT], ns_[CPT], e_[CPT];
  uint32_t mine[CPT];  // lane L keeps the word of token 32m + L
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int chain = tid + i * NT;
    const int kvc = chain / kD, c = chain % kD;  // a warp covers 32 consecutive channels of one kv
    Xc[i] = reinterpret_cast<const float4 *>(X + (kvc * kD + c) * LD);
    bs[i] = bits_s + kvc * TILE * 4 + (c >> 5);
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < TILE / 4; ++q) {
      const float4 t = Xc[i][q];
      acc = __fadd_rn(acc, fabsf(t.x));
      acc = __fadd_rn(acc, fabsf(t.y));
      acc = __fadd_rn(acc, fabsf(t.z));
      acc = __fadd_rn(acc, fabsf(t.w));
    }
    const float mean = __fmul_rn(acc, 1.0f / TILE);
    const __half s16 = __float2half_rn(fminf(mean, 65504.0f));
    s_[i] = __half2float(s16);
    ns_[i] = -s_[i];
    e_[i] = 0.0f;
    mine[i] = 0u;
    (kvc == 0 ? kscale : vscale)[out_tile * kD + c] = __half_as_ushort(s16);
  }
#pragma unroll
  for (int q = 0; q < TILE / 4; ++q) {
    float tv[CPT][4];
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const float4 t = Xc[i][q];
      tv[i][0] = t.x; tv[i][1] = t.y; tv[i][2] = t.z; tv[i][3] = t.w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int j = 4 * q + r;
#pragma unroll
      for (int i = 0; i < CPT; ++i) {
        const float u = __fadd_rn(tv[i][r], e_[i]);
        const bool bit = u >= 0.0f;
        e_[i] = __fsub_rn(u, bit ? s_[i] : ns_[i]);
        const uint32_t w = __ballot_sync(0xffffffffu, bit);
        mine[i] = lane == (j & 31) ? w : mine[i];
        if ((j & 31) == 31) bs[i][(j - 31 + lane) * 4] = mine[i];
      }
    }
  }
  __syncthreads();
  // ---- store bits: 2 * TILE uint4 (token-major)
  for (int i = tid; i < 2 * TILE; i += NT) {
    const int kvi = i / TILE, jj = i - kvi * TILE;
    const uint4 w = reinterpret_cast<const uint4 *>(bits_s)[i];
    uint32_t *dst = (kvi == 0 ? kbits : vbits) + (out_tile * TILE + jj) * 4;
    *reinterpret_cast<uint4 *>(dst) = w;
  }
}

// ---------------------------------------------------------- tile scores ----
// One CTA (256 threads, 8 warps) covers 16 consecutive tiles of one (b, h);
// each warp scores 2 tiles.  Warp 0 first forms q' = T(mean of the group's
// query heads).  Per tile: w_c = q'_c * s_c, M = max|w|, wq = rint(w*127/M),
// bit planes of wq via ballots, S_j = 2*sum_c wq_c*bit_jc - sum wq from
// popcounts, score = float(max_j S_j) * (M/127).  With `select` set, the
// last CTA of each (b, h) to finish runs the block top-k over that row.
constexpr int kScoreTilesPerCta = 16;
constexpr int64_t kSelectSmemScores = 8192;  // rows up to this many tiles are selected from shared memory

__host__ __device__ inline size_t select_cand_bytes(int k_sel) {
  int P = 1;
  while (P < k_sel) P <<= 1;
  return align_up((size_t)P * 8, 16);
}

struct SelectArgs {
  int k_sel;
  int64_t ex_t0, ex_t1, tile_base;
  int32_t *sel;         // (B, n_kv, k_sel)
  float *sel_scores;    // (B, n_kv, k_sel) or null
  unsigned *counters;   // (B, n_kv), zero on entry, reset on exit
  const uint32_t *vbits;   // optional: V data of the scanned tiles is
  const uint16_t *vscale;  // prefetched into L2 for the attention kernel
  RowPrefetch rows;        // optional (k[s] null = none): exact rows prefetched into L2
  unsigned *err;           // the workspace's error word (bounded waits that gave up)
};


// Selection of one (b, h) row by the whole block (NT threads): the k_sel
// largest scores outside [ex_t0, ex_t1) as unique keys (score desc, index
// asc), written as indices + tile_base; -1 past the row's tile count.
template <int NT>
__device__ void select_row(const float *scores, int64_t row, int64_t n_tiles, const SelectArgs &sa,
                           unsigned char *dyn_smem) {
  TopkSmem &tsm = *reinterpret_cast<TopkSmem *>(dyn_smem);
  unsigned long long *cand = reinterpret_cast<unsigned long long *>(dyn_smem + align_up(sizeof(TopkSmem), 16));
  const float *srow = scores + row * n_tiles;
  const int64_t ex0 = sa.ex_t0, ex1 = sa.ex_t1;
  const int kk = (int)(n_tiles < sa.k_sel ? n_tiles : sa.k_sel);
  if (kk > 0) {
    if (n_tiles <= kSelectSmemScores) {
      // one pass over L2 into shared memory; the radix passes then stay on chip
      float *row_s = reinterpret_cast<float *>(dyn_smem + align_up(sizeof(TopkSmem), 16) + select_cand_bytes(sa.k_sel));
      for (int64_t i = threadIdx.x; i < n_tiles; i += NT)
        row_s[i] = (i >= ex0 && i < ex1) ? -INFINITY : __ldcg(srow + i);
      __syncthreads();
      if (kk <= 32) {
        unsigned long long *lists = tsm.lists;
        block_topk_warp32<NT>(row_s, n_tiles, kk, lists, cand);
      } else {
        block_topk<NT>([&](int64_t i) -> float { return row_s[i]; }, n_tiles, kk, cand, tsm);
      }
    } else {
      block_topk<NT>(
          [&](int64_t i) -> float { return (i >= ex0 && i < ex1) ? -INFINITY : __ldcg(srow + i); }, n_tiles, kk,
          cand, tsm);
    }
  }
  for (int j = threadIdx.x; j < sa.k_sel; j += NT) {
    const bool ok = j < kk;
    sa.sel[row * sa.k_sel + j] = ok ? (int32_t)(key_index(cand[j]) + sa.tile_base) : -1;
    if (sa.sel_scores) sa.sel_scores[row * sa.k_sel + j] = ok ? key_score(cand[j]) : -INFINITY;
  }
}

template <int DTQ, int TILE>
__global__ void __launch_bounds__(256) sd1_score_kernel(
    const void *__restrict__ q, int n_q, int n_kv, const uint32_t *__restrict__ kbits,
    const uint16_t *__restrict__ kscale, int64_t nt_cap, int64_t n_tiles, int kind,
    float *__restrict__ scores /* (B, n_kv, n_tiles) */, float *__restrict__ qprime /* (B, n_q, d) or null */,
    SelectArgs sa, int do_select, int64_t tpc) {
  __shared__ float lee_s[kD];
  __shared__ __align__(16) float buf_s[8][2 * kD];
  __shared__ __align__(16) float qp_s[kD];
  __shared__ int last_s;
  extern __shared__ __align__(16) unsigned char dyn_smem[];

  KVR_TRACE_POINT(0, 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = blockIdx.y, b = blockIdx.z;
  const int g = n_q / n_kv;
  const int64_t row = (int64_t)b * n_kv + h;
  load_lee(lee_s);

  // Each CTA owns tiles [blockIdx.x * tpc, +tpc) of its row; warp w scores
  // the pairs w, w + 8, ... of that range.  The first pair is loaded while q'
  // is formed, and every later pair is loaded before the current one is
  // scored (software pipeline in registers).
  constexpr int TPL = TILE / 32;  // tokens per lane
  const int64_t cta_t0 = (int64_t)blockIdx.x * tpc;
  const int64_t cta_t1 = min(n_tiles, cta_t0 + tpc);
  uint4 kb[2][TPL];
  uint16_t ks[2][4];
  auto load_pair = [&](int64_t t_first, uint4 (&kbd)[2][TPL], uint16_t (&ksd)[2][4]) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t t = min(t_first + u, cta_t1 - 1);  // a lone last tile is scored twice, stored once
      const int64_t tix = row * nt_cap + t;
      const uint4 *src = reinterpret_cast<const uint4 *>(kbits + tix * TILE * 4);
#pragma unroll
      for (int r = 0; r < TPL; ++r) kbd[u][r] = __ldg(src + lane + 32 * r);
#pragma unroll
      for (int m = 0; m < 4; ++m) ksd[u][m] = __ldg(kscale + tix * kD + lane + 32 * m);
      if (sa.vbits != nullptr && lane == 0 && t == t_first + u) {
        // the selected tiles' V is read right after this kernel: stage every
        // scanned tile's V bits + scales in L2 while this (latency-bound) scan runs
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sa.vbits + tix * TILE * 4),
                     "r"((unsigned)(TILE * 16)) : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sa.vscale + tix * kD),
                     "r"((unsigned)(kD * 2)) : "memory");
      }
    }
  };
  // batched decode: this row's exact K/V rows (read by the attention kernel
  // that follows) stream into L2 while the ALU-bound scan runs
#pragma unroll 1
  for (int s = 0; s < 2; ++s) {
    if (sa.rows.k[s] == nullptr) continue;
    const int64_t base = b * sa.rows.batch_stride[s] + (int64_t)h * kD;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < sa.rows.n[s];
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t off = base + i * sa.rows.tok_stride;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sa.rows.k[s] + off), "r"(kD * 2) : "memory");
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sa.rows.v[s] + off), "r"(kD * 2) : "memory");
    }
  }
  int64_t t_cur = cta_t0 + 2 * warp;
  if (t_cur < cta_t1) load_pair(t_cur, kb, ks);
  // launched as a programmatic dependent of the previous kernel: everything
  // above reads only the store; q is read, and anything written, after the
  // previous kernel has finished.  Only then may the attention kernel that
  // follows start (it shares the workspace with the previous one).
  griddep_wait();
  asm volatile("griddepcontrol.launch_dependents;");
  if (kind == KVR_DCT) {
    // strided layout (lane l: elements l + 32 s), the shuffle DCT: warp 0
    // forms q' of the group mean, the other warps of CTA 0 the per-head T q_h
    const int64_t qb = ((int64_t)b * n_q + (int64_t)h * g) * kD;
    float xv[4];
    if (warp == 0) {
#pragma unroll
      for (int s = 0; s < 4; ++s) xv[s] = load1<DTQ>(q, qb + lane + 32 * s);
      for (int i = 1; i < g; ++i)
#pragma unroll
        for (int s = 0; s < 4; ++s) xv[s] = __fadd_rn(xv[s], load1<DTQ>(q, qb + (int64_t)i * kD + lane + 32 * s));
#pragma unroll
      for (int s = 0; s < 4; ++s) xv[s] = __fdiv_rn(xv[s], (float)g);
    }
    __syncthreads();  // Lee factors in shared memory
    if (warp == 0) {
      dct128_fwd_shfl(xv, lane, lee_s);
#pragma unroll
      for (int s = 0; s < 4; ++s) qp_s[lane + 32 * s] = xv[s];
    } else if (blockIdx.x == 0 && qprime != nullptr) {
      for (int i = warp - 1; i < g; i += 7) {
        const int64_t qh = qb + (int64_t)i * kD;
#pragma unroll
        for (int s = 0; s < 4; ++s) xv[s] = load1<DTQ>(q, qh + lane + 32 * s);
        dct128_fwd_shfl(xv, lane, lee_s);
#pragma unroll
        for (int s = 0; s < 4; ++s) qprime[qh + lane + 32 * s] = xv[s];
      }
    }
    __syncthreads();
  } else {
  // warp 0: all g query heads of the group are loaded before the (ordered) sum
  float qv[8][4];
  if (warp == 0) {
    const int64_t qb = ((int64_t)b * n_q + (int64_t)h * g) * kD + lane * 4;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < g) load4<DTQ>(q, qb + (int64_t)i * kD, qv[i]);
  }
  __syncthreads();
  if (warp == 0) {
    float acc[4] = {qv[0][0], qv[0][1], qv[0][2], qv[0][3]};
#pragma unroll
    for (int i = 1; i < 8; ++i)
      if (i < g)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r] = __fadd_rn(acc[r], qv[i][r]);
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] = __fdiv_rn(acc[r], (float)g);
    transform128(acc, lane, kind, false, buf_s[0], lee_s);
    reinterpret_cast<float4 *>(qp_s)[lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  } else if (blockIdx.x == 0 && qprime != nullptr) {
    // per-head transformed queries for the attention kernel
    for (int i = warp - 1; i < g; i += 7) {
      float x[4];
      const int64_t qh = (int64_t)b * n_q + (int64_t)h * g + i;
      load4<DTQ>(q, qh * kD + lane * 4, x);
      transform128(x, lane, kind, false, buf_s[warp], lee_s);
      reinterpret_cast<float4 *>(qprime + qh * kD)[lane] = make_float4(x[0], x[1], x[2], x[3]);
    }
  }
  __syncthreads();
  }
  KVR_TRACE_POINT(0, 1);

  while (t_cur < cta_t1) {  // warp-uniform
    const int64_t t_next = t_cur + 16;
    uint4 kbn[2][TPL];
    uint16_t ksn[2][4];
    if (t_next < cta_t1) load_pair(t_next, kbn, ksn);
    float sc[2];
    sd1_score_tile2<TILE>(qp_s, kb, ks, lane, sc);
    if (lane == 0) {
      scores[row * n_tiles + t_cur] = sc[0];
      if (t_cur + 1 < cta_t1) scores[row * n_tiles + t_cur + 1] = sc[1];
    }
    t_cur = t_next;
    if (t_cur < cta_t1) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
#pragma unroll
        for (int r = 0; r < TPL; ++r) kb[u][r] = kbn[u][r];
#pragma unroll
        for (int m = 0; m < 4; ++m) ks[u][m] = ksn[u][m];
      }
    }
  }
  if (!do_select) return;

  // ---- fused selection by the last CTA of this (b, h)
  __syncthreads();
  KVR_TRACE_POINT(0, 2);
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&sa.counters[row], 1u);
    last_s = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  KVR_TRACE_POINT(0, 3);
  select_row<256>(scores, row, n_tiles, sa, dyn_smem);
  KVR_TRACE_POINT(0, 4);
  if (threadIdx.x == 0) sa.counters[row] = 0u;
}


// ------------------------------------------------------ flat tile scan ----
// Batched steps: the CTAs take equal ranges of the flattened (row, tile)
// space, so every SM gets the same number of tiles whatever the row count
// (one CTA per row leaves SMs with one row next to SMs with two).  A range
// covers at most two rows; its warps score tile pairs inside a row segment
// with the arithmetic of sd1_score_kernel (sd1_score_tile2, one pair loaded
// ahead), and the CTA whose tiles complete a row (per-row tile counter)
// selects that row.  q' of each row is formed with sd1_score_kernel's
// operations.

// One warp: q' = T(mean of the group's query heads) of KV head h into out[128].
template <int DTQ>
__device__ void warp_group_qprime(const void *__restrict__ q, int n_q, int g, int64_t b, int h, int kind,
                                  const float *lee, float *buf, float *out) {
  const int lane = threadIdx.x & 31;
  const int64_t qb = (b * n_q + (int64_t)h * g) * kD;
  if (kind == KVR_DCT) {
    float xv[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) xv[s] = load1<DTQ>(q, qb + lane + 32 * s);
    for (int i = 1; i < g; ++i)
#pragma unroll
      for (int s = 0; s < 4; ++s) xv[s] = __fadd_rn(xv[s], load1<DTQ>(q, qb + (int64_t)i * kD + lane + 32 * s));
#pragma unroll
    for (int s = 0; s < 4; ++s) xv[s] = __fdiv_rn(xv[s], (float)g);
    dct128_fwd_shfl(xv, lane, lee);
#pragma unroll
    for (int s = 0; s < 4; ++s) out[lane + 32 * s] = xv[s];
    return;
  }
  float acc[4], x[4];
  load4<DTQ>(q, qb + lane * 4, acc);
  for (int i = 1; i < g; ++i) {
    load4<DTQ>(q, qb + (int64_t)i * kD + lane * 4, x);
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] = __fadd_rn(acc[r], x[r]);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r] = __fdiv_rn(acc[r], (float)g);
  transform128(acc, lane, kind, false, buf, lee);
  reinterpret_cast<float4 *>(out)[lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// One warp: T q of query head qh (global index) into qprime.
template <int DTQ>
__device__ void warp_head_qprime(const void *__restrict__ q, int64_t qh, int kind, const float *lee, float *buf,
                                 float *__restrict__ qprime) {
  const int lane = threadIdx.x & 31;
  if (kind == KVR_DCT) {
    float xv[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) xv[s] = load1<DTQ>(q, qh * kD + lane + 32 * s);
    dct128_fwd_shfl(xv, lane, lee);
#pragma unroll
    for (int s = 0; s < 4; ++s) qprime[qh * kD + lane + 32 * s] = xv[s];
    return;
  }
  float x[4];
  load4<DTQ>(q, qh * kD + lane * 4, x);
  transform128(x, lane, kind, false, buf, lee);
  reinterpret_cast<float4 *>(qprime + qh * kD)[lane] = make_float4(x[0], x[1], x[2], x[3]);
}

// Per-warp copy ring of the flat scan: kStages pairs of tiles in flight.
template <int TILE>
struct FlatRing {
  static constexpr int kStages = TILE == 128 ? 2 : 4;
  static constexpr size_t kBytes = (size_t)8 * kStages * 2 * (TILE * 16 + kD * 2);  // 8 warps
};

template <int DTQ, int TILE>
__global__ void __launch_bounds__(256, 2) sd1_score_flat_kernel(
    const void *__restrict__ q, int n_q, int n_kv, const uint32_t *__restrict__ kbits,
    const uint16_t *__restrict__ kscale, int64_t nt_cap, int64_t n_tiles, int kind, int64_t rows,
    float *__restrict__ scores, float *__restrict__ qprime, SelectArgs sa, int do_select, int64_t tpc) {
  __shared__ float lee_s[kD];
  __shared__ __align__(16) float buf_s[8][2 * kD];
  __shared__ __align__(16) float qp_s[2][kD];
  __shared__ int last_rows[2];
  __shared__ int n_last;
  __shared__ uint64_t ring_bar[8][FlatRing<TILE>::kStages];
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = n_q / n_kv;
  const int64_t f0 = (int64_t)blockIdx.x * tpc;
  const int64_t f1 = min(rows * n_tiles, f0 + tpc);
  const int64_t r0 = f0 / n_tiles;                 // tpc <= n_tiles: rows r0 and at most r0 + 1
  const int nrows = (int)((f1 - 1) / n_tiles - r0) + 1;
  // segment 0: tiles [st0, st0 + n0) of row r0; segment 1: tiles [0, n1) of row r0 + 1
  const int st0 = (int)(f0 - r0 * n_tiles);
  const int n0 = (int)(min(f1, (r0 + 1) * n_tiles) - f0);
  const int n1 = nrows == 2 ? (int)(f1 - (r0 + 1) * n_tiles) : 0;
  const int pairs0 = (int)((n0 + 1) / 2), n_pairs = pairs0 + (int)((n1 + 1) / 2);
  KVR_TRACE_POINT(2, 0);
  load_lee(lee_s);
  // the CTA holding tile 0 of a row streams that row's exact K/V rows into L2
  // for the attention kernel that follows (a hint: no ordering needed)
  for (int sl = 0; sl < nrows; ++sl) {
    if (sl == 0 && st0 != 0) continue;
    const int64_t r = r0 + sl, b = r / n_kv;
    const int h = (int)(r - b * n_kv);
#pragma unroll 1
    for (int s = 0; s < 2; ++s) {
      if (sa.rows.k[s] == nullptr) continue;
      const int64_t base = b * sa.rows.batch_stride[s] + (int64_t)h * kD;
      for (int64_t i = threadIdx.x; i < sa.rows.n[s]; i += blockDim.x) {
        const int64_t off = base + i * sa.rows.tok_stride;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sa.rows.k[s] + off), "r"(kD * 2) : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sa.rows.v[s] + off), "r"(kD * 2) : "memory");
      }
    }
  }
  constexpr int TPL = TILE / 32;  // tokens per lane
  constexpr int TB = TILE * 16, SB = kD * 2, PB = 2 * (TB + SB), NS = FlatRing<TILE>::kStages;
  // pair p -> (row slot, first tile, last tile of its segment)
  auto pair_at = [&](int p, int &sl, int &t_first, int &t_end) {
    sl = p < pairs0 ? 0 : 1;
    t_first = sl == 0 ? st0 + 2 * p : 2 * (p - pairs0);
    t_end = sl == 0 ? st0 + n0 : n1;
  };
  // Each warp streams its pairs (sign bits + scales of two tiles, PB bytes)
  // through an NS-stage ring of bulk copies in shared memory, NS pairs ahead
  // of the one it scores: enough bytes in flight per SM to cover DRAM latency.
  unsigned char *ring = dyn_smem + (size_t)warp * NS * PB;
  auto issue = [&](int p, int st) {  // lane 0
    int sl, t_first, t_end;
    pair_at(p, sl, t_first, t_end);
    mbar_expect_tx(&ring_bar[warp][st], PB);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int t = min(t_first + u, t_end - 1);  // a lone last tile is scored twice, stored once
      const int64_t tix = (r0 + sl) * nt_cap + t;
      bulk_g2s(ring + st * PB + u * TB, kbits + tix * TILE * 4, TB, &ring_bar[warp][st]);
      bulk_g2s(ring + st * PB + 2 * TB + u * SB, kscale + tix * kD, SB, &ring_bar[warp][st]);
    }
  };
  int issued = 0;  // pairs issued by this warp (warp-uniform)
  if (lane == 0)
    for (int st = 0; st < NS; ++st) mbar_init(&ring_bar[warp][st], 1);
  __syncwarp();
  for (int st = 0; st < NS && warp + 8 * st < n_pairs; ++st, ++issued)
    if (lane == 0) issue(warp + 8 * st, st);
  KVR_TRACE_POINT(2, 6);
  // q is read, and anything written, after the previous kernel has finished
  griddep_wait();
  KVR_TRACE_POINT(2, 7);
  asm volatile("griddepcontrol.launch_dependents;");
  __syncthreads();  // Lee factors
  if (warp < nrows) {
    const int64_t r = r0 + warp, b = r / n_kv;
    warp_group_qprime<DTQ>(q, n_q, g, b, (int)(r - b * n_kv), kind, lee_s, buf_s[warp], qp_s[warp]);
  }
  __syncthreads();
  KVR_TRACE_POINT(2, 1);
  int it = 0;
  for (int p = warp; p < n_pairs; p += 8, ++it) {  // warp-uniform
    const int st = it % NS;
    if (!mbar_wait_bounded(&ring_bar[warp][st], (unsigned)(it / NS) & 1u)) {
      // gave up: report, stop scoring, let the copies in flight land before
      // the shared memory is reused by the selection
      if (lane == 0 && sa.err) atomicOr(sa.err, 4u);
      for (int j = it; j < issued; ++j) mbar_wait_bounded(&ring_bar[warp][j % NS], (unsigned)(j / NS) & 1u);
      break;
    }
    int sl, t_first, t_end;
    pair_at(p, sl, t_first, t_end);
    uint4 kb[2][TPL];
    uint16_t ks[2][4];
    {
      // token rows lane + 32 r of both tiles, channel scales lane + 32 m
      const uint4 *bw = reinterpret_cast<const uint4 *>(ring + st * PB);
      const uint16_t *sw = reinterpret_cast<const uint16_t *>(ring + st * PB + 2 * TB);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
#pragma unroll
        for (int r = 0; r < TPL; ++r) kb[u][r] = bw[u * TILE + lane + 32 * r];
#pragma unroll
        for (int m = 0; m < 4; ++m) ks[u][m] = sw[u * kD + lane + 32 * m];
      }
    }
    __syncwarp();
    if (p + 8 * NS < n_pairs) {
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(p + 8 * NS, st);
      }
      ++issued;
    }
    float sc[2];
    sd1_score_tile2<TILE>(qp_s[sl], kb, ks, lane, sc);
    if (lane == 0) {
      const int64_t r = r0 + sl;
      scores[r * n_tiles + t_first] = sc[0];
      if (t_first + 1 < t_end) scores[r * n_tiles + t_first + 1] = sc[1];
    }
  }
  // per-head T q for the attention kernel (which reads it after this grid
  // has completed), from the CTA holding the row's tile 0: off the path to
  // the first tile scores
  if (qprime != nullptr) {
    for (int it = warp; it < 2 * g; it += 8) {
      const int s2 = it / g, i = it - s2 * g;
      if (s2 >= nrows || (s2 == 0 && st0 != 0)) continue;
      const int64_t r = r0 + s2, b = r / n_kv;
      warp_head_qprime<DTQ>(q, (b * n_q + (r - b * n_kv) * g + i), kind, lee_s, buf_s[warp], qprime);
    }
  }
  KVR_TRACE_POINT(2, 2);
  if (!do_select) return;  // the consumer selects from the scores
  // the CTA whose tiles complete a row selects it
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    int nl = 0;
    for (int s2 = 0; s2 < nrows; ++s2) {
      const unsigned cnt = (unsigned)(s2 == 0 ? n0 : n1);
      const unsigned prev = atomicAdd(&sa.counters[r0 + s2], cnt);
      if (prev + cnt == (unsigned)n_tiles) last_rows[nl++] = s2;
    }
    n_last = nl;
  }
  __syncthreads();
  for (int i = 0; i < n_last; ++i) {
    __threadfence();
    const int64_t r = r0 + last_rows[i];
    select_row<256>(scores, r, n_tiles, sa, dyn_smem);
    if (threadIdx.x == 0) sa.counters[r] = 0u;
    __syncthreads();
  }
  KVR_TRACE_POINT(2, 3 + n_last);
}

// ---------------------------------------------------------- tile decode ----
// One warp per (b, h, selected slot, token): k_hat = T^T(s * (2 bit - 1)).
__global__ void __launch_bounds__(256) sd1_decode_tiles_kernel(
    const uint32_t *__restrict__ kbits, const uint16_t *__restrict__ kscale, const uint32_t *__restrict__ vbits,
    const uint16_t *__restrict__ vscale, int64_t nt_cap, int n_kv, int tile, int kind,
    const int64_t *__restrict__ sel, int k, float *__restrict__ out_k, uint16_t *__restrict__ out_v,
    int64_t total_rows) {
  __shared__ float lee_s[kD];
  __shared__ __align__(16) float buf_s[8][2 * kD];
  load_lee(lee_s);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < total_rows; r += (int64_t)gridDim.x * 8) {
    // r enumerates (b, h, slot, j)
    const int j = (int)(r % tile);
    const int64_t bhs = r / tile;
    const int slot = (int)(bhs % k);
    const int64_t bh = bhs / k;
    const int h = (int)(bh % n_kv);
    const int64_t b = bh / n_kv;
    const int64_t t = sel[bh * k + slot];
    const int64_t orow = ((b * k + slot) * tile + j) * n_kv + h;  // (B, k*t, n_kv, d)
    if (t < 0) {
      reinterpret_cast<float4 *>(out_k + orow * kD)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<uint2 *>(out_v + orow * kD)[lane] = make_uint2(0u, 0u);
      continue;
    }
    const int64_t tix = bh * nt_cap + t;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const uint32_t *bits = (kv == 0 ? kbits : vbits) + (tix * tile + j) * 4;
      const uint16_t *sc = (kv == 0 ? kscale : vscale) + tix * kD;
      const uint32_t w = __ldg(bits + (lane >> 3));
      float x[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int c = lane * 4 + q;
        const float s = __half2float(__ushort_as_half(__ldg(sc + c)));
        x[q] = ((w >> (c & 31)) & 1u) ? s : -s;
      }
      transform128(x, lane, kind, true, buf_s[warp], lee_s);
      if (kv == 0) {
        reinterpret_cast<float4 *>(out_k + orow * kD)[lane] = make_float4(x[0], x[1], x[2], x[3]);
      } else {
        __half2 a = __floats2half2_rn(x[0], x[1]), c2 = __floats2half2_rn(x[2], x[3]);
        reinterpret_cast<uint2 *>(out_v + orow * kD)[lane] =
            make_uint2(*reinterpret_cast<uint32_t *>(&a), *reinterpret_cast<uint32_t *>(&c2));
      }
    }
  }
}

static int grid_for(int64_t items, int per_block) {
  int64_t g = (items + per_block - 1) / per_block;
  if (g > 148 * 64) g = 148 * 64;
  return (int)(g < 1 ? 1 : g);
}

template <int DT>
static int launch_encode(int tile, dim3 grid, size_t smem, cudaStream_t st, const void *k, const void *v,
                         int n_kv, int64_t bs, int64_t ts, const float *c, const float *s, int64_t rs, int64_t pos0,
                         int kind, uint32_t *kb, uint16_t *ks, uint32_t *vb, uint16_t *vs, int64_t cap,
                         int64_t t0, int vec16) {
  switch (tile) {
#define KVR_ENC(T)                                                                                       \
  case T:                                                                                                \
    cudaFuncSetAttribute(sd1_encode_kernel<DT, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    sd1_encode_kernel<DT, T><<<grid, 2 * T, smem, st>>>(k, v, n_kv, bs, ts, c, s, rs, pos0, kind, kb, ks, vb, \
                                                         vs, cap, t0, vec16);                            \
    break;
    KVR_ENC(32)
    KVR_ENC(64)
    KVR_ENC(128)
#undef KVR_ENC
    default:
      return set_error(KVR_ENOTSUP, "sd1: tile must be 32, 64 or 128 (got %d)", tile);
  }
  return check_launch("kvr_sd1_encode");
}

size_t select_dyn_smem(int k_sel, int64_t n_tiles) {
  return align_up(sizeof(TopkSmem), 16) + select_cand_bytes(k_sel) +
         (n_tiles <= kSelectSmemScores ? (size_t)(n_tiles > 0 ? n_tiles : 1) * 4 : 0);
}

// Raises a kernel's dynamic shared-memory limit (once per device and size)
// when its static + dynamic shared memory may pass the default 48 KB.
template <typename F>
static void ensure_dyn_smem(F *fn, size_t dyn_bytes) {
  constexpr int kMaxDev = 64;
  if (dyn_bytes + 16 * 1024 <= 48 * 1024) return;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDev) dev = 0;
  static thread_local std::vector<std::pair<const void *, size_t>> done[kMaxDev];
  for (auto &e : done[dev])
    if (e.first == reinterpret_cast<const void *>(fn) && e.second >= dyn_bytes) return;
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_bytes);
  done[dev].emplace_back(reinterpret_cast<const void *>(fn), dyn_bytes);
}

template <int DTQ>
static int launch_score(int tile, dim3 grid, int64_t tpc, cudaStream_t st, const void *q, int n_q, int n_kv,
                        const uint32_t *kb, const uint16_t *ks, int64_t cap, int64_t nt, int kind, float *scores,
                        float *qprime, SelectArgs sa, int do_select) {
  const size_t smem = do_select ? select_dyn_smem(sa.k_sel, nt) : 0;
  switch (tile) {
#define KVR_SC(T)                                                                                        \
  case T:                                                                                                \
    ensure_dyn_smem(sd1_score_kernel<DTQ, T>, smem);                                                    \
    {                                                                                                    \
      cudaLaunchConfig_t cfg{};                                                                          \
      cfg.gridDim = grid;                                                                                \
      cfg.blockDim = dim3(256);                                                                          \
      cfg.dynamicSmemBytes = smem;                                                                       \
      cfg.stream = st;                                                                                   \
      cudaLaunchAttribute at[1];                                                                         \
      at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;                                     \
      at[0].val.programmaticStreamSerializationAllowed = 1;                                              \
      cfg.attrs = at;                                                                                    \
      cfg.numAttrs = 1;                                                                                  \
      cudaLaunchKernelEx(&cfg, sd1_score_kernel<DTQ, T>, q, n_q, n_kv, kb, ks, cap, nt, kind, scores,     \
                         qprime, sa, do_select, tpc);                                                    \
    }                                                                                                    \
    break;
    KVR_SC(32)
    KVR_SC(64)
    KVR_SC(128)
#undef KVR_SC
    default:
      return set_error(KVR_ENOTSUP, "sd1: tile must be 32, 64 or 128 (got %d)", tile);
  }
  return check_launch("sd1 tile scores");
}


template <int DTQ>
static int launch_score_flat(int tile, int64_t rows, int64_t tpc, cudaStream_t st, const void *q, int n_q,
                             int n_kv, const uint32_t *kb, const uint16_t *ks, int64_t cap, int64_t nt, int kind,
                             float *scores, float *qprime, SelectArgs sa, int do_select) {
  const size_t sel_smem = do_select ? select_dyn_smem(sa.k_sel, nt) : 0;
  const size_t ring = tile == 32 ? FlatRing<32>::kBytes : tile == 64 ? FlatRing<64>::kBytes : FlatRing<128>::kBytes;
  const size_t smem = sel_smem > ring ? sel_smem : ring;  // the selection reuses the ring after the scan
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)((rows * nt + tpc - 1) / tpc));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  switch (tile) {
#define KVR_SF(T)                                                                                       \
  case T:                                                                                               \
    ensure_dyn_smem(sd1_score_flat_kernel<DTQ, T>, smem);                                               \
    cudaLaunchKernelEx(&cfg, sd1_score_flat_kernel<DTQ, T>, q, n_q, n_kv, kb, ks, cap, nt, kind, rows,  \
                       scores, qprime, sa, do_select, tpc);                                             \
    break;
    KVR_SF(32)
    KVR_SF(64)
    KVR_SF(128)
#undef KVR_SF
    default:
      return set_error(KVR_ENOTSUP, "sd1: tile must be 32, 64 or 128 (got %d)", tile);
  }
  return check_launch("sd1 tile scores (flat)");
}

int sd1_scores_impl(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint32_t *kbits,
                    const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind, float *scores,
                    float *qprime, SelectArgs sa, int do_select, cudaStream_t st) {
  const int64_t rows = (int64_t)batch * n_kv;
  // Batched steps: equal flat ranges of the (row, tile) space,
  // two CTAs per SM, once that gives every CTA at least 16 tiles and at most
  // one row's worth (KVR_SD1_SCAN=flat / warps forces a path where valid).
  {
    const char *scan = getenv("KVR_SD1_SCAN");
    const bool force_flat = scan && strcmp(scan, "flat") == 0, force_warps = scan && strcmp(scan, "warps") == 0;
    const int64_t total = rows * n_tiles;
    const int64_t ftpc = (total + 295) / 296;
    if (sa.vbits == nullptr && n_tiles >= 16 && !force_warps &&
        (force_flat ? (total > 0 && ftpc <= n_tiles) : (ftpc >= 16 && ftpc <= n_tiles && rows > 1))) {
      const int64_t t = force_flat && ftpc < 16 ? (n_tiles < 16 ? n_tiles : 16) : ftpc;
      switch (q_dtype) {
        case KVR_F32: return launch_score_flat<KVR_F32>(tile, rows, t, st, q, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, kind, scores, qprime, sa, do_select);
        case KVR_F16: return launch_score_flat<KVR_F16>(tile, rows, t, st, q, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, kind, scores, qprime, sa, do_select);
        default: return launch_score_flat<KVR_BF16>(tile, rows, t, st, q, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, kind, scores, qprime, sa, do_select);
      }
    }
  }
  // Tiles per CTA: about one resident wave (2 CTAs per SM) in total, at least
  // 16 (two per warp); each CTA forms q' once for all of its tiles.
  int64_t cph = 296 / (rows > 0 ? rows : 1);
  const int64_t max_cph = (n_tiles + kScoreTilesPerCta - 1) / kScoreTilesPerCta;
  cph = cph < 1 ? 1 : (cph > max_cph ? max_cph : cph);
  if (cph < 1) cph = 1;
  int64_t tpc = (n_tiles + cph - 1) / cph;
  tpc = (tpc + kScoreTilesPerCta - 1) / kScoreTilesPerCta * kScoreTilesPerCta;
  if (tpc < kScoreTilesPerCta) tpc = kScoreTilesPerCta;
  dim3 grid((unsigned)(n_tiles > 0 ? (n_tiles + tpc - 1) / tpc : 1), n_kv, batch);
  switch (q_dtype) {
    case KVR_F32: return launch_score<KVR_F32>(tile, grid, tpc, st, q, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, kind, scores, qprime, sa, do_select);
    case KVR_F16: return launch_score<KVR_F16>(tile, grid, tpc, st, q, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, kind, scores, qprime, sa, do_select);
    default: return launch_score<KVR_BF16>(tile, grid, tpc, st, q, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, kind, scores, qprime, sa, do_select);
  }
}

}  // namespace kvr

using namespace kvr;

static int check_common_sd1(int batch, int n_q, int n_kv, int tile, int kind) {
  KVR_REQUIRE(batch > 0 && n_kv > 0 && n_q > 0 && n_q % n_kv == 0, "sd1: bad batch/head counts (B=%d n_q=%d n_kv=%d)", batch, n_q, n_kv);
  KVR_REQUIRE(tile == 32 || tile == 64 || tile == 128, "sd1: tile must be 32, 64 or 128 (got %d)", tile);
  KVR_REQUIRE(kind == KVR_HADAMARD || kind == KVR_DCT, "sd1: unknown transform kind %d", kind);
  return KVR_OK;
}

extern "C" int kvr_transform(const float *x, float *y, int64_t rows, int kind, int inverse, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(x && y && rows >= 0, "kvr_transform: null pointer or negative rows");
  KVR_REQUIRE(kind == KVR_HADAMARD || kind == KVR_DCT, "kvr_transform: unknown kind %d", kind);
  if (rows == 0) return KVR_OK;
  transform_kernel<<<grid_for(rows, 8), 256, 0, as_cuda(stream)>>>(x, y, rows, kind, inverse);
  return check_launch("kvr_transform");
}

extern "C" int kvr_sd1_encode(const void *k, const void *v, int dtype, int batch, int n_kv, int64_t n_tiles,
                              int tile, int64_t batch_stride, int64_t tok_stride, const float *cos_tbl,
                              const float *sin_tbl, int64_t rope_stride, int64_t pos0, int kind, uint32_t *kbits,
                              uint16_t *kscale, uint32_t *vbits, uint16_t *vscale, int64_t nt_cap, int64_t tile0,
                              kvr_stream_t stream) {
  clear_error();
  int rc = check_common_sd1(batch, n_kv, n_kv, tile, kind);
  if (rc) return rc;
  KVR_REQUIRE(valid_dtype(dtype), "kvr_sd1_encode: bad dtype %d", dtype);
  KVR_REQUIRE(k && v && kbits && kscale && vbits && vscale, "kvr_sd1_encode: null pointer");
  KVR_REQUIRE(n_tiles >= 0 && tile0 >= 0 && tile0 + n_tiles <= nt_cap, "kvr_sd1_encode: tiles [%lld, %lld) exceed nt_cap %lld",
              (long long)tile0, (long long)(tile0 + n_tiles), (long long)nt_cap);
  KVR_REQUIRE(tok_stride % 4 == 0 && batch_stride % 4 == 0, "kvr_sd1_encode: strides must be multiples of 4 elements");
  KVR_REQUIRE((cos_tbl == nullptr) == (sin_tbl == nullptr), "kvr_sd1_encode: give both rope tables or neither");
  KVR_REQUIRE(cos_tbl == nullptr || (rope_stride % 4 == 0 && pos0 >= 0), "kvr_sd1_encode: bad rope table stride/pos0");
  KVR_REQUIRE(n_tiles <= 0x7fffffff, "kvr_sd1_encode: too many tiles per launch");
  if (n_tiles == 0) return KVR_OK;
  const int es = dtype == KVR_F32 ? 4 : 2;
  auto al = [](const void *p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  KVR_REQUIRE(al(k, 8) && al(v, 8) && (cos_tbl == nullptr || (al(cos_tbl, 8) && al(sin_tbl, 8))),
              "kvr_sd1_encode: k, v and rope tables must be 8-byte aligned");
  // 16-byte staging copies when every row start is 16-byte aligned, else 8-byte ones
  const int vec16 = al(k, 16) && al(v, 16) && (tok_stride * es) % 16 == 0 && (batch_stride * es) % 16 == 0 &&
                    (cos_tbl == nullptr || (al(cos_tbl, 16) && al(sin_tbl, 16) && (rope_stride * 4) % 16 == 0));
  // X[2][128][tile + 4] fp32, aliased by the staging rows (+ RoPE rows)
  const size_t x_bytes = (size_t)2 * kD * (tile + 4) * 4;
  const size_t stage = (size_t)2 * tile * (kD * es + 16) + (cos_tbl ? (size_t)2 * tile * (kD * 4 + 16) : 0);
  const size_t smem = x_bytes > stage ? x_bytes : stage;
  dim3 grid((unsigned)n_tiles, n_kv, batch);
  cudaStream_t st = as_cuda(stream);
  switch (dtype) {
    case KVR_F32: return launch_encode<KVR_F32>(tile, grid, smem, st, k, v, n_kv, batch_stride, tok_stride, cos_tbl, sin_tbl, rope_stride, pos0, kind, kbits, kscale, vbits, vscale, nt_cap, tile0, vec16);
    case KVR_F16: return launch_encode<KVR_F16>(tile, grid, smem, st, k, v, n_kv, batch_stride, tok_stride, cos_tbl, sin_tbl, rope_stride, pos0, kind, kbits, kscale, vbits, vscale, nt_cap, tile0, vec16);
    default: return launch_encode<KVR_BF16>(tile, grid, smem, st, k, v, n_kv, batch_stride, tok_stride, cos_tbl, sin_tbl, rope_stride, pos0, kind, kbits, kscale, vbits, vscale, nt_cap, tile0, vec16);
  }
}

extern "C" int kvr_sd1_tile_scores(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint32_t *kbits,
                                   const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind,
                                   float *scores, kvr_stream_t stream) {
  clear_error();
  int rc = check_common_sd1(batch, n_q, n_kv, tile, kind);
  if (rc) return rc;
  KVR_REQUIRE(valid_dtype(q_dtype), "kvr_sd1_tile_scores: bad dtype %d", q_dtype);
  KVR_REQUIRE(q && kbits && kscale && scores, "kvr_sd1_tile_scores: null pointer");
  KVR_REQUIRE(n_tiles >= 0 && n_tiles <= nt_cap, "kvr_sd1_tile_scores: n_tiles > nt_cap");
  if (n_tiles == 0) return KVR_OK;
  SelectArgs sa{};
  return sd1_scores_impl(q, q_dtype, batch, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, tile, kind, scores,
                         nullptr, sa, 0, as_cuda(stream));
}

namespace kvr {
// Selection with explicit scratch: counters (B*n_kv) and scores (B*n_kv*n_tiles).
int sd1_select_scratch(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint32_t *kbits,
                       const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind, int k_sel,
                       int64_t ex_t0, int64_t ex_t1, int64_t tile_base, int32_t *sel, float *sel_scores,
                       float *qprime, unsigned *counters, float *scores, cudaStream_t st,
                       const uint32_t *vbits, const uint16_t *vscale, int do_select, const RowPrefetch *rows) {
  int rc = check_common_sd1(batch, n_q, n_kv, tile, kind);
  if (rc) return rc;
  KVR_REQUIRE(valid_dtype(q_dtype), "kvr_sd1_select: bad dtype %d", q_dtype);
  KVR_REQUIRE(q && sel && qprime, "kvr_sd1_select: null pointer");
  KVR_REQUIRE(k_sel >= 0 && k_sel <= 4096, "kvr_sd1_select: k_sel must be in [0, 4096]");
  KVR_REQUIRE(n_tiles >= 0 && n_tiles <= nt_cap, "kvr_sd1_select: n_tiles > nt_cap");
  KVR_REQUIRE(n_tiles == 0 || (kbits && kscale), "kvr_sd1_select: null store pointers");
  KVR_REQUIRE((int64_t)batch * n_kv <= kWsMaxRows, "kvr_sd1_select: batch*n_kv > %d", kWsMaxRows);
  SelectArgs sa{k_sel, ex_t0, ex_t1, tile_base, sel, sel_scores, counters, vbits, vscale, RowPrefetch{}};
  if (rows) sa.rows = *rows;
  // every workspace that holds the selection counters starts with the error word
  sa.err = reinterpret_cast<unsigned *>(reinterpret_cast<char *>(counters) - kWsSelCounters);
  // With no full tile there is nothing to score; the kernel still forms q'
  // and writes an all-empty selection.
  return sd1_scores_impl(q, q_dtype, batch, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, tile, kind, scores, qprime,
                         sa, do_select, st);
}
}  // namespace kvr

extern "C" size_t kvr_sd1_select_workspace_bytes(int batch, int n_kv, int64_t n_tiles) {
  const size_t rows = (size_t)batch * n_kv;
  return kWsHeader + align_up(rows * (size_t)(n_tiles > 0 ? n_tiles : 1) * 4, 256);
}

extern "C" int kvr_sd1_select(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint32_t *kbits,
                              const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind, int k_sel,
                              int64_t ex_t0, int64_t ex_t1, int64_t tile_base, int32_t *sel, float *sel_scores,
                              float *qprime, void *workspace, size_t workspace_bytes, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(workspace, "kvr_sd1_select: null workspace");
  KVR_REQUIRE(batch > 0 && n_kv > 0, "kvr_sd1_select: bad batch/head counts");
  const size_t need = kvr_sd1_select_workspace_bytes(batch, n_kv, n_tiles);
  KVR_REQUIRE(workspace_bytes >= need, "kvr_sd1_select: workspace %zu < %zu bytes", workspace_bytes, need);
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "kvr_sd1_select: workspace must be 256-byte aligned");
  char *p = reinterpret_cast<char *>(workspace);
  return sd1_select_scratch(q, q_dtype, batch, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, tile, kind, k_sel, ex_t0,
                            ex_t1, tile_base, sel, sel_scores, qprime, reinterpret_cast<unsigned *>(p + kWsSelCounters),
                            reinterpret_cast<float *>(p + kWsHeader), as_cuda(stream), nullptr, nullptr, 1, nullptr);
}

extern "C" int kvr_sd1_decode_tiles(const uint32_t *kbits, const uint16_t *kscale, const uint32_t *vbits,
                                    const uint16_t *vscale, int64_t nt_cap, int batch, int n_kv, int tile, int kind,
                                    const int64_t *sel, int k, float *out_k, uint16_t *out_v, kvr_stream_t stream) {
  clear_error();
  int rc = check_common_sd1(batch, n_kv, n_kv, tile, kind);
  if (rc) return rc;
  KVR_REQUIRE(kbits && kscale && vbits && vscale && sel && out_k && out_v, "kvr_sd1_decode_tiles: null pointer");
  KVR_REQUIRE(k >= 0, "kvr_sd1_decode_tiles: negative k");
  const int64_t rows = (int64_t)batch * n_kv * k * tile;
  if (rows == 0) return KVR_OK;
  sd1_decode_tiles_kernel<<<grid_for(rows, 8), 256, 0, as_cuda(stream)>>>(kbits, kscale, vbits, vscale, nt_cap, n_kv,
                                                                           tile, kind, sel, k, out_k, out_v, rows);
  return check_launch("kvr_sd1_decode_tiles");
}

#ifdef KVR_TRACE
extern "C" KVR_API int kvr_debug_trace_sd1(unsigned long long *host, int n) {
  return cudaMemcpyFromSymbol(host, kvr::g_kvr_trace, sizeof(unsigned long long) * n) == cudaSuccess ? 0 : 2;
}
#endif
