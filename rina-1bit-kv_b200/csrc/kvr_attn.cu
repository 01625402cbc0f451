// Decode attention over exact K/V segments and sd1 1-bit tiles (sm_100a).
//
// Work decomposition: for every (batch b, KV head h) the tokens are cut into
// units — 64-token chunks of up to two exact segments (the fp16 window ring,
// the pending tail, or the retrieved rows of the int4w path) and selected
// sd1 tiles.  One CTA of 256 threads handles one unit for all g = n_q/n_kv
// query heads of the group and writes a log-sum-exp partial (m, l, o); the
// last CTA of each (b, h) to finish merges the partials (no grid-wide wait).
// sd1 units work in the transformed domain: scores use q' = T q because T is
// orthonormal, their partial o' is merged first and mapped back with one
// inverse transform per query head.  Selected tiles are staged into shared
// memory with bulk asynchronous copies completing on an mbarrier.
//
// Reference behaviour replaced: exact softmax over window + retrieved tokens
// with GQA kvh = hq / g (modules/kvr_window.py:43-69, kvr_hook.py:274-282,
// kvr_triton.py:42-79, kvr_generator.py:448-450).
#include "kvr_common.cuh"
#include "kvr_topk.cuh"
#include "kvr_transform.cuh"

#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>

namespace kvr {

constexpr int kChunk = 64;
constexpr int kMaxG = 8;
constexpr int kKsStride = kD + 4;  // padded fp32 row of the staged K chunk
// workspace partial row of one CTA slot and query head:
// [m, l, pad, pad, o_exact[128], o_transformed[128]] (16-byte aligned rows)
constexpr int kPartStride = 4 + 2 * kD;
constexpr int kPartEx = 4;
constexpr int kPartTr = 4 + kD;

struct AttnArgs {
  const void *q;
  int q_dt, n_q, n_kv, g;
  float inv_scale;
  const float *qprime;  // (B, n_q, d), sd1 units only
  const void *k[2];
  const void *v[2];
  int kdt[2], vdt[2];
  int64_t n[2], tok_stride[2], batch_stride[2];
  int nchunk[2];
  const uint32_t *kbits;
  const uint16_t *kscale;
  const uint32_t *vbits;
  const uint16_t *vscale;
  int64_t nt_cap;
  int tile, kind, k_sel;
  const int32_t *sel;  // (B, n_kv, k_sel)
  // selection inside the tile units (batch-1 decode): scores of the row
  // (B, n_kv, rank_n), exclusion range, and where the chosen indices go
  const float *rank_scores;
  int64_t rank_n, rank_ex0, rank_ex1;
  int32_t *sel_out;
  void *out;
  int out_dt;
  float *partial_out;  // (B, n_q, d+2) or null
  float *part;         // (B, n_kv, units, g, d+2)
  unsigned *counters;  // (B, n_kv)
  unsigned *err;
  int units;  // work units per (b, h)
  int upc;    // units per CTA
  int slots;  // CTAs per (b, h) = ceil(units / upc)
  int pipelined;  // batched rows over fp16 exact data: attn_rows_kernel
  const int32_t *n1_dev;  // optional device-side bound on segment 1's rows (exact units only)
};

// ---- runtime-dtype loads
__device__ __forceinline__ void load4_rt(const void *p, int64_t i, int dt, float (&x)[4]) {
  if (dt == KVR_F32) load4<KVR_F32>(p, i, x);
  else if (dt == KVR_F16) load4<KVR_F16>(p, i, x);
  else load4<KVR_BF16>(p, i, x);
}

// ---- shared memory plan (bytes)
struct AttnSmem {
  static constexpr int kKs = 0;                                      // fp32 [64][132]
  static constexpr int kVs = kKs + kChunk * kKsStride * 4;           // fp32 [64][128]
  static constexpr int kExactEnd = kVs + kChunk * kD * 4;
  // sd1 tile unit reuses the region: bits, scales, LUT
  static constexpr int kKB = 0;                                      // u32 [128][4]
  static constexpr int kVB = kKB + 128 * 16;                         // u32 [128][4]
  static constexpr int kKS = kVB + 128 * 16;                         // fp16 [128]
  static constexpr int kVS = kKS + kD * 2;                           // fp16 [128]
  static constexpr int kLUT = kVS + kD * 2;                          // fp32 [g][32][16]
  static constexpr int kTileEnd = kLUT + kMaxG * 32 * 16 * 4;
  // the unit region also hosts the batched-decode staging (RowSmem); its size
  // is kept at two 64-row K + V chunks of padded fp16 rows
  static constexpr int kRawRow = kD * 2 + 16;
  static constexpr int kRawBuf = 2 * kChunk * kRawRow;
  static constexpr int kUnion0 = kExactEnd > kTileEnd ? kExactEnd : kTileEnd;
  static constexpr int kUnion = kUnion0 > 2 * kRawBuf ? kUnion0 : 2 * kRawBuf;
  static constexpr int kQ = kUnion;                                  // fp32 [8][128]
  static constexpr int kS = kQ + kMaxG * kD * 4;                     // fp32 [8][128] scores / reduce
  static constexpr int kP = kS + kMaxG * kD * 4;                     // fp32 [128][8] probabilities
  static constexpr int kML = kP + 128 * kMaxG * 4;                   // fp32 [8][2]
  static constexpr int kBar = kML + kMaxG * 2 * 4;                   // u64
  static constexpr int kFlag = kBar + 16;
  static constexpr int kLee = kFlag + 16;                             // fp32 [128] DCT factors
  static constexpr int kAccM = kLee + kD * 4;                         // fp32 [8] running max
  static constexpr int kAccL = kAccM + kMaxG * 4;                     // fp32 [8] running sum
  static constexpr int kAccSC = kAccL + kMaxG * 4;                    // fp32 [8][2] fold factors
  static constexpr int kAccEx = kAccSC + kMaxG * 2 * 4;               // fp32 [8][128] exact part
  static constexpr int kAccTr = kAccEx + kMaxG * kD * 4;              // fp32 [8][128] transformed part
  static constexpr int kTotal = kAccTr + kMaxG * kD * 4;
};

// Softmax over the scores S[hq][0..nt) of every query head; writes P[j][hq],
// ML[hq] = (m, l).  Rows with no valid token get m = -inf, l = 0.
__device__ __forceinline__ void softmax_rows(const AttnArgs &a, int nt, const float *S, float *P, float *ML) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int hq = warp; hq < a.g; hq += 8) {
    float mx = -INFINITY;
    for (int j = lane; j < nt; j += 32) mx = fmaxf(mx, S[hq * kD + j]);
    mx = warp_max(mx);
    float l = 0.0f;
    for (int j = lane; j < 128; j += 32) {
      float p = 0.0f;
      if (j < nt && mx != -INFINITY) p = expf(S[hq * kD + j] - mx);
      P[j * kMaxG + hq] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      ML[hq * 2] = mx;
      ML[hq * 2 + 1] = l;
    }
  }
}

__device__ __forceinline__ float *part_row(const AttnArgs &a, int64_t row, int slot, int hq) {
  return a.part + (((row * a.slots + slot) * a.g) + hq) * (int64_t)kPartStride;
}

// Folds the unit just computed (unit m, l in ML; unit output rows in S[hq][128])
// into the CTA's running accumulators (online softmax).
__device__ void fold_unit(const AttnArgs &a, unsigned char *sm, bool into_tr) {
  float *M = reinterpret_cast<float *>(sm + AttnSmem::kAccM);
  float *L = reinterpret_cast<float *>(sm + AttnSmem::kAccL);
  float *SC = reinterpret_cast<float *>(sm + AttnSmem::kAccSC);
  float *Ex = reinterpret_cast<float *>(sm + AttnSmem::kAccEx);
  float *Tr = reinterpret_cast<float *>(sm + AttnSmem::kAccTr);
  const float *UML = reinterpret_cast<const float *>(sm + AttnSmem::kML);
  const float *S = reinterpret_cast<const float *>(sm + AttnSmem::kS);
  const int tid = threadIdx.x;
  if (tid < a.g) {
    const float mo = M[tid], mu = UML[2 * tid], lu = UML[2 * tid + 1];
    const float mn = fmaxf(mo, mu);
    const float al = (mo == -INFINITY) ? 0.0f : expf(mo - mn);
    const float be = (mu == -INFINITY) ? 0.0f : expf(mu - mn);
    SC[2 * tid] = al;
    SC[2 * tid + 1] = be;
    M[tid] = mn;
    L[tid] = L[tid] * al + lu * be;
  }
  __syncthreads();
  for (int i = tid; i < a.g * kD; i += blockDim.x) {
    const int hq = i >> 7;
    const float al = SC[2 * hq], be = SC[2 * hq + 1];
    const float u = S[i] * be;
    Ex[i] = Ex[i] * al + (into_tr ? 0.0f : u);
    Tr[i] = Tr[i] * al + (into_tr ? u : 0.0f);
  }
  __syncthreads();
}

// ----------------------------------------------------------- exact unit ----
__device__ void exact_unit(const AttnArgs &a, unsigned char *sm, int64_t b, int h, int seg, int chunk, int u) {
  float *Ks = reinterpret_cast<float *>(sm + AttnSmem::kKs);
  float *Vs = reinterpret_cast<float *>(sm + AttnSmem::kVs);
  float *Qs = reinterpret_cast<float *>(sm + AttnSmem::kQ);
  float *S = reinterpret_cast<float *>(sm + AttnSmem::kS);
  float *P = reinterpret_cast<float *>(sm + AttnSmem::kP);
  float *ML = reinterpret_cast<float *>(sm + AttnSmem::kML);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = b * a.n_kv + h;
  const int64_t t0 = (int64_t)chunk * kChunk;
  int64_t nseg = a.n[seg];
  if (seg == 1 && a.n1_dev) {
    const int64_t nd = __ldg(a.n1_dev);
    nseg = nd < nseg ? nd : nseg;
  }
  const int nt = (int)(nseg - t0 < kChunk ? nseg - t0 : kChunk);

  // Stage q (scaled) and the K/V chunk as fp32: every global load of the
  // chunk is issued before the first shared-memory store, so the chunk
  // arrives in one DRAM round trip.
  const int64_t base = b * a.batch_stride[seg] + (int64_t)h * kD;
  const int kdt = a.kdt[seg], vdt = a.vdt[seg];
  uint4 rk[8], rv[8], rq = make_uint4(0u, 0u, 0u, 0u);
  const bool has_q = tid < a.g * 32;
  if (has_q) rq = raw4(a.q, (b * a.n_q + (int64_t)h * a.g + (tid >> 5)) * kD + (tid & 31) * 4, a.q_dt);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = tid + i * 256, j = idx >> 5, qd = idx & 31;
    rk[i] = rv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (j < nt) {
      const int64_t off = base + (t0 + j) * a.tok_stride[seg] + qd * 4;
      rk[i] = raw4(a.k[seg], off, kdt);
      rv[i] = raw4(a.v[seg], off, vdt);
    }
  }
  if (has_q) {
    const float4 x = cvt4(rq, a.q_dt);
    reinterpret_cast<float4 *>(Qs + (tid >> 5) * kD)[tid & 31] =
        make_float4(x.x * a.inv_scale, x.y * a.inv_scale, x.z * a.inv_scale, x.w * a.inv_scale);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = tid + i * 256, j = idx >> 5, qd = idx & 31;
    *reinterpret_cast<float4 *>(Ks + j * kKsStride + qd * 4) = cvt4(rk[i], kdt);
    *reinterpret_cast<float4 *>(Vs + j * kD + qd * 4) = cvt4(rv[i], vdt);
  }
  __syncthreads();
  KVR_TRACE_POINT(1, 1);
  // scores: (hq, 32-token block) pairs, lane = token
  for (int p = warp; p < a.g * 2; p += 8) {
    const int hq = p >> 1, j = (p & 1) * 32 + lane;
    const float4 *kr = reinterpret_cast<const float4 *>(Ks + j * kKsStride);
    const float4 *qr = reinterpret_cast<const float4 *>(Qs + hq * kD);
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 8
    for (int c = 0; c < 32; ++c) {
      const float4 kk = kr[c], qq = qr[c];
      a0 = fmaf(qq.x, kk.x, a0);
      a1 = fmaf(qq.y, kk.y, a1);
      a2 = fmaf(qq.z, kk.z, a2);
      a3 = fmaf(qq.w, kk.w, a3);
    }
    S[hq * kD + j] = j < nt ? (a0 + a1) + (a2 + a3) : -INFINITY;
  }
  __syncthreads();
  softmax_rows(a, nt, S, P, ML);
  __syncthreads();
  KVR_TRACE_POINT(1, 2);
  // P.V: thread = (channel, token half)
  const int c = tid & 127, half = tid >> 7;
  float o[kMaxG];
#pragma unroll
  for (int i = 0; i < kMaxG; ++i) o[i] = 0.0f;
  for (int j = half * 32; j < half * 32 + 32; ++j) {
    const float vv = Vs[j * kD + c];
    const float4 p0 = *reinterpret_cast<const float4 *>(P + j * kMaxG);
    const float4 p1 = *reinterpret_cast<const float4 *>(P + j * kMaxG + 4);
    o[0] = fmaf(p0.x, vv, o[0]); o[1] = fmaf(p0.y, vv, o[1]);
    o[2] = fmaf(p0.z, vv, o[2]); o[3] = fmaf(p0.w, vv, o[3]);
    if (a.g > 4) {
      o[4] = fmaf(p1.x, vv, o[4]); o[5] = fmaf(p1.y, vv, o[5]);
      o[6] = fmaf(p1.z, vv, o[6]); o[7] = fmaf(p1.w, vv, o[7]);
    }
  }
  if (half == 1)
    for (int hq = 0; hq < a.g; ++hq) S[hq * kD + c] = o[hq];
  __syncthreads();
  if (half == 0)
    for (int hq = 0; hq < a.g; ++hq) S[hq * kD + c] += o[hq];
  __syncthreads();
  fold_unit(a, sm, false);
}

// ------------------------------------------------------- in-unit select ----
// Tile unit `slot` attends the tile of rank `slot` (score desc, index asc).
// Every tile unit of a row finds its own order statistic of the row's scores
// with a block radix select, so the selection needs no cross-CTA hand-off
// (no counter, no second pass over L2); the result equals the selection
// kernel's sel[row][slot] exactly (the keys are unique).  Uses the unit
// staging region before the unit's copies are issued.
constexpr int64_t kRankMaxTiles = 4096;
__device__ int32_t rank_select(const AttnArgs &a, unsigned char *sm, int64_t row, int slot) {
  const int64_t n = a.rank_n;
  const int kk = (int)(n < a.k_sel ? n : a.k_sel);
  int32_t t = -1;
  if (slot < kk) {
    float *sc = reinterpret_cast<float *>(sm);
    TopkSmem &ts = *reinterpret_cast<TopkSmem *>(sm + kRankMaxTiles * 4);
    const float *src = a.rank_scores + row * n;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
      sc[i] = (i >= a.rank_ex0 && i < a.rank_ex1) ? -INFINITY : __ldcg(src + i);
    __syncthreads();
    KVR_TRACE_POINT(3, 4);
    const unsigned long long key = block_kth_largest<256>([&](int64_t i) -> float { return sc[i]; }, n, slot + 1, ts);
    KVR_TRACE_POINT(3, 5);
    t = (int32_t)key_index(key);
    __syncthreads();  // the region is reused for the unit's copies
  }
  if (threadIdx.x == 0 && a.sel_out != nullptr) a.sel_out[row * a.k_sel + slot] = t;
  return t;
}

static_assert(kRankMaxTiles * 4 + sizeof(TopkSmem) <= AttnSmem::kQ, "in-unit selection must fit the unit region");

// ------------------------------------------------------------- sd1 unit ----
template <int TILE>
__device__ void tile_unit(const AttnArgs &a, unsigned char *sm, int64_t b, int h, int slot, int u) {
  uint32_t *KB = reinterpret_cast<uint32_t *>(sm + AttnSmem::kKB);
  uint32_t *VB = reinterpret_cast<uint32_t *>(sm + AttnSmem::kVB);
  const uint16_t *KS = reinterpret_cast<const uint16_t *>(sm + AttnSmem::kKS);
  const uint16_t *VS = reinterpret_cast<const uint16_t *>(sm + AttnSmem::kVS);
  float *LUT = reinterpret_cast<float *>(sm + AttnSmem::kLUT);
  float *Qs = reinterpret_cast<float *>(sm + AttnSmem::kQ);
  float *S = reinterpret_cast<float *>(sm + AttnSmem::kS);
  float *P = reinterpret_cast<float *>(sm + AttnSmem::kP);
  float *ML = reinterpret_cast<float *>(sm + AttnSmem::kML);
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm + AttnSmem::kBar);
  int *flag = reinterpret_cast<int *>(sm + AttnSmem::kFlag);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = b * a.n_kv + h;
  griddep_wait();  // sel (or the scores) and qprime come from the selection kernel
  KVR_TRACE_POINT(3, 6);
  const int32_t t = a.rank_scores != nullptr ? rank_select(a, sm, row, slot) : a.sel[row * a.k_sel + slot];
  if (t < 0) return;  // empty slot: nothing to fold
  const int64_t tix = row * a.nt_cap + t;
  constexpr unsigned kBits = TILE * 16, kScale = kD * 2;
  if (tid == 0) {
    flag[0] = 1;
    mbar_init(bar, 1);
    mbar_expect_tx(bar, 2 * kBits + 2 * kScale);
    bulk_g2s(KB, a.kbits + tix * TILE * 4, kBits, bar);
    bulk_g2s(VB, a.vbits + tix * TILE * 4, kBits, bar);
    bulk_g2s(sm + AttnSmem::kKS, a.kscale + tix * kD, kScale, bar);
    bulk_g2s(sm + AttnSmem::kVS, a.vscale + tix * kD, kScale, bar);
  }
  // transformed queries while the copies fly
  for (int i = tid; i < a.g * 32; i += blockDim.x) {
    const int hq = i >> 5, qd = i & 31;
    const float4 x =
        __ldg(reinterpret_cast<const float4 *>(a.qprime + (b * a.n_q + (int64_t)h * a.g + hq) * kD) + qd);
    reinterpret_cast<float4 *>(Qs + hq * kD)[qd] =
        make_float4(x.x * a.inv_scale, x.y * a.inv_scale, x.z * a.inv_scale, x.w * a.inv_scale);
  }
  __syncthreads();  // barrier initialised, Qs staged
  KVR_TRACE_POINT(1, 1);
  if (!mbar_wait_bounded(bar, 0)) {
    atomicOr(a.err, 1u);
    flag[0] = 0;  // benign race: every thread that fails writes 0
    mbar_wait_bounded(bar, 0);  // let copies in flight land before smem is reused
  }
  __syncthreads();
  if (!flag[0]) return;  // dropped after a bounded wait gave up (reported via the error word)
  if (warp < a.g) {
    // one warp per query head: nibble LUT, scores, softmax and the bit-serial
    // P.V of this head without block barriers
    const int hq = warp;
    {
      const int grp = lane;
      float av[4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
        av[r] = Qs[hq * kD + 4 * grp + r] * __half2float(__ushort_as_half(KS[4 * grp + r]));
      float *Lw = LUT + (hq * 32 + grp) * 16;
#pragma unroll
      for (int x = 0; x < 16; ++x) {
        float s = 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) s += ((x >> r) & 1) ? av[r] : -av[r];
        Lw[x] = s;
      }
    }
    __syncwarp();
    constexpr int TPLw = TILE / 32;
    const float *Lh = LUT + hq * 32 * 16;
    float sj[TPLw];
#pragma unroll
    for (int r = 0; r < TPLw; ++r) {
      const uint4 w4 = reinterpret_cast<const uint4 *>(KB)[lane + 32 * r];
      const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int grp = 0; grp < 32; ++grp) acc[grp & 3] += Lh[grp * 16 + ((w[grp >> 3] >> (4 * (grp & 7))) & 15u)];
      sj[r] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    }
    float mx = sj[0];
#pragma unroll
    for (int r = 1; r < TPLw; ++r) mx = fmaxf(mx, sj[r]);
    mx = warp_max(mx);
    float l = 0.0f;
#pragma unroll
    for (int r = 0; r < TPLw; ++r) {
      const float p = expf(sj[r] - mx);
      P[(lane + 32 * r) * kMaxG + hq] = p;
      l += p;
    }
    l = warp_sum(l);
    __syncwarp();
    KVR_TRACE_POINT(1, 2);
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int j = 0; j < TILE; ++j) {
      const float pj = P[j * kMaxG + hq];
      const uint4 v4 = reinterpret_cast<const uint4 *>(VB)[j];
      const uint32_t vw[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int mask = (int)(vw[m] << (31 - lane)) >> 31;  // all ones if channel lane + 32 m is set
        o[m] += __int_as_float(__float_as_int(pj) & mask);
      }
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int c = lane + 32 * m;
      S[hq * kD + c] = __half2float(__ushort_as_half(VS[c])) * (2.0f * o[m] - l);
    }
    if (lane == 0) {
      ML[hq * 2] = mx;
      ML[hq * 2 + 1] = l;
    }
    KVR_TRACE_POINT(1, 7);
  }
  __syncthreads();
  if (a.upc == 1 && a.slots > 1) {
    // one unit per CTA: its (m, l, o) is the CTA's partial row
    for (int i = tid; i < a.g * (kD / 4); i += blockDim.x) {
      const int hq = i / (kD / 4), c4 = i - hq * (kD / 4);
      float *pr = part_row(a, row, blockIdx.x, hq);
      reinterpret_cast<float4 *>(pr + kPartEx)[c4] = make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4 *>(pr + kPartTr)[c4] = reinterpret_cast<const float4 *>(S + hq * kD)[c4];
      if (c4 == 0) *reinterpret_cast<float2 *>(pr) = make_float2(ML[2 * hq], ML[2 * hq + 1]);
    }
    if (tid == 0) flag[2] = 1;
    __syncthreads();
    return;
  }
  fold_unit(a, sm, true);
}

// ------------------------------------------------------------- finalize ----
// Ex/Tr: [g][128] exact and transformed sums, ML: [g] (M, L).  Maps Tr back
// with one inverse transform per query head and writes out (or the partial
// rows [m, l, o] for a sequence-split merge).
__device__ void finalize_group(const AttnArgs &a, unsigned char *sm, int64_t b, int h, const float *Ex,
                               const float *Tr, const float *ML, float *buf, bool any_tiles) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float *lee = reinterpret_cast<const float *>(sm + AttnSmem::kLee);
  if (any_tiles && a.kind == KVR_DCT) {
    // strided layout (lane l: elements l + 32 s), the shuffle inverse DCT
    for (int hq = warp; hq < a.g; hq += 8) {
      float x[4];
#pragma unroll
      for (int s = 0; s < 4; ++s) x[s] = Tr[hq * kD + lane + 32 * s];
      dct128_inv_shfl(x, lane, lee);
      KVR_TRACE_POINT(3, 3);
      const int64_t qh = b * a.n_q + (int64_t)h * a.g + hq;
      const float M = ML[hq * 2], L = ML[hq * 2 + 1];
      if (a.partial_out) {
        float *pr = a.partial_out + qh * (kD + 2);
        if (lane == 0) {
          pr[0] = M;
          pr[1] = L;
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) pr[2 + lane + 32 * s] = Ex[hq * kD + lane + 32 * s] + x[s];
      } else {
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const int64_t idx = qh * kD + lane + 32 * s;
          const float y = (Ex[hq * kD + lane + 32 * s] + x[s]) * inv;
          if (a.out_dt == KVR_F32) store_elem<KVR_F32>(a.out, idx, y);
          else if (a.out_dt == KVR_F16) store_elem<KVR_F16>(a.out, idx, y);
          else store_elem<KVR_BF16>(a.out, idx, y);
        }
      }
    }
    return;
  }
  for (int hq = warp; hq < a.g; hq += 8) {
    float x[4];
    const float4 t4 = reinterpret_cast<const float4 *>(Tr + hq * kD)[lane];
    x[0] = t4.x; x[1] = t4.y; x[2] = t4.z; x[3] = t4.w;
    if (any_tiles) transform128(x, lane, a.kind, true, buf + warp * 2 * kD, lee);
    KVR_TRACE_POINT(1, 7);
    const float4 e4 = reinterpret_cast<const float4 *>(Ex + hq * kD)[lane];
    const float y[4] = {e4.x + (any_tiles ? x[0] : 0.f), e4.y + (any_tiles ? x[1] : 0.f),
                        e4.z + (any_tiles ? x[2] : 0.f), e4.w + (any_tiles ? x[3] : 0.f)};
    const int64_t qh = b * a.n_q + (int64_t)h * a.g + hq;
    const float M = ML[hq * 2], L = ML[hq * 2 + 1];
    if (a.partial_out) {
      float *pr = a.partial_out + qh * (kD + 2);
      if (lane == 0) {
        pr[0] = M;
        pr[1] = L;
      }
      reinterpret_cast<float2 *>(pr + 2)[2 * lane] = make_float2(y[0], y[1]);
      reinterpret_cast<float2 *>(pr + 2)[2 * lane + 1] = make_float2(y[2], y[3]);
    } else {
      const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t idx = qh * kD + lane * 4 + r;
        if (a.out_dt == KVR_F32) store_elem<KVR_F32>(a.out, idx, y[r] * inv);
        else if (a.out_dt == KVR_F16) store_elem<KVR_F16>(a.out, idx, y[r] * inv);
        else store_elem<KVR_BF16>(a.out, idx, y[r] * inv);
      }
    }
  }
}

// ---------------------------------------------------------------- merge ----
// Run by the last CTA of a (b, h) when several CTAs share its units: one L2
// round trip for the slot rows (o loads in registers while other threads
// stage the slots' (m, l) in shared memory).
__device__ void merge_slots(const AttnArgs &a, unsigned char *sm, int64_t b, int h, bool any_tiles) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = b * a.n_kv + h;
  const int NS = a.slots;
  // layout (the unit staging region is free now): WL [NS][8] float2 | Ex | Tr | buf
  float2 *WL = reinterpret_cast<float2 *>(sm);
  float *Ex = reinterpret_cast<float *>(sm) + 2 * NS * kMaxG;
  float *Tr = Ex + kMaxG * kD;
  float *buf = Tr + kMaxG * kD;
  float *ML = reinterpret_cast<float *>(sm + AttnSmem::kML);
  constexpr int UB = 8;
  const int pairs = a.g * 32;
  const int nparts = blockDim.x / pairs;  // 2 for g = 4, 1 for g = 8
  const int p = tid % pairs, part = tid / pairs;
  const int hq = p >> 5, c4 = p & 31;
  float4 ex = make_float4(0.f, 0.f, 0.f, 0.f), tr = ex;
  // (m, l) of every slot -> per-head weights exp(m - M) and the merged (M, L)
  auto slot_ml_loads = [&]() {
    for (int i = tid; i < NS * a.g; i += blockDim.x) {
      const int s = i / a.g, h2 = i - s * a.g;
      WL[s * kMaxG + h2] = __ldcg(reinterpret_cast<const float2 *>(part_row(a, row, s, h2)));
    }
  };
  bool ml_loaded = false;
  auto slot_weights = [&]() {
    if (!ml_loaded) slot_ml_loads();
    __syncthreads();
    for (int h2 = warp; h2 < a.g; h2 += 8) {
      float mx = -INFINITY;
      for (int s = lane; s < NS; s += 32) mx = fmaxf(mx, WL[s * kMaxG + h2].x);
      mx = warp_max(mx);
      float l = 0.0f;
      for (int s = lane; s < NS; s += 32) {
        const float2 v = WL[s * kMaxG + h2];
        const float w = (v.x == -INFINITY) ? 0.0f : expf(v.x - mx);
        WL[s * kMaxG + h2].x = w;  // (m, l) -> (weight, l)
        l += w * v.y;
      }
      l = warp_sum(l);
      if (lane == 0) {
        ML[h2 * 2] = mx;
        ML[h2 * 2 + 1] = l;
      }
    }
    __syncthreads();
  };
  // One unit per CTA: a slot carries an exact-domain part (window / tail
  // unit) or a transformed part (tile unit), never both.  The halves that
  // matter are copied into shared memory with asynchronous copies issued
  // together with the (m, l) loads: one round trip, no registers held.
  constexpr int kStage = 18432;
  const int n_exact = a.nchunk[0] + a.nchunk[1];
  const bool staged = a.upc == 1 && 2 * NS * kMaxG * 4 + 4 * kMaxG * kD * 4 <= kStage &&
                      kStage + NS * a.g * 512 <= AttnSmem::kQ;
  if (staged) {
    // the (m, l) pairs first: the weights are formed while the bulk halves travel
    slot_ml_loads();
    ml_loaded = true;
    float4 *stg = reinterpret_cast<float4 *>(sm + kStage);
    for (int idx = tid; idx < NS * a.g * 32; idx += blockDim.x) {
      const int s = idx / (a.g * 32), r = idx - s * a.g * 32;
      const float *src = part_row(a, row, s, r >> 5) + (s < n_exact ? kPartEx : kPartTr) + 4 * (r & 31);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(stg + idx)), "l"(src) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    slot_weights();
    KVR_TRACE_POINT(3, 0);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    KVR_TRACE_POINT(3, 1);
    if (part < nparts)
      for (int s = part; s < NS; s += nparts) {
        const float4 v = stg[(s * a.g + hq) * 32 + c4];
        const float w = WL[s * kMaxG + hq].x;
        if (s < n_exact) {
          ex.x = fmaf(w, v.x, ex.x); ex.y = fmaf(w, v.y, ex.y); ex.z = fmaf(w, v.z, ex.z); ex.w = fmaf(w, v.w, ex.w);
        } else {
          tr.x = fmaf(w, v.x, tr.x); tr.y = fmaf(w, v.y, tr.y); tr.z = fmaf(w, v.z, tr.z); tr.w = fmaf(w, v.w, tr.w);
        }
      }
  }
  for (int s0 = 0; s0 < (staged ? 0 : NS); s0 += UB * nparts) {
    float4 oe[UB], ot[UB];
#pragma unroll
    for (int k = 0; k < UB; ++k) {
      const int s = s0 + part + nparts * k;
      const bool ok = part < nparts && s < NS;
      const float *pr = ok ? part_row(a, row, s, hq) : nullptr;
      oe[k] = ok ? __ldcg(reinterpret_cast<const float4 *>(pr + kPartEx) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
      ot[k] = ok ? __ldcg(reinterpret_cast<const float4 *>(pr + kPartTr) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (s0 == 0) slot_weights();
#pragma unroll
    for (int k = 0; k < UB; ++k) {
      const int s = s0 + part + nparts * k;
      if (part >= nparts || s >= NS) break;
      const float w = WL[s * kMaxG + hq].x;
      ex.x = fmaf(w, oe[k].x, ex.x); ex.y = fmaf(w, oe[k].y, ex.y);
      ex.z = fmaf(w, oe[k].z, ex.z); ex.w = fmaf(w, oe[k].w, ex.w);
      tr.x = fmaf(w, ot[k].x, tr.x); tr.y = fmaf(w, ot[k].y, tr.y);
      tr.z = fmaf(w, ot[k].z, tr.z); tr.w = fmaf(w, ot[k].w, tr.w);
    }
  }
  for (int q = 0; q < nparts; ++q) {
    if (part == q) {
      float4 *e = reinterpret_cast<float4 *>(Ex + hq * kD) + c4;
      float4 *t = reinterpret_cast<float4 *>(Tr + hq * kD) + c4;
      if (q == 0) {
        *e = ex;
        *t = tr;
      } else {
        const float4 e0 = *e, t0 = *t;
        *e = make_float4(e0.x + ex.x, e0.y + ex.y, e0.z + ex.z, e0.w + ex.w);
        *t = make_float4(t0.x + tr.x, t0.y + tr.y, t0.z + tr.z, t0.w + tr.w);
      }
    }
    __syncthreads();
  }
  KVR_TRACE_POINT(1, 6);
  finalize_group(a, sm, b, h, Ex, Tr, ML, buf, any_tiles);
}

// End of a CTA's units: the CTA accumulators (kAccM/L/Ex/Tr) hold its
// result.  A CTA that owns the whole row finalizes it; otherwise it writes its
// partial rows and the last CTA of the row merges them.
__device__ void attn_finish(const AttnArgs &a, unsigned char *sm, int64_t b, int h) {
  const int tid = threadIdx.x;
  const int64_t row = b * a.n_kv + h;
  const int slot = blockIdx.x;
  const int n_exact = a.nchunk[0] + a.nchunk[1];
  float *AM = reinterpret_cast<float *>(sm + AttnSmem::kAccM);
  float *AL = reinterpret_cast<float *>(sm + AttnSmem::kAccL);
  float *AEx = reinterpret_cast<float *>(sm + AttnSmem::kAccEx);
  float *ATr = reinterpret_cast<float *>(sm + AttnSmem::kAccTr);
  const bool any_tiles = a.units > n_exact;
  if (a.slots == 1) {
    // this CTA owns every unit of its row: no partials, no merge
    float *ML = reinterpret_cast<float *>(sm + AttnSmem::kML);
    if (tid < a.g) {
      ML[2 * tid] = AM[tid];
      ML[2 * tid + 1] = AL[tid];
    }
    __syncthreads();
    finalize_group(a, sm, b, h, AEx, ATr, ML, reinterpret_cast<float *>(sm), any_tiles);
    return;
  }
  // write this CTA's partial rows, then the last CTA of the row merges
  const bool written = reinterpret_cast<const int *>(sm + AttnSmem::kFlag)[2] != 0;
  if (!written)
  for (int i = tid; i < a.g * (kD / 4); i += blockDim.x) {
    const int hq = i / (kD / 4), c4 = i - hq * (kD / 4);
    float *pr = part_row(a, row, slot, hq);
    reinterpret_cast<float4 *>(pr + kPartEx)[c4] = reinterpret_cast<const float4 *>(AEx + hq * kD)[c4];
    reinterpret_cast<float4 *>(pr + kPartTr)[c4] = reinterpret_cast<const float4 *>(ATr + hq * kD)[c4];
    if (c4 == 0) *reinterpret_cast<float2 *>(pr) = make_float2(AM[hq], AL[hq]);
  }
  __syncthreads();
  int *last = reinterpret_cast<int *>(sm + AttnSmem::kFlag) + 1;
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&a.counters[row], 1u);
    *last = (prev == (unsigned)a.slots - 1);
  }
  __syncthreads();
  if (!*last) return;
  __threadfence();
  KVR_TRACE_POINT(1, 4);
  merge_slots(a, sm, b, h, any_tiles);
  KVR_TRACE_POINT(1, 5);
  if (tid == 0) a.counters[row] = 0u;
}

template <int TILE>
__global__ void __launch_bounds__(256) attn_kernel(AttnArgs a) {
  extern __shared__ __align__(128) unsigned char sm[];
  const int slot = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t row = b * a.n_kv + h;
  const int tid = threadIdx.x;
  KVR_TRACE_POINT(1, 0);
  // the next layer's selection kernel may start its store loads now; it
  // waits for this kernel to finish before it reads q or writes anything
  asm volatile("griddepcontrol.launch_dependents;");
  if (a.kind == KVR_DCT) load_lee(reinterpret_cast<float *>(sm + AttnSmem::kLee));
  float *AM = reinterpret_cast<float *>(sm + AttnSmem::kAccM);
  float *AL = reinterpret_cast<float *>(sm + AttnSmem::kAccL);
  float *AEx = reinterpret_cast<float *>(sm + AttnSmem::kAccEx);
  float *ATr = reinterpret_cast<float *>(sm + AttnSmem::kAccTr);
  for (int i = tid; i < a.g * kD; i += blockDim.x) {
    AEx[i] = 0.0f;
    ATr[i] = 0.0f;
  }
  if (tid < a.g) {
    AM[tid] = -INFINITY;
    AL[tid] = 0.0f;
  }
  if (tid == 0) reinterpret_cast<int *>(sm + AttnSmem::kFlag)[2] = 0;  // partial row written by the unit
  __syncthreads();
  const int n_exact = a.nchunk[0] + a.nchunk[1];
  const int u_end = min(a.units, (slot + 1) * a.upc);
  for (int u = slot * a.upc; u < u_end; ++u) {
    if (u < a.nchunk[0]) {
      exact_unit(a, sm, b, h, 0, u, u);
    } else if (u < n_exact) {
      exact_unit(a, sm, b, h, 1, u - a.nchunk[0], u);
    } else {
      tile_unit<TILE>(a, sm, b, h, u - n_exact, u);
    }
    __syncthreads();
  }
  KVR_TRACE_POINT(1, 3);
  attn_finish(a, sm, b, h);
}

// ------------------------------------------------------ batched decode ----
// Many (b, h) rows (batched decode, bandwidth-bound).  The units of a CTA are
// cut into 32-token pieces (half a 64-token exact chunk, or a 32-token slice
// of a selected tile) that its 8 warps take round-robin, so no barrier is
// crossed until the CTA's last piece is done.  Every warp keeps its own online
// softmax state and computes both products of a piece on the tensor cores
// (mma.sync m16n8k16, fp16 operands, fp32 accumulation):
//   S^T = K q^T   M = 32 tokens, N = 8 query heads, K = 128 channels
//   O^T = V^T P^T M = 128 channels, N = 8 query heads, K = 16 tokens a step
// K, V (fp16 rows) and the sd1 values +-scale are exact in fp16; q and P are
// split into fp16 hi + lo parts (two MMAs), which keeps about 22 bits.  q is
// first scaled by a power of two per row so that both parts stay in fp16
// range.  Lane l = 4 g + t reads its A fragments straight from memory: exact
// rows as 16-byte loads (channels paired as (c, c+1)); sd1 rows as bit words,
// with channels paired as (c, c+16) so that one shift and mask of a word gives
// the two sign bits of a half2 register.  Its accumulator holds channels
// 16 g .. 16 g + 15 of heads 2t, 2t+1 (exact pieces in the natural domain, sd1
// pieces in the transformed domain).  A warp's exact pieces come before its
// sd1 pieces: at the switch the exact sum is parked in shared memory with the
// running max it is relative to.  At the end the warp states are folded into
// the CTA accumulators in warp order.
constexpr int kPiece = 32;
constexpr int kPStride = 40;  // halves per head row of the P staging (conflict-free B loads)
struct RowSmem {
  static constexpr int kFm = 0;                              // fp32 [8 warps][8] running max at the end
  static constexpr int kFl = kFm + 8 * kMaxG * 4;            // fp32 [8][8] running sum
  static constexpr int kFs = kFl + 8 * kMaxG * 4;            // fp32 [8][8] max of the parked sum
  static constexpr int kFex = kFs + 8 * kMaxG * 4;           // fp32 [8 warps][8][128] parked exact sums
  static constexpr int kQBx = kFex + 8 * kMaxG * kD * 4;     // uint4 [8 k-steps][32 lanes] q B fragments
  static constexpr int kQBt = kQBx + 8 * 32 * 16;            // uint4 [8][32] q' B fragments
  static constexpr int kP = kQBt + 8 * 32 * 16;              // per warp: fp16 [hi, lo][8 heads][40]
  static constexpr int kPWarp = 2 * kMaxG * kPStride * 2;
  static constexpr int kSc = kP + 8 * kPWarp;                // per warp: fp16 [-ks, -vs][128]
  static constexpr int kEnd = kSc + 8 * 2 * kD * 2;
  static constexpr int kFtr = kQBx;                          // fp32 [8][8][128], after every warp is done
  static constexpr int kFEnd = kFtr + 8 * kMaxG * kD * 4;
  static constexpr int kRed = kFEnd;                         // fp32 [8] max |q| per warp (start only)
};
static_assert(RowSmem::kEnd <= AttnSmem::kQ && RowSmem::kFEnd + 64 <= AttnSmem::kQ,
              "batched decode staging must stay inside the unit region");
// In-kernel selection of the batched path: scores (<= kRowsRankMax), the
// warp lists and the candidates in the parked-sum region, the chosen tiles
// (<= 32) after the piece staging.
constexpr int64_t kRowsRankMax = 4096;
constexpr int kRowsRankMaxK = 32;
static_assert(4 * kRowsRankMax + 8 * 32 * 8 + kRowsRankMaxK * 8 <= RowSmem::kQBx - RowSmem::kFex &&
                  RowSmem::kEnd + 4 * kRowsRankMaxK <= AttnSmem::kQ,
              "batched in-kernel selection must fit the free staging");

__device__ __forceinline__ void hmma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// x -> fp16 hi + lo (x = hi + lo to about 22 bits for |x| in fp16 range)
__device__ __forceinline__ void split_f16(float x0, float x1, uint32_t &hi, uint32_t &lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  hi = h2u(h);
  lo = h2u(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}

// sign bits of the half2 pair (bit c -> bit 15, bit c + 16 -> bit 31) applied to -scale
__device__ __forceinline__ uint32_t sgn_pair(uint32_t neg_scale2, uint32_t w_shifted) {
  return neg_scale2 ^ (w_shifted & 0x80008000u);
}

struct RowState {
  float m[2], l[2];  // running max / sum of query heads 2t, 2t+1
  float o[8][4];     // m-tile j: (channel 16g + 2j, heads 2t, 2t+1), (16g + 2j + 1, heads 2t, 2t+1)
};

// Online softmax of a piece's scores s[mt][r] (token 16 mt + g (+8 for r >= 2),
// head 2t + (r & 1); log2 units: the scores carry a factor log2(e)), then P
// (hi, lo) into the warp's staging.
__device__ __forceinline__ void row_softmax(RowState &st, float (&s)[2][4], __half *Ph, int nt, int g_heads) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int tok = 16 * mt + g + (r >= 2 ? 8 : 0), hq = 2 * t + (r & 1);
      if (tok >= nt || hq >= g_heads) s[mt][r] = -INFINITY;
    }
  float al[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    float pm = fmaxf(fmaxf(s[0][e], s[0][e + 2]), fmaxf(s[1][e], s[1][e + 2]));
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o));
    const float mn = fmaxf(st.m[e], pm);
    al[e] = st.m[e] == -INFINITY ? 0.0f : exp2f(st.m[e] - mn);
    float ps = 0.0f;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int r = e + 2 * rr;
        const float p = s[mt][r] == -INFINITY ? 0.0f : exp2f(s[mt][r] - mn);
        s[mt][r] = p;
        ps += p;
      }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    st.l[e] = fmaf(st.l[e], al[e], ps);
    st.m[e] = mn;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    st.o[j][0] *= al[0];
    st.o[j][1] *= al[1];
    st.o[j][2] *= al[0];
    st.o[j][3] *= al[1];
  }
  // P[head][token] as fp16 hi / lo
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int tok = 16 * mt + g + (r >= 2 ? 8 : 0), hq = 2 * t + (r & 1);
      const __half hi = __float2half_rn(s[mt][r]);
      Ph[hq * kPStride + tok] = hi;
      Ph[(kMaxG + hq) * kPStride + tok] = __float2half_rn(s[mt][r] - __half2float(hi));
    }
  __syncwarp();
}

// O^T += V^T P^T for one 16-token step: A fragments of m-tile j from the
// packed pairs (token 2t, 2t+1) and (2t+8, 2t+9) of channel 16g + 2j (+1).
template <bool PLO, typename AF>
__device__ __forceinline__ void row_pv_step(RowState &st, const __half *Ph, int k0, AF a_frag) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t *P32 = reinterpret_cast<const uint32_t *>(Ph);
  const uint32_t bh0 = P32[(g * kPStride + k0 + 2 * t) >> 1];
  const uint32_t bh1 = P32[(g * kPStride + k0 + 2 * t + 8) >> 1];
  const uint32_t bl0 = P32[((kMaxG + g) * kPStride + k0 + 2 * t) >> 1];
  const uint32_t bl1 = P32[((kMaxG + g) * kPStride + k0 + 2 * t + 8) >> 1];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint32_t a0, a1, a2, a3;
    a_frag(j, a0, a1, a2, a3);
    hmma16816(st.o[j], a0, a1, a2, a3, bh0, bh1);
    if (PLO) hmma16816(st.o[j], a0, a1, a2, a3, bl0, bl1);
  }
}

// Exact piece: nt fp16 rows at kp / vp (token stride ts, elements).
template <bool PLO>
__device__ __forceinline__ void row_piece_exact(RowState &st, const uint4 *QB, __half *Ph, int nt, const __half *kp,
                                                const __half *vp, int64_t ts, float sscale, int g_heads) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  // scores: rows g, g + 8 of both m-tiles, channels 32p + 8t .. +8; both
  // m-tiles' rows in one round trip, four independent MMA chains (m-tile x
  // hi / lo part of q)
  uint4 kr[2][2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int r = 16 * mt + g + 8 * rh;
#pragma unroll
      for (int p = 0; p < 4; ++p)
        kr[mt][rh][p] = r < nt ? __ldg(reinterpret_cast<const uint4 *>(kp + r * ts + 32 * p + 8 * t))
                               : make_uint4(0u, 0u, 0u, 0u);
    }
  float ch[2][4] = {}, cl[2][4] = {};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint4 q0 = QB[(2 * p) * 32 + lane], q1 = QB[(2 * p + 1) * 32 + lane];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint4 &ka = kr[mt][0][p], &kb = kr[mt][1][p];
      hmma16816(ch[mt], ka.x, kb.x, ka.y, kb.y, q0.x, q0.y);
      hmma16816(cl[mt], ka.x, kb.x, ka.y, kb.y, q0.z, q0.w);
      hmma16816(ch[mt], ka.z, kb.z, ka.w, kb.w, q1.x, q1.y);
      hmma16816(cl[mt], ka.z, kb.z, ka.w, kb.w, q1.z, q1.w);
    }
  }
  float s[2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int r = 0; r < 4; ++r) s[mt][r] = (ch[mt][r] + cl[mt][r]) * sscale;
  // V rows of the 4 tokens 2t, 2t+1, 2t+8, 2t+9 of each step, channels 16g .. +16
  uint4 vr[2][4][2];
#pragma unroll
  for (int k = 0; k < 2; ++k)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = 16 * k + 2 * t + (i & 1) + (i >> 1) * 8;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        vr[k][i][hh] = tok < nt ? __ldg(reinterpret_cast<const uint4 *>(vp + tok * ts + 16 * g + 8 * hh))
                                : make_uint4(0u, 0u, 0u, 0u);
    }
  row_softmax(st, s, Ph, nt, g_heads);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    auto word = [&](int i, int j) -> uint32_t {  // channels 16g + 2j, 2j + 1 of token i
      const uint4 &u = vr[k][i][j >> 2];
      const int e = j & 3;
      return e == 0 ? u.x : (e == 1 ? u.y : (e == 2 ? u.z : u.w));
    };
    row_pv_step<PLO>(st, Ph, 16 * k, [&](int j, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
      a0 = __byte_perm(word(0, j), word(1, j), 0x5410);
      a1 = __byte_perm(word(0, j), word(1, j), 0x7632);
      a2 = __byte_perm(word(2, j), word(3, j), 0x5410);
      a3 = __byte_perm(word(2, j), word(3, j), 0x7632);
    });
  }
  __syncwarp();
}

// sd1 piece: 32 token rows of 4 bit words at kw / vw, the tile's fp16 scales
// at ksg / vsg; SC = the warp's staging for the negated scales.
template <bool PLO>
__device__ __forceinline__ void row_piece_sd1(RowState &st, const uint4 *QB, __half *Ph, const uint32_t *kw,
                                              const uint32_t *vw, const uint16_t *ksg, const uint16_t *vsg,
                                              __half *SC, float sscale, int g_heads) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  // one round trip: the scales, the K words of rows g, g+8 of both m-tiles
  // and the V words (word g / 2) of tokens 2t, 2t+1, 2t+8, 2t+9 of each step
  const uint2 ksr = __ldg(reinterpret_cast<const uint2 *>(ksg) + lane);
  const uint2 vsr = __ldg(reinterpret_cast<const uint2 *>(vsg) + lane);
  uint32_t kwd[2][2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int rh = 0; rh < 2; ++rh)
#pragma unroll
      for (int p = 0; p < 4; ++p) kwd[mt][rh][p] = __ldg(kw + (16 * mt + g + 8 * rh) * 4 + p);
  uint32_t vwd[2][4];
#pragma unroll
  for (int k = 0; k < 2; ++k)
#pragma unroll
    for (int i = 0; i < 4; ++i) vwd[k][i] = __ldg(vw + (16 * k + 2 * t + (i & 1) + (i >> 1) * 8) * 4 + (g >> 1));
  // negated scales into the warp's staging, then gathered in fragment order
  reinterpret_cast<uint2 *>(SC)[lane] = make_uint2(ksr.x ^ 0x80008000u, ksr.y ^ 0x80008000u);
  reinterpret_cast<uint2 *>(SC + kD)[lane] = make_uint2(vsr.x ^ 0x80008000u, vsr.y ^ 0x80008000u);
  __syncwarp();
  // -ks pairs (32p + 8s + t, +16) and (32p + 8s + 4 + t, +16) of k-step 2p + s
  uint32_t ksp[8][2];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int c0 = 32 * (kk >> 1) + 8 * (kk & 1) + t;
    ksp[kk][0] = h2u(__halves2half2(SC[c0], SC[c0 + 16]));
    ksp[kk][1] = h2u(__halves2half2(SC[c0 + 4], SC[c0 + 20]));
  }
  float ch[2][4] = {}, cl[2][4] = {};
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int p = kk >> 1, c0 = 8 * (kk & 1) + t;
    const uint4 q = QB[kk * 32 + lane];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint32_t a0 = sgn_pair(ksp[kk][0], kwd[mt][0][p] << (15 - c0));
      const uint32_t a1 = sgn_pair(ksp[kk][0], kwd[mt][1][p] << (15 - c0));
      const uint32_t a2 = sgn_pair(ksp[kk][1], kwd[mt][0][p] << (11 - c0));
      const uint32_t a3 = sgn_pair(ksp[kk][1], kwd[mt][1][p] << (11 - c0));
      hmma16816(ch[mt], a0, a1, a2, a3, q.x, q.y);
      hmma16816(cl[mt], a0, a1, a2, a3, q.z, q.w);
    }
  }
  float s[2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int r = 0; r < 4; ++r) s[mt][r] = (ch[mt][r] + cl[mt][r]) * sscale;
  // -vs of channels 16g + 2j (even) and + 1 (odd), both halves
  uint32_t vse[8], vso[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __half e = SC[kD + 16 * g + 2 * j], o = SC[kD + 16 * g + 2 * j + 1];
    vse[j] = h2u(__halves2half2(e, e));
    vso[j] = h2u(__halves2half2(o, o));
  }
  row_softmax(st, s, Ph, kPiece, g_heads);
  const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;  // this lane's 16 channels are half g & 1 of the word
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint32_t x01 = __byte_perm(vwd[k][0], vwd[k][1], sel);
    const uint32_t x23 = __byte_perm(vwd[k][2], vwd[k][3], sel);
    row_pv_step<PLO>(st, Ph, 16 * k, [&](int j, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
      a0 = sgn_pair(vse[j], x01 << (15 - 2 * j));
      a1 = sgn_pair(vso[j], x01 << (14 - 2 * j));
      a2 = sgn_pair(vse[j], x23 << (15 - 2 * j));
      a3 = sgn_pair(vso[j], x23 << (14 - 2 * j));
    });
  }
  __syncwarp();
}

// q B fragments of one k-step for lane l = 4g + t (head g): natural channel
// pairs for exact K (pairs ch, ch + 1 at 32p + 8t + 4s) or (c, c + 16) pairs at
// 32p + 8s + t (+4) for sd1 K.  q is multiplied by the power of two qsc.
__device__ __forceinline__ uint4 q_bfrag(const float *Qrow, int kk, int lane, bool sd1, float qsc) {
  const int t = lane & 3, p = kk >> 1, s = kk & 1;
  float x[4];
  if (!sd1) {
    const int c = 32 * p + 8 * t + 4 * s;
    x[0] = Qrow[c]; x[1] = Qrow[c + 1]; x[2] = Qrow[c + 2]; x[3] = Qrow[c + 3];
  } else {
    const int c = 32 * p + 8 * s + t;
    x[0] = Qrow[c]; x[1] = Qrow[c + 16]; x[2] = Qrow[c + 4]; x[3] = Qrow[c + 20];
  }
  uint4 r;
  split_f16(x[0] * qsc, x[1] * qsc, r.x, r.z);
  split_f16(x[2] * qsc, x[3] * qsc, r.y, r.w);
  return r;
}

// power of two bringing max |q| near 2^12 (fp16 range for hi, normal range for lo)
__device__ __forceinline__ float pow2_scale(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 1.0f;
  int e;
  frexpf(amax, &e);  // amax in [2^(e-1), 2^e)
  return ldexpf(1.0f, 12 - e);
}

// PLO: the P.V products also take the fp16 low part of P (fp32 and fp16
// outputs, partial rows); a bf16 output rounds at 2^-9, far above the 2^-12
// of the high part alone.
template <int TILE, bool PLO>
__global__ void __launch_bounds__(256, 2) attn_rows_kernel(AttnArgs a) {
  extern __shared__ __align__(128) unsigned char sm[];
  const int slot = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t row = b * a.n_kv + h;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int n_exact = a.nchunk[0] + a.nchunk[1];
  KVR_TRACE_POINT(1, 0);
  asm volatile("griddepcontrol.launch_dependents;");
  if (a.kind == KVR_DCT) load_lee(reinterpret_cast<float *>(sm + AttnSmem::kLee));
  if (tid == 0) reinterpret_cast<int *>(sm + AttnSmem::kFlag)[2] = 0;
  // q of the group staged as fp32 rows (rows of heads >= g zero).  q is
  // ready before the preceding selection kernel started, so the window /
  // tail pieces run while that kernel finishes; q' and the selection are
  // read after the grid dependency wait below.
  float *Qs = reinterpret_cast<float *>(sm + AttnSmem::kQ);   // fp32 [8][128]
  float *Qps = reinterpret_cast<float *>(sm + AttnSmem::kS);  // fp32 [8][128]
  float *red = reinterpret_cast<float *>(sm + RowSmem::kRed);
  const bool any_tiles = a.units > n_exact;
  // stage the group's rows of q (sd1 = false) or q' (sd1 = true) as B
  // fragments, multiplied by the power of two that brings max |.| near 2^12
  auto stage_bfrags = [&](bool sd1, float *rows, uint4 *QB) -> float {
    float amx = 0.0f;
    for (int i = tid; i < kMaxG * 32; i += blockDim.x) {
      const int hq = i >> 5, qd = i & 31;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (hq < a.g) {
        const int64_t qh = b * a.n_q + (int64_t)h * a.g + hq;
        x = sd1 ? __ldcg(reinterpret_cast<const float4 *>(a.qprime + qh * kD) + qd)
                : cvt4(raw4(a.q, qh * kD + qd * 4, a.q_dt), a.q_dt);
      }
      amx = fmaxf(amx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
      reinterpret_cast<float4 *>(rows + hq * kD)[qd] = x;
    }
    amx = warp_max(amx);
    if (lane == 0) red[(sd1 ? 8 : 0) + warp] = amx;
    __syncthreads();
    float qs = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) qs = fmaxf(qs, red[(sd1 ? 8 : 0) + w]);
    qs = pow2_scale(qs);
    const int kk = tid >> 5;  // 8 k-steps x 32 lanes = 256 threads
    QB[kk * 32 + lane] = q_bfrag(rows + g * kD, kk, lane, sd1, qs);
    __syncthreads();
    return qs;
  };
  uint4 *QBx = reinterpret_cast<uint4 *>(sm + RowSmem::kQBx);
  uint4 *QBt = reinterpret_cast<uint4 *>(sm + RowSmem::kQBt);
  const float qsx = stage_bfrags(false, Qs, QBx);
  KVR_TRACE_POINT(1, 1);
  constexpr float kLog2e = 1.4426950408889634f;
  const float sx = a.inv_scale * kLog2e / qsx;
  float stl = 0.0f;

  RowState st;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) st.o[j][i] = 0.0f;
  __half *Ph = reinterpret_cast<__half *>(sm + RowSmem::kP + warp * RowSmem::kPWarp);
  __half *SC = reinterpret_cast<__half *>(sm + RowSmem::kSc) + warp * 2 * kD;
  float *Fex = reinterpret_cast<float *>(sm + RowSmem::kFex) + warp * kMaxG * kD;
  float m_park[2] = {-INFINITY, -INFINITY};
  bool parked = false;
  // the accumulator's (channel, head) entries as [head][channel] rows
  auto store_acc = [&](float *dst) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = 16 * g + 2 * j;
      dst[(2 * t) * kD + c] = st.o[j][0];
      dst[(2 * t + 1) * kD + c] = st.o[j][1];
      dst[(2 * t) * kD + c + 1] = st.o[j][2];
      dst[(2 * t + 1) * kD + c + 1] = st.o[j][3];
    }
  };
  auto park = [&]() {
    store_acc(Fex);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) st.o[j][i] = 0.0f;
    m_park[0] = st.m[0];
    m_park[1] = st.m[1];
    parked = true;
  };

  const int u0 = slot * a.upc, u1 = min(a.units, u0 + a.upc);
  const int ex_units = max(0, min(u1, n_exact) - u0);
  constexpr int PPT = TILE / kPiece;  // pieces per tile
  const int n_pieces = 2 * ex_units + PPT * max(0, u1 - u0 - ex_units);
  // The row's selected tiles: from the selection kernel (a.sel), or, with
  // rank scores given, the top k_sel of the row's tile scores picked here
  // after the grid dependency wait (the same keys and order as the selection
  // kernel's pick), into RS.
  const bool rank_rows = a.rank_scores != nullptr && any_tiles;
  int32_t *RS = reinterpret_cast<int32_t *>(sm + RowSmem::kEnd);
  auto tile_of = [&](int j) -> int32_t { return rank_rows ? RS[j] : __ldcg(a.sel + row * a.k_sel + j); };
  // Every piece of this warp is requested into L2 first (no registers held):
  // the loads of the pieces then wait for L2 instead of a DRAM round trip each.
  // Exact pieces (pc < 2 * ex_units) come first in every warp's sequence.
  auto prefetch_pieces = [&](int pc0, int pc1) {
    for (int pc = pc0; pc < pc1; pc += 8) {
      if (pc < 2 * ex_units) {
        const int u = u0 + pc / 2;
        const int seg = u < a.nchunk[0] ? 0 : 1;
        const int64_t t0 = (int64_t)(seg == 0 ? u : u - a.nchunk[0]) * kChunk + (pc & 1) * kPiece;
        if (t0 + lane < a.n[seg]) {
          const int64_t off = b * a.batch_stride[seg] + (int64_t)h * kD + (t0 + lane) * a.tok_stride[seg];
          prefetch_l2(reinterpret_cast<const __half *>(a.k[seg]) + off, kD * 2);
          prefetch_l2(reinterpret_cast<const __half *>(a.v[seg]) + off, kD * 2);
        }
      } else if (lane < 4) {
        const int r = pc - 2 * ex_units;
        const int u = u0 + ex_units + r / PPT, sub = r % PPT;
        const int32_t tsel = tile_of(u - n_exact);
        if (tsel >= 0) {
          const int64_t tix = row * a.nt_cap + tsel;
          const int64_t w0 = (tix * TILE + sub * kPiece) * 4;
          if (lane == 0) prefetch_l2(a.kbits + w0, kPiece * 16);
          if (lane == 1) prefetch_l2(a.vbits + w0, kPiece * 16);
          if (lane == 2) prefetch_l2(a.kscale + tix * kD, kD * 2);
          if (lane == 3) prefetch_l2(a.vscale + tix * kD, kD * 2);
        }
      }
    }
  };
  // first sd1 piece of this warp's sequence
  const int pc_t = warp >= 2 * ex_units ? warp : warp + (2 * ex_units - warp + 7) / 8 * 8;
  prefetch_pieces(warp, min(n_pieces, 2 * ex_units));
  for (int pc = warp; pc < min(n_pieces, 2 * ex_units); pc += 8) {
    const int u = u0 + pc / 2;
    const int seg = u < a.nchunk[0] ? 0 : 1;
    const int chunk = seg == 0 ? u : u - a.nchunk[0];
    const int64_t t0 = (int64_t)chunk * kChunk + (pc & 1) * kPiece;
    const int64_t left = a.n[seg] - t0;
    if (left <= 0) continue;
    const int nt = (int)(left < kPiece ? left : kPiece);
    const int64_t base = b * a.batch_stride[seg] + (int64_t)h * kD + t0 * a.tok_stride[seg];
    row_piece_exact<PLO>(st, QBx, Ph, nt, reinterpret_cast<const __half *>(a.k[seg]) + base,
                         reinterpret_cast<const __half *>(a.v[seg]) + base, a.tok_stride[seg], sx, a.g);
  }
  // q' and the selection come from the preceding kernel
  griddep_wait();
  if (rank_rows) {
    // the parked-sum region is free until the first tile piece
    float *sc = reinterpret_cast<float *>(sm + RowSmem::kFex);
    unsigned long long *lists = reinterpret_cast<unsigned long long *>(sm + RowSmem::kFex + 4 * kRowsRankMax);
    unsigned long long *cand = lists + 8 * 32;
    const int64_t n = a.rank_n;
    const int kk = (int)(n < a.k_sel ? n : a.k_sel);
    const float *src = a.rank_scores + row * n;
    for (int64_t i = tid; i < n; i += blockDim.x)
      sc[i] = (i >= a.rank_ex0 && i < a.rank_ex1) ? -INFINITY : __ldcg(src + i);
    __syncthreads();
    if (kk > 0) block_topk_warp32<256>(sc, n, kk, lists, cand);
    if (tid < a.k_sel) {
      const int32_t v = tid < kk ? (int32_t)key_index(cand[tid]) : -1;
      RS[tid] = v;
      if (slot == 0 && a.sel_out != nullptr) a.sel_out[row * a.k_sel + tid] = v;
    }
    __syncthreads();
  }
  if (any_tiles) {
    const float qst = stage_bfrags(true, Qps, QBt);  // block-wide: every warp arrives here
    stl = a.inv_scale * kLog2e / qst;
    prefetch_pieces(pc_t, n_pieces);
  }
  for (int pc = pc_t; pc < n_pieces; pc += 8) {
    if (!parked) park();
    const int r = pc - 2 * ex_units;
    const int u = u0 + ex_units + r / PPT, sub = r % PPT;
    const int32_t tsel = tile_of(u - n_exact);
    if (tsel < 0) continue;
    const int64_t tix = row * a.nt_cap + tsel;
    const int64_t w0 = (tix * TILE + sub * kPiece) * 4;
    row_piece_sd1<PLO>(st, QBt, Ph, a.kbits + w0, a.vbits + w0, a.kscale + tix * kD, a.vscale + tix * kD, SC,
                       stl, a.g);
  }
  if (!parked) park();  // only exact pieces (or none): the sd1 sum is zero

  // fold the 8 warp states into the CTA accumulators (warp order)
  __syncthreads();  // the B fragments and P staging are dead from here on
  KVR_TRACE_POINT(1, 2);
  float *Ftr = reinterpret_cast<float *>(sm + RowSmem::kFtr);
  float *Fm = reinterpret_cast<float *>(sm + RowSmem::kFm);
  float *Fl = reinterpret_cast<float *>(sm + RowSmem::kFl);
  float *Fs = reinterpret_cast<float *>(sm + RowSmem::kFs);
  if (g == 0) {
    // maxima back to natural units (the CTA fold and the merge use expf)
    constexpr float kLn2 = 0.6931471805599453f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      Fm[warp * kMaxG + 2 * t + e] = st.m[e] * kLn2;
      Fl[warp * kMaxG + 2 * t + e] = st.l[e];
      Fs[warp * kMaxG + 2 * t + e] = m_park[e] * kLn2;
    }
  }
  store_acc(Ftr + warp * kMaxG * kD);
  __syncthreads();
  float *AM = reinterpret_cast<float *>(sm + AttnSmem::kAccM);
  float *AL = reinterpret_cast<float *>(sm + AttnSmem::kAccL);
  float *AEx = reinterpret_cast<float *>(sm + AttnSmem::kAccEx);
  float *ATr = reinterpret_cast<float *>(sm + AttnSmem::kAccTr);
  const float *FexAll = reinterpret_cast<const float *>(sm + RowSmem::kFex);
  for (int i = tid; i < a.g * kD; i += blockDim.x) {
    const int hq = i >> 7, c = i & (kD - 1);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, Fm[w * kMaxG + hq]);
    float ex = 0.0f, tr = 0.0f, L = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float mw = Fm[w * kMaxG + hq], ms = Fs[w * kMaxG + hq];
      if (mw == -INFINITY) continue;
      const float sc = expf(mw - M);
      tr = fmaf(Ftr[(w * kMaxG + hq) * kD + c], sc, tr);
      L = fmaf(Fl[w * kMaxG + hq], sc, L);
      if (ms != -INFINITY) ex = fmaf(FexAll[(w * kMaxG + hq) * kD + c], expf(ms - M), ex);
    }
    AEx[i] = ex;
    ATr[i] = tr;
    if (c == 0) {
      AM[hq] = M;
      AL[hq] = L;
    }
  }
  __syncthreads();
  KVR_TRACE_POINT(1, 3);
  attn_finish(a, sm, b, h);
  KVR_TRACE_POINT(1, 6);
}

// Merge kernel for sequence-split partials: one warp per query row.
__global__ void lse_merge_kernel(const float *__restrict__ part, int P, int n_q, void *out, int out_dt) {
  const int lane = threadIdx.x & 31;
  const int qh = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (qh >= n_q) return;
  float mx = -INFINITY;
  for (int p = 0; p < P; ++p) mx = fmaxf(mx, part[((int64_t)p * n_q + qh) * (kD + 2)]);
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, l = 0.0f;
  for (int p = 0; p < P; ++p) {
    const float *pr = part + ((int64_t)p * n_q + qh) * (kD + 2);
    const float m = pr[0];
    if (m == -INFINITY) continue;
    const float w = expf(m - mx);
    l = fmaf(w, pr[1], l);
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] = fmaf(w, pr[2 + lane * 4 + r], acc[r]);
  }
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t idx = (int64_t)qh * kD + lane * 4 + r;
    if (out_dt == KVR_F32) store_elem<KVR_F32>(out, idx, acc[r] * inv);
    else if (out_dt == KVR_F16) store_elem<KVR_F16>(out, idx, acc[r] * inv);
    else store_elem<KVR_BF16>(out, idx, acc[r] * inv);
  }
}

// ------------------------------------------------------------ host side ----
struct AttnWs {
  unsigned *err, *counters;
  float *part;
  size_t bytes;
};

static size_t merge_smem_bytes(int slots) {
  return (size_t)slots * kMaxG * 8 + 2 * kMaxG * kD * 4 + 8 * 2 * kD * 4;
}

static AttnWs attn_ws_layout(void *base, int batch, int n_kv, int units, int g) {
  AttnWs w{};
  char *p = reinterpret_cast<char *>(base);
  const size_t rows = (size_t)batch * n_kv;
  w.err = reinterpret_cast<unsigned *>(p);
  w.counters = reinterpret_cast<unsigned *>(p + kWsAttnCounters);
  w.part = reinterpret_cast<float *>(p + kWsHeader);
  w.bytes = kWsHeader + align_up(rows * (size_t)units * g * kPartStride * 4, 256);
  return w;
}

int sd1_select_scratch(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint32_t *kbits,
                       const uint16_t *kscale, int64_t nt_cap, int64_t n_tiles, int tile, int kind, int k_sel,
                       int64_t ex_t0, int64_t ex_t1, int64_t tile_base, int32_t *sel, float *sel_scores,
                       float *qprime, unsigned *counters, float *scores, cudaStream_t st,
                       const uint32_t *vbits, const uint16_t *vscale, int do_select, const RowPrefetch *rows);

// Units per CTA: one unit per CTA while the rows leave the GPU idle (batch 1,
// latency-bound), more as rows grow, so about two CTAs per SM are launched
// and each folds its units on chip (batched decode, bandwidth-bound).
static int attn_upc(int64_t units, int64_t rows) {
  const int64_t target = 2 * 148;
  int64_t upc = (units * rows + target - 1) / target;
  return (int)(upc < 1 ? 1 : (upc > units ? units : upc));
}

int launch_attn(AttnArgs &a, int batch, cudaStream_t st, const char *what, bool pdl = false) {
  if (a.units <= 0) return set_error(KVR_EINVAL, "%s: nothing to attend", what);
  size_t smem = AttnSmem::kTotal;
  const int upc = attn_upc(a.units, (int64_t)batch * a.n_kv);

  a.slots = (a.units + upc - 1) / upc;
  if (upc > 1) {
    // batched rows: one CTA per row once the rows fill every SM (one wave,
    // each warp with the same number of pieces), else about two CTAs per SM
    const int64_t rows = (int64_t)batch * a.n_kv;
    const int64_t want = rows >= 148 ? 1 : (296 + rows / 2) / rows;
    a.slots = (int)(want < a.units ? want : a.units);
  }
  a.upc = (a.units + a.slots - 1) / a.slots;  // even split over the slots
  a.slots = (a.units + a.upc - 1) / a.upc;
  // the batched path reads fp16 rows as 8-byte quads
  bool f16 = upc > 1;
  for (int s = 0; s < 2; ++s) {
    if (a.n[s] == 0) continue;
    f16 = f16 && a.kdt[s] == KVR_F16 && a.vdt[s] == KVR_F16 && (a.tok_stride[s] % 8) == 0 &&
          (a.batch_stride[s] % 8) == 0 && (reinterpret_cast<uintptr_t>(a.k[s]) % 16) == 0 &&
          (reinterpret_cast<uintptr_t>(a.v[s]) % 16) == 0;
  }
  a.pipelined = (f16 && a.n1_dev == nullptr) ? 1 : 0;
  KVR_REQUIRE(a.rank_scores == nullptr || upc == 1 ||
                  (a.pipelined && a.k_sel <= kRowsRankMaxK && a.rank_n <= kRowsRankMax),
              "%s: in-kernel selection needs one unit per CTA or the batched fp16 path", what);
  const size_t ms = merge_smem_bytes(a.slots);
  if (ms > (size_t)AttnSmem::kML) return set_error(KVR_ENOTSUP, "%s: too many units (%d)", what, a.units);
  dim3 grid(a.slots, a.n_kv, batch);
  // per-device attribute cache (the attribute is per function and device)
  static thread_local int cached_dev = -1;
  static thread_local bool smem_set[3] = {false, false, false};
  static thread_local bool rows_set[3][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    smem_set[0] = smem_set[1] = smem_set[2] = false;
    for (auto &r : rows_set) r[0] = r[1] = false;
    cached_dev = dev;
  }
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  switch (a.tile) {
#define KVR_AT(T)                                                                                  \
  case T:                                                                                          \
    if (!smem_set[T / 64]) {                                                                       \
      cudaFuncSetAttribute(attn_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
      smem_set[T / 64] = true;                                                                     \
    }                                                                                              \
    cfg.gridDim = grid;                                                                            \
    cfg.blockDim = dim3(256);                                                                      \
    cfg.dynamicSmemBytes = smem;                                                                   \
    cfg.stream = st;                                                                               \
    cfg.attrs = attr;                                                                              \
    cfg.numAttrs = pdl ? 1 : 0;                                                                    \
    if (a.pipelined) {                                                                             \
      const bool plo = a.out_dt != KVR_BF16 || a.partial_out != nullptr;                           \
      auto *fn = plo ? attn_rows_kernel<T, true> : attn_rows_kernel<T, false>;                     \
      if (!rows_set[T / 64][plo]) {                                                                \
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);          \
        rows_set[T / 64][plo] = true;                                                              \
      }                                                                                            \
      if (cudaLaunchKernelEx(&cfg, fn, a) != cudaSuccess) return check_launch(what);               \
    } else if (cudaLaunchKernelEx(&cfg, attn_kernel<T>, a) != cudaSuccess) {                       \
      return check_launch(what);                                                                   \
    }                                                                                              \
    break;
    KVR_AT(32)
    KVR_AT(64)
    KVR_AT(128)
#undef KVR_AT
    default:
      return set_error(KVR_ENOTSUP, "%s: tile must be 32, 64 or 128", what);
  }
  return check_launch(what);
}

}  // namespace kvr

using namespace kvr;

namespace kvr {
int sd1_dsmem_step(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint16_t *win_k,
                   const uint16_t *win_v, int64_t win_cap, int64_t n_win, const uint16_t *tail_k,
                   const uint16_t *tail_v, int64_t n_tail, const uint32_t *kbits, const uint16_t *kscale,
                   const uint32_t *vbits, const uint16_t *vscale, int64_t nt_cap, int64_t n_tiles, int tile,
                   int kind, int k_sel, int64_t ex_t0, int64_t ex_t1, float scale, void *out, int out_dtype,
                   float *partial_out, int32_t *sel_out, unsigned *err, cudaStream_t st, bool pdl,
                   int force_c, const Sd1StepUpdate *upd = nullptr);
}

extern "C" size_t kvr_decode_attn_workspace_bytes(int n_q, int n_kv, int d, int64_t n_tok_total) {
  (void)d;
  if (n_kv <= 0 || n_q <= 0) return 0;
  const int units = (int)((n_tok_total + kChunk - 1) / kChunk) + 2;
  return attn_ws_layout(nullptr, 1, n_kv, units, n_q / n_kv).bytes;
}

static int decode_attn_impl(const void *q, int q_dtype, int n_q, int n_kv, int d, const void *k0, const void *v0,
                            int kdt0, int vdt0, int64_t n0, int64_t tok_stride0, const void *k1, const void *v1,
                            int kdt1, int vdt1, int64_t n1, int64_t tok_stride1, float scale, void *out,
                            int out_dtype, void *workspace, size_t workspace_bytes, const int32_t *n1_dev,
                            kvr_stream_t stream, const char *what) {
  KVR_REQUIRE(d == kD, "%s: head_dim must be 128 (got %d)", what, d);
  KVR_REQUIRE(n_kv > 0 && n_q > 0 && n_q % n_kv == 0 && n_q / n_kv <= kMaxG,
              "%s: need n_q %% n_kv == 0 and n_q/n_kv <= 8 (n_q=%d n_kv=%d)", what, n_q, n_kv);
  KVR_REQUIRE(valid_dtype(q_dtype) && valid_dtype(out_dtype), "%s: bad q/out dtype", what);
  KVR_REQUIRE(q && out && workspace, "%s: null pointer", what);
  KVR_REQUIRE(n0 >= 0 && n1 >= 0, "%s: negative token count", what);
  KVR_REQUIRE(n0 == 0 || (k0 && v0 && valid_dtype(kdt0) && valid_dtype(vdt0) && tok_stride0 % 4 == 0),
              "%s: bad segment 0", what);
  KVR_REQUIRE(n1 == 0 || (k1 && v1 && valid_dtype(kdt1) && valid_dtype(vdt1) && tok_stride1 % 4 == 0),
              "%s: bad segment 1", what);
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "%s: workspace must be 256-byte aligned", what);
  AttnArgs a{};
  a.q = q; a.q_dt = q_dtype; a.n_q = n_q; a.n_kv = n_kv; a.g = n_q / n_kv;
  a.inv_scale = (float)(1.0 / (scale > 0.f ? (double)scale : sqrt((double)d)));
  a.k[0] = k0; a.v[0] = v0; a.kdt[0] = kdt0; a.vdt[0] = vdt0; a.n[0] = n0; a.tok_stride[0] = tok_stride0;
  a.k[1] = k1; a.v[1] = v1; a.kdt[1] = kdt1; a.vdt[1] = vdt1; a.n[1] = n1; a.tok_stride[1] = tok_stride1;
  a.nchunk[0] = (int)((n0 + kChunk - 1) / kChunk);
  a.nchunk[1] = (int)((n1 + kChunk - 1) / kChunk);
  a.units = a.nchunk[0] + a.nchunk[1];
  a.tile = 64; a.kind = KVR_HADAMARD;
  a.out = out; a.out_dt = out_dtype;
  a.n1_dev = n1 > 0 ? n1_dev : nullptr;
  if (a.units == 0) {
    cudaMemsetAsync(out, 0, (size_t)n_q * d * dtype_size(out_dtype), as_cuda(stream));
    return check_launch(what);
  }
  KVR_REQUIRE(n_kv <= kWsMaxRows, "%s: n_kv > %d", what, kWsMaxRows);
  AttnWs w = attn_ws_layout(workspace, 1, n_kv, a.units, a.g);
  KVR_REQUIRE(workspace_bytes >= w.bytes, "%s: workspace %zu < %zu bytes", what, workspace_bytes, w.bytes);
  a.err = w.err; a.counters = w.counters; a.part = w.part;
  return launch_attn(a, 1, as_cuda(stream), what);
}

extern "C" int kvr_decode_attn(const void *q, int q_dtype, int n_q, int n_kv, int d, const void *k0, const void *v0,
                               int kdt0, int vdt0, int64_t n0, int64_t tok_stride0, const void *k1, const void *v1,
                               int kdt1, int vdt1, int64_t n1, int64_t tok_stride1, float scale, void *out,
                               int out_dtype, void *workspace, size_t workspace_bytes, kvr_stream_t stream) {
  clear_error();
  return decode_attn_impl(q, q_dtype, n_q, n_kv, d, k0, v0, kdt0, vdt0, n0, tok_stride0, k1, v1, kdt1, vdt1, n1,
                          tok_stride1, scale, out, out_dtype, workspace, workspace_bytes, nullptr, stream,
                          "kvr_decode_attn");
}

extern "C" int kvr_decode_attn_counted(const void *q, int q_dtype, int n_q, int n_kv, int d, const void *k0,
                                       const void *v0, int kdt0, int vdt0, int64_t n0, int64_t tok_stride0,
                                       const void *k1, const void *v1, int kdt1, int vdt1, int64_t n1,
                                       int64_t tok_stride1, const int32_t *n1_count, float scale, void *out,
                                       int out_dtype, void *workspace, size_t workspace_bytes, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(n1_count || n1 == 0, "kvr_decode_attn_counted: null row count");
  return decode_attn_impl(q, q_dtype, n_q, n_kv, d, k0, v0, kdt0, vdt0, n0, tok_stride0, k1, v1, kdt1, vdt1, n1,
                          tok_stride1, scale, out, out_dtype, workspace, workspace_bytes, n1_count, stream,
                          "kvr_decode_attn_counted");
}

static int sd1_units(int64_t n_win, int64_t n_tail, int k_sel) {
  return (int)((n_win + kChunk - 1) / kChunk + (n_tail + kChunk - 1) / kChunk) + k_sel;
}

extern "C" size_t kvr_sd1_attend_workspace_bytes(int batch, int n_q, int n_kv, int tile, int k_sel, int64_t n_win,
                                                 int64_t n_tail) {
  (void)tile;
  if (n_kv <= 0 || n_q <= 0 || batch <= 0) return 0;
  return attn_ws_layout(nullptr, batch, n_kv, sd1_units(n_win, n_tail, k_sel), n_q / n_kv).bytes;
}

static int sd1_attend_impl(const void *q, int q_dtype, const float *qprime, int batch, int n_q, int n_kv,
                           const uint16_t *win_k, const uint16_t *win_v, int64_t win_cap, int64_t n_win,
                           const uint16_t *tail_k, const uint16_t *tail_v, int64_t n_tail, const uint32_t *kbits,
                           const uint16_t *kscale, const uint32_t *vbits, const uint16_t *vscale, int64_t nt_cap,
                           int tile, int kind, const int32_t *sel, int k_sel, float scale, void *out,
                           int out_dtype, float *partial_out, void *workspace, size_t workspace_bytes,
                           kvr_stream_t stream, bool pdl, const float *rank_scores = nullptr,
                           int64_t rank_n = 0, int64_t rank_ex0 = 0, int64_t rank_ex1 = 0,
                           int32_t *sel_out = nullptr) {
  KVR_REQUIRE(batch > 0 && n_kv > 0 && n_q > 0 && n_q % n_kv == 0 && n_q / n_kv <= kMaxG,
              "kvr_sd1_attend: need n_q %% n_kv == 0 and n_q/n_kv <= 8");
  KVR_REQUIRE(tile == 32 || tile == 64 || tile == 128, "kvr_sd1_attend: tile must be 32, 64 or 128");
  KVR_REQUIRE(kind == KVR_HADAMARD || kind == KVR_DCT, "kvr_sd1_attend: unknown transform kind");
  KVR_REQUIRE(valid_dtype(q_dtype) && valid_dtype(out_dtype), "kvr_sd1_attend: bad dtype");
  KVR_REQUIRE(q && workspace && (out || partial_out), "kvr_sd1_attend: null pointer");
  KVR_REQUIRE(n_win >= 0 && n_win <= win_cap && (n_win == 0 || (win_k && win_v)), "kvr_sd1_attend: bad window");
  KVR_REQUIRE(n_tail >= 0 && n_tail <= tile && (n_tail == 0 || (tail_k && tail_v)), "kvr_sd1_attend: bad tail");
  KVR_REQUIRE(k_sel >= 0 && (k_sel == 0 || (sel && qprime && kbits && kscale && vbits && vscale)),
              "kvr_sd1_attend: bad selection/store");
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "kvr_sd1_attend: workspace must be 256-byte aligned");
  AttnArgs a{};
  a.q = q; a.q_dt = q_dtype; a.n_q = n_q; a.n_kv = n_kv; a.g = n_q / n_kv;
  a.inv_scale = (float)(1.0 / (scale > 0.f ? (double)scale : sqrt((double)kD)));
  a.qprime = qprime;
  const int64_t tokw = (int64_t)n_kv * kD;
  a.k[0] = win_k; a.v[0] = win_v; a.kdt[0] = KVR_F16; a.vdt[0] = KVR_F16; a.n[0] = n_win;
  a.tok_stride[0] = tokw; a.batch_stride[0] = win_cap * tokw;
  a.k[1] = tail_k; a.v[1] = tail_v; a.kdt[1] = KVR_F16; a.vdt[1] = KVR_F16; a.n[1] = n_tail;
  a.tok_stride[1] = tokw; a.batch_stride[1] = (int64_t)tile * tokw;
  a.nchunk[0] = (int)((n_win + kChunk - 1) / kChunk);
  a.nchunk[1] = (int)((n_tail + kChunk - 1) / kChunk);
  a.kbits = kbits; a.kscale = kscale; a.vbits = vbits; a.vscale = vscale; a.nt_cap = nt_cap;
  a.tile = tile; a.kind = kind; a.sel = sel; a.k_sel = k_sel;
  a.rank_scores = rank_scores; a.rank_n = rank_n; a.rank_ex0 = rank_ex0; a.rank_ex1 = rank_ex1;
  a.sel_out = sel_out;
  a.out = out; a.out_dt = out_dtype; a.partial_out = partial_out;
  a.units = sd1_units(n_win, n_tail, k_sel);
  if (a.units == 0) {
    cudaStream_t st = as_cuda(stream);
    if (partial_out) {
      // m = -inf rows: fill with a tiny kernel-free pattern via memset is not possible for -inf;
      // an all-empty step is reported as an error instead.
      return set_error(KVR_EINVAL, "kvr_sd1_attend: no tokens to attend");
    }
    cudaMemsetAsync(out, 0, (size_t)batch * n_q * kD * dtype_size(out_dtype), st);
    return check_launch("kvr_sd1_attend (empty)");
  }
  KVR_REQUIRE((int64_t)batch * n_kv <= kWsMaxRows, "kvr_sd1_attend: batch*n_kv > %d", kWsMaxRows);
  AttnWs w = attn_ws_layout(workspace, batch, n_kv, a.units, a.g);
  KVR_REQUIRE(workspace_bytes >= w.bytes, "kvr_sd1_attend: workspace %zu < %zu bytes", workspace_bytes, w.bytes);
  a.err = w.err; a.counters = w.counters; a.part = w.part;
  return launch_attn(a, batch, as_cuda(stream), "kvr_sd1_attend", pdl);
}

extern "C" int kvr_sd1_attend(const void *q, int q_dtype, const float *qprime, int batch, int n_q, int n_kv,
                              const uint16_t *win_k, const uint16_t *win_v, int64_t win_cap, int64_t n_win,
                              const uint16_t *tail_k, const uint16_t *tail_v, int64_t n_tail, const uint32_t *kbits,
                              const uint16_t *kscale, const uint32_t *vbits, const uint16_t *vscale, int64_t nt_cap,
                              int tile, int kind, const int32_t *sel, int k_sel, float scale, void *out,
                              int out_dtype, float *partial_out, void *workspace, size_t workspace_bytes,
                              kvr_stream_t stream) {
  clear_error();
  return sd1_attend_impl(q, q_dtype, qprime, batch, n_q, n_kv, win_k, win_v, win_cap, n_win, tail_k, tail_v, n_tail,
                         kbits, kscale, vbits, vscale, nt_cap, tile, kind, sel, k_sel, scale, out, out_dtype,
                         partial_out, workspace, workspace_bytes, stream, false);
}

static std::atomic<int> g_sd1_step_path{[] {
  const char *e = getenv("KVR_SD1_STEP");
  return (e != nullptr && strcmp(e, "split") == 0) ? 1 : 0;
}()};

extern "C" int kvr_set_sd1_step_path(int path) {
  return g_sd1_step_path.exchange(path == 1 || path == 2 ? path : 0);
}

// decode_step layout: [header | attention partials | tile scores | sel | qprime]
extern "C" size_t kvr_sd1_workspace_bytes(int batch, int n_q, int n_kv, int64_t n_tiles, int tile, int k_sel,
                                          int64_t n_win, int64_t n_tail) {
  const size_t a = align_up(kvr_sd1_attend_workspace_bytes(batch, n_q, n_kv, tile, k_sel, n_win, n_tail), 256);
  const size_t s = align_up((size_t)batch * n_kv * (size_t)(n_tiles > 0 ? n_tiles : 1) * 4, 256);
  const size_t sel = align_up((size_t)batch * n_kv * (k_sel > 0 ? k_sel : 1) * 4, 256);
  const size_t qp = align_up((size_t)batch * n_q * kD * 4, 256);
  return a + s + sel + qp;
}

extern "C" int kvr_sd1_decode_step(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint16_t *win_k,
                                   const uint16_t *win_v, int64_t win_cap, int64_t n_win, const uint16_t *tail_k,
                                   const uint16_t *tail_v, int64_t n_tail, const uint32_t *kbits,
                                   const uint16_t *kscale, const uint32_t *vbits, const uint16_t *vscale,
                                   int64_t nt_cap, int64_t n_tiles, int tile, int kind, int k_sel, int64_t ex_t0,
                                   int64_t ex_t1, float scale, void *out, int out_dtype, int32_t *sel_out,
                                   void *workspace, size_t workspace_bytes, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(batch > 0 && n_kv > 0 && n_q > 0 && n_q % n_kv == 0, "kvr_sd1_decode_step: bad head counts");
  const size_t need = kvr_sd1_workspace_bytes(batch, n_q, n_kv, n_tiles, tile, k_sel, n_win, n_tail);
  KVR_REQUIRE(workspace && workspace_bytes >= need, "kvr_sd1_decode_step: workspace %zu < %zu bytes",
              workspace_bytes, need);
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "kvr_sd1_decode_step: workspace must be 256-byte aligned");
  char *p = reinterpret_cast<char *>(workspace);
  const size_t a_bytes = align_up(kvr_sd1_attend_workspace_bytes(batch, n_q, n_kv, tile, k_sel, n_win, n_tail), 256);
  const size_t s_bytes = align_up((size_t)batch * n_kv * (size_t)(n_tiles > 0 ? n_tiles : 1) * 4, 256);
  const size_t sel_bytes = align_up((size_t)batch * n_kv * (k_sel > 0 ? k_sel : 1) * 4, 256);
  float *scores = reinterpret_cast<float *>(p + a_bytes);
  int32_t *sel = sel_out ? sel_out : reinterpret_cast<int32_t *>(p + a_bytes + s_bytes);
  float *qprime = reinterpret_cast<float *>(p + a_bytes + s_bytes + sel_bytes);
  // Few rows (batch-1 decode): one kernel, a thread-block cluster per row
  // (kvr_dsmem_step.cu).  KVR_SD1_STEP=split keeps the two-kernel path.
  const int path = g_sd1_step_path.load(std::memory_order_relaxed);
  if (path != 1 && (int64_t)batch * n_kv <= 16) {
    const int rc = sd1_dsmem_step(q, q_dtype, batch, n_q, n_kv, win_k, win_v, win_cap, n_win, tail_k, tail_v, n_tail,
                                  kbits, kscale, vbits, vscale, nt_cap, n_tiles, tile, kind, k_sel, ex_t0, ex_t1,
                                  scale, out, out_dtype, nullptr, sel_out, reinterpret_cast<unsigned *>(p),
                                  as_cuda(stream), true, path == 2 ? 8 : 0);
    if (rc != KVR_ENOTSUP) return rc;
  }
  // One unit per attention CTA (batch-1, latency-bound): the selection
  // kernel only scores, every tile unit picks its own tile by rank, and the
  // scan prefetches the V data of every scanned tile into L2 (at larger
  // batches that prefetch would double the DRAM traffic for tiles that are
  // mostly never selected).
  const bool rank = k_sel > 0 && n_tiles > 0 && n_tiles <= kRankMaxTiles &&
                    attn_upc(sd1_units(n_win, n_tail, k_sel), (int64_t)batch * n_kv) == 1;
  // Batched steps: the selection kernel is ALU-bound with DRAM mostly idle, so
  // it streams the window / tail rows into L2 for the attention kernel.
  RowPrefetch rows{};
  const int64_t tokw = (int64_t)n_kv * kD;
  rows.k[0] = n_win > 0 ? win_k : nullptr; rows.v[0] = win_v; rows.n[0] = n_win; rows.batch_stride[0] = win_cap * tokw;
  rows.k[1] = n_tail > 0 ? tail_k : nullptr; rows.v[1] = tail_v; rows.n[1] = n_tail;
  rows.batch_stride[1] = (int64_t)tile * tokw;
  rows.tok_stride = tokw;
  const bool rows_ok = (reinterpret_cast<uintptr_t>(win_k) | reinterpret_cast<uintptr_t>(win_v) |
                        reinterpret_cast<uintptr_t>(tail_k) | reinterpret_cast<uintptr_t>(tail_v)) % 16 == 0;
  // Batched steps on the fp16 rows path: the scan only scores and every
  // attention CTA picks its row's top k_sel itself (no per-row counter and
  // no selection tail at the end of the scan).
  const bool rows_rank = !rank && rows_ok && k_sel > 0 && k_sel <= kRowsRankMaxK && n_tiles > 0 &&
                         n_tiles <= kRowsRankMax;
  const bool self_select = rank || rows_rank;
  int rc = sd1_select_scratch(q, q_dtype, batch, n_q, n_kv, kbits, kscale, nt_cap, n_tiles, tile, kind, k_sel, ex_t0,
                              ex_t1, 0, sel, nullptr, qprime, reinterpret_cast<unsigned *>(p + kWsSelCounters), scores,
                              as_cuda(stream), rank ? vbits : nullptr, rank ? vscale : nullptr, self_select ? 0 : 1,
                              !rank && rows_ok ? &rows : nullptr);
  if (rc) return rc;
  // the attention kernel is a programmatic dependent of the selection
  // kernel: its window/tail units overlap the tile scan, its tile units wait
  return sd1_attend_impl(q, q_dtype, qprime, batch, n_q, n_kv, win_k, win_v, win_cap, n_win, tail_k, tail_v, n_tail,
                         kbits, kscale, vbits, vscale, nt_cap, tile, kind, sel, k_sel, scale, out, out_dtype, nullptr,
                         workspace, a_bytes, stream, true, self_select ? scores : nullptr, n_tiles, ex_t0, ex_t1,
                         self_select ? sel : nullptr);
}

// The decode step with the layer's store update fused in (batch 1): one
// cluster launch rotates q and the new k, builds the new window row in place
// of the slot's old one, moves the old row to the tail and attends; where the
// cluster path does not apply, the store-update kernel and the step run back
// to back, with identical results.
extern "C" int kvr_sd1_decode_step_update(const void *q, const void *k, const void *v, int dtype, int n_q, int n_kv,
                                          const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                                          int64_t pos, void *q_out, uint16_t *win_k, uint16_t *win_v,
                                          int64_t win_cap, int64_t n_win, int64_t slot, uint16_t *tail_k,
                                          uint16_t *tail_v, int64_t n_tail, int evict, const uint32_t *kbits,
                                          const uint16_t *kscale, const uint32_t *vbits, const uint16_t *vscale,
                                          int64_t nt_cap, int64_t n_tiles, int tile, int kind, int k_sel,
                                          int64_t ex_t0, int64_t ex_t1, float scale, void *out, int out_dtype,
                                          int32_t *sel_out, void *workspace, size_t workspace_bytes,
                                          kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(valid_dtype(dtype) && q && k && v && cos_tbl && sin_tbl && q_out && win_k && win_v,
              "kvr_sd1_decode_step_update: bad dtype or null pointer");
  KVR_REQUIRE(n_kv > 0 && n_q > 0 && n_q % n_kv == 0, "kvr_sd1_decode_step_update: bad head counts");
  KVR_REQUIRE(n_win >= 1 && n_win <= win_cap && slot >= 0 && slot < n_win,
              "kvr_sd1_decode_step_update: the slot must lie in the window's valid rows");
  KVR_REQUIRE(pos >= 0 && rope_stride >= kD && rope_stride % 4 == 0, "kvr_sd1_decode_step_update: bad RoPE position");
  KVR_REQUIRE(!evict || (tail_k && tail_v && n_tail >= 1 && n_tail <= tile),
              "kvr_sd1_decode_step_update: an eviction needs a tail with room (n_tail counts the evicted row)");
  KVR_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                reinterpret_cast<uintptr_t>(q_out) | reinterpret_cast<uintptr_t>(cos_tbl) |
                reinterpret_cast<uintptr_t>(sin_tbl)) & 15) == 0,
              "kvr_sd1_decode_step_update: q, k, v, q_out and the tables must be 16-byte aligned");
  const size_t need = kvr_sd1_workspace_bytes(1, n_q, n_kv, n_tiles, tile, k_sel, n_win, n_tail);
  KVR_REQUIRE(workspace && workspace_bytes >= need, "kvr_sd1_decode_step_update: workspace %zu < %zu bytes",
              workspace_bytes, need);
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
              "kvr_sd1_decode_step_update: workspace must be 256-byte aligned");
  const float *cr = cos_tbl + pos * rope_stride, *sr = sin_tbl + pos * rope_stride;
  const int path = g_sd1_step_path.load(std::memory_order_relaxed);
  if (path != 1 && n_kv <= 16) {
    const Sd1StepUpdate u{k, v, cr, sr, q_out, slot, evict ? n_tail - 1 : -1};
    const int rc = sd1_dsmem_step(q, dtype, 1, n_q, n_kv, win_k, win_v, win_cap, n_win, tail_k, tail_v, n_tail, kbits,
                                  kscale, vbits, vscale, nt_cap, n_tiles, tile, kind, k_sel, ex_t0, ex_t1, scale, out,
                                  out_dtype, nullptr, sel_out, reinterpret_cast<unsigned *>(workspace),
                                  as_cuda(stream), true, path == 2 ? 8 : 0, &u);
    if (rc != KVR_ENOTSUP) return rc;
  }
  int rc = kvr_decode_store_update(q, k, v, dtype, n_q, n_kv, kD, cos_tbl, sin_tbl, rope_stride, pos, q_out, win_k,
                                   win_v, win_cap, slot, evict ? tail_k : nullptr, evict ? tail_v : nullptr,
                                   evict ? n_tail - 1 : 0, 1, stream);
  if (rc) return rc;
  return kvr_sd1_decode_step(q_out, dtype, 1, n_q, n_kv, win_k, win_v, win_cap, n_win, tail_k, tail_v, n_tail, kbits,
                             kscale, vbits, vscale, nt_cap, n_tiles, tile, kind, k_sel, ex_t0, ex_t1, scale, out,
                             out_dtype, sel_out, workspace, workspace_bytes, stream);
}

#ifdef KVR_TRACE
extern "C" KVR_API int kvr_debug_trace_attn(unsigned long long *host, int n) {
  return cudaMemcpyFromSymbol(host, kvr::g_kvr_trace, sizeof(unsigned long long) * n) == cudaSuccess ? 0 : 2;
}
#endif

extern "C" int kvr_lse_merge(const float *partials, int P, int n_q, int d, void *out, int out_dtype,
                             kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == kD, "kvr_lse_merge: head_dim must be 128");
  KVR_REQUIRE(partials && out && P > 0 && n_q > 0 && valid_dtype(out_dtype), "kvr_lse_merge: bad arguments");
  lse_merge_kernel<<<(n_q + 7) / 8, 256, 0, as_cuda(stream)>>>(partials, P, n_q, out, out_dtype);
  return check_launch("kvr_lse_merge");
}

extern "C" int kvr_workspace_status(const void *workspace, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(workspace, "kvr_workspace_status: null workspace");
  unsigned flag = 0;
  cudaStream_t st = as_cuda(stream);
  if (cudaMemcpyAsync(&flag, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return check_launch("kvr_workspace_status");
  if (flag) {
    cudaMemsetAsync(const_cast<void *>(workspace), 0, 4, st);
    return set_error(KVR_ETIMEOUT, "a bounded device-side wait gave up (flag %u)", flag);
  }
  return KVR_OK;
}

// ------------------------------------------------- allocation-free variant ----
// Some callers cannot allocate device memory at all: plugins that run inside a
// host whose allocator owns the whole GPU heap, or code on a path where a
// cudaMalloc would stall the device or break a latency budget.  For them,
// kvr_decode_attn_noalloc keeps its scratch (error word, per-head counters and
// log-sum-exp partials) in this fixed array, which every GPU that loads the
// library holds until the process exits.
namespace kvr {
constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static void *g_scratch_ptr[kMaxDevices] = {nullptr};
static std::mutex g_scratch_mu;

// Device address of g_attn_scratch on the current device (looked up once per
// device; the name itself is only a host-side stand-in).
static int scratch_address(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("kvr_decode_attn_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(KVR_ENOTSUP, "kvr_decode_attn_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess)
      return set_error(KVR_ECUDA, "kvr_decode_attn_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KVR_OK;
}
}  // namespace kvr

extern "C" size_t kvr_decode_attn_noalloc_max_scratch_bytes(void) { return kvr::kNoAllocScratchBytes; }

extern "C" int kvr_decode_attn_noalloc(const void *q, int q_dtype, int n_q, int n_kv, int d, const void *k0,
                                       const void *v0, int kdt0, int vdt0, int64_t n0, int64_t tok_stride0,
                                       const void *k1, const void *v1, int kdt1, int vdt1, int64_t n1,
                                       int64_t tok_stride1, float scale, void *out, int out_dtype,
                                       kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == kD, "kvr_decode_attn_noalloc: head_dim must be 128 (got %d)", d);
  KVR_REQUIRE(n_kv > 0 && n_q > 0 && n_q % n_kv == 0 && n_q / n_kv <= kMaxG,
              "kvr_decode_attn_noalloc: need n_q %% n_kv == 0 and n_q/n_kv <= 8 (n_q=%d n_kv=%d)", n_q, n_kv);
  KVR_REQUIRE(n_kv <= kWsMaxRows, "kvr_decode_attn_noalloc: n_kv > %d", kWsMaxRows);
  KVR_REQUIRE(valid_dtype(q_dtype) && valid_dtype(out_dtype), "kvr_decode_attn_noalloc: bad q/out dtype");
  KVR_REQUIRE(q && out, "kvr_decode_attn_noalloc: null pointer");
  KVR_REQUIRE(n0 >= 0 && n1 >= 0, "kvr_decode_attn_noalloc: negative token count");
  KVR_REQUIRE(n0 == 0 || (k0 && v0 && valid_dtype(kdt0) && valid_dtype(vdt0) && tok_stride0 % 4 == 0),
              "kvr_decode_attn_noalloc: bad segment 0");
  KVR_REQUIRE(n1 == 0 || (k1 && v1 && valid_dtype(kdt1) && valid_dtype(vdt1) && tok_stride1 % 4 == 0),
              "kvr_decode_attn_noalloc: bad segment 1");
  AttnArgs a{};
  a.q = q; a.q_dt = q_dtype; a.n_q = n_q; a.n_kv = n_kv; a.g = n_q / n_kv;
  a.inv_scale = (float)(1.0 / (scale > 0.f ? (double)scale : sqrt((double)d)));
  a.k[0] = k0; a.v[0] = v0; a.kdt[0] = kdt0; a.vdt[0] = vdt0; a.n[0] = n0; a.tok_stride[0] = tok_stride0;
  a.k[1] = k1; a.v[1] = v1; a.kdt[1] = kdt1; a.vdt[1] = vdt1; a.n[1] = n1; a.tok_stride[1] = tok_stride1;
  a.nchunk[0] = (int)((n0 + kChunk - 1) / kChunk);
  a.nchunk[1] = (int)((n1 + kChunk - 1) / kChunk);
  a.units = a.nchunk[0] + a.nchunk[1];
  a.tile = 64; a.kind = KVR_HADAMARD;
  a.out = out; a.out_dt = out_dtype;
  cudaStream_t st = as_cuda(stream);
  if (a.units == 0) {
    cudaMemsetAsync(out, 0, (size_t)n_q * d * dtype_size(out_dtype), st);
    return check_launch("kvr_decode_attn_noalloc (empty)");
  }
  const size_t need = attn_ws_layout(nullptr, 1, n_kv, a.units, a.g).bytes;
  if (need > kNoAllocScratchBytes)
    return set_error(KVR_EINVAL,
                     "kvr_decode_attn_noalloc: this call needs %zu bytes of scratch, the built-in maximum is %zu "
                     "(fewer tokens or heads per call, or use kvr_decode_attn with a caller workspace)",
                     need, kNoAllocScratchBytes);
  void *base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return rc;
  // The array keeps whatever the previous call left: zero the error word and
  // this call's counters, which must start at zero.
  if (cudaMemsetAsync(base, 0, 4, st) != cudaSuccess ||
      cudaMemsetAsync(static_cast<char *>(base) + kWsAttnCounters, 0, (size_t)n_kv * 4, st) != cudaSuccess)
    return check_launch("kvr_decode_attn_noalloc: clearing scratch");
  AttnWs w = attn_ws_layout(base, 1, n_kv, a.units, a.g);
  a.err = w.err; a.counters = w.counters; a.part = w.part;
  return launch_attn(a, 1, st, "kvr_decode_attn_noalloc");
}
