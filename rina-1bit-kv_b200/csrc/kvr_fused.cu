// Fused sd1 decode step: one kernel per layer on thread-block clusters.
//
// One cluster of CS CTAs (CS = 16, or 8 where 16 cannot be scheduled) serves
// one (batch b, KV head h) row:
//   1. every CTA bulk-copies its slice of the head's K tiles (bits + scales)
//      into shared memory and forms the transformed queries (q' of each head
//      of the group, and the group mean for selection) itself;
//   2. every CTA scores its slice (sd1_score_tile, bit-exact with the
//      selection kernel) and arrives on the cluster barrier;
//   3. rank 0 gathers all tile scores through distributed shared memory and
//      selects the top k_sel tiles; ranks >= 1 meanwhile attend their share
//      of the exact window/tail tokens;
//   4. the selected tiles are spread over the cluster (slot j -> rank j % CS),
//      bulk-copied from HBM and attended in the transformed domain;
//   5. rank 0 merges the CTAs' log-sum-exp partials through distributed
//      shared memory, maps the transformed part back with one inverse
//      transform per query head, and writes the output.
// Scores, selection and partials never leave the SMs: no atomics, no global
// scratch, one launch — the batch-1 decode step is latency-bound and this
// removes the global round trips of the two-kernel path.  Same results as
// kvr_sd1_select + kvr_sd1_attend (selection bit-identical).
#include <cooperative_groups.h>

#include "kvr_common.cuh"
#include "kvr_sd1_score.cuh"
#include "kvr_topk.cuh"
#include "kvr_transform.cuh"

namespace cg = cooperative_groups;

namespace kvr {

__host__ __device__ __forceinline__ int64_t clamp64(int64_t x, int64_t lo, int64_t hi) {
  return x < lo ? lo : (x > hi ? hi : x);
}

constexpr int kFThreads = 512;
constexpr int kFWarps = kFThreads / 32;
constexpr int kFChunk = 64;
constexpr int kFMaxG = 8;
constexpr int kFKsStride = kD + 4;
constexpr int kFMaxSel = 64;
constexpr int kFMaxTiles = 4096;

struct FusedArgs {
  const void *q;
  int q_dt, n_q, n_kv, g;
  float inv_scale;
  const uint16_t *win_k, *win_v;
  int64_t win_cap, n_win;
  const uint16_t *tail_k, *tail_v;
  int64_t n_tail, tail_cap;
  const uint32_t *kbits;
  const uint16_t *kscale;
  const uint32_t *vbits;
  const uint16_t *vscale;
  int64_t nt_cap, n_tiles, ex_t0, ex_t1;
  int kind, k_sel, nt_per, cs;
  void *out;
  int out_dt;
  int32_t *sel_out;
  unsigned *err;
};

// shared-memory plan; the K slice follows the fixed part
struct FSmem {
  static constexpr int kLee = 0;                                  // f32 [128]
  static constexpr int kBuf = kLee + kD * 4;                       // f32 [9][256]
  static constexpr int kQp = kBuf + (kFMaxG + 1) * 2 * kD * 4;     // f32 [8][128] q' * inv_scale
  static constexpr int kQs = kQp + kFMaxG * kD * 4;                // f32 [8][128] q * inv_scale
  static constexpr int kQavg = kQs + kFMaxG * kD * 4;              // f32 [128]
  static constexpr int kStage = kQavg + kD * 4;                    // union (exact | tile)
  static constexpr int kKs = kStage;                               // f32 [64][132]
  static constexpr int kVs = kKs + kFChunk * kFKsStride * 4;       // f32 [64][128]
  static constexpr int kStageExactEnd = kVs + kFChunk * kD * 4;
  static constexpr int kKB = kStage;                               // u32 [128][4]
  static constexpr int kVB = kKB + 128 * 16;
  static constexpr int kKS = kVB + 128 * 16;                       // f16 [128]
  static constexpr int kVS = kKS + kD * 2;
  static constexpr int kLUT = kVS + kD * 2;                        // f32 [8][32][16]
  static constexpr int kStageTileEnd = kLUT + kFMaxG * 32 * 16 * 4;
  static constexpr int kStageEnd = kStageExactEnd > kStageTileEnd ? kStageExactEnd : kStageTileEnd;
  static constexpr int kS = kStageEnd;                             // f32 [8][128]
  static constexpr int kP = kS + kFMaxG * kD * 4;                  // f32 [128][8]
  static constexpr int kRed = kP + 128 * kFMaxG * 4;               // f32 [4][8][128] quarter sums
  static constexpr int kAccM = kRed + 4 * kFMaxG * kD * 4;         // f32 [8] running max
  static constexpr int kAccL = kAccM + kFMaxG * 4;                 // f32 [8]
  static constexpr int kUnitML = kAccL + kFMaxG * 4;               // f32 [8][2] unit (m, l)
  static constexpr int kScale = kUnitML + kFMaxG * 2 * 4;          // f32 [8][2] (alpha, beta)
  static constexpr int kOex = kScale + kFMaxG * 2 * 4;             // f32 [8][128]
  static constexpr int kOtr = kOex + kFMaxG * kD * 4;              // f32 [8][128]
  static constexpr int kSel = kOtr + kFMaxG * kD * 4;              // i32 [64]
  static constexpr int kTopk = kSel + kFMaxSel * 4;                // TopkSmem
  static constexpr int kCand = kTopk + 8192;                       // u64 [64]
  static constexpr int kBars = kCand + kFMaxSel * 8;               // u64 [4]
  static constexpr int kFlags = kBars + 32;                        // i32 [4]
  static constexpr int kGather = kFlags + 16;                      // f32 [kFMaxTiles] (rank 0)
  static constexpr int kFixed = kGather + kFMaxTiles * 4;          // then: slice scores, bits, scales
};
static_assert(sizeof(TopkSmem) <= 8192, "TopkSmem grew");

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Fold the unit partial (unit m/l in kUnitML, unit o in `src` rows [hq][128])
// into the running accumulators; `into_tr` picks the transformed-domain sum.
__device__ void fold_unit(const FusedArgs &a, unsigned char *sm, const float *src, bool into_tr) {
  float *M = reinterpret_cast<float *>(sm + FSmem::kAccM);
  float *L = reinterpret_cast<float *>(sm + FSmem::kAccL);
  const float *UML = reinterpret_cast<const float *>(sm + FSmem::kUnitML);
  float *SC = reinterpret_cast<float *>(sm + FSmem::kScale);
  float *oex = reinterpret_cast<float *>(sm + FSmem::kOex);
  float *otr = reinterpret_cast<float *>(sm + FSmem::kOtr);
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
  for (int i = tid; i < a.g * kD; i += kFThreads) {
    const int hq = i >> 7;
    const float al = SC[2 * hq], be = SC[2 * hq + 1];
    const float u = src[i] * be;
    oex[i] = oex[i] * al + (into_tr ? 0.0f : u);
    otr[i] = otr[i] * al + (into_tr ? u : 0.0f);
  }
  __syncthreads();
}

// Softmax over S[hq][0..nt) -> P[j][hq], unit (m, l).
__device__ __forceinline__ void fused_softmax(const FusedArgs &a, unsigned char *sm, int nt) {
  const float *S = reinterpret_cast<const float *>(sm + FSmem::kS);
  float *P = reinterpret_cast<float *>(sm + FSmem::kP);
  float *UML = reinterpret_cast<float *>(sm + FSmem::kUnitML);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int hq = warp; hq < a.g; hq += kFWarps) {
    float mx = -INFINITY;
    for (int j = lane; j < nt; j += 32) mx = fmaxf(mx, S[hq * kD + j]);
    mx = warp_max(mx);
    float l = 0.0f;
    for (int j = lane; j < 128; j += 32) {
      float p = 0.0f;
      if (j < nt && mx != -INFINITY) p = expf(S[hq * kD + j] - mx);
      P[j * kFMaxG + hq] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      UML[2 * hq] = mx;
      UML[2 * hq + 1] = l;
    }
  }
}

// P.V over rows Vs (fp32 [nt][128]) or V bits; thread = (channel, quarter).
// Writes the unit output rows [hq][128] into kRed quarter 0.
template <bool BITS>
__device__ __forceinline__ void fused_pv(const FusedArgs &a, unsigned char *sm, int nt) {
  const float *P = reinterpret_cast<const float *>(sm + FSmem::kP);
  float *red = reinterpret_cast<float *>(sm + FSmem::kRed);
  const int tid = threadIdx.x, c = tid & 127, qtr = tid >> 7;
  const int per = (nt + 3) / 4;
  float o[kFMaxG];
#pragma unroll
  for (int i = 0; i < kFMaxG; ++i) o[i] = 0.0f;
  const float *Vs = reinterpret_cast<const float *>(sm + FSmem::kVs);
  const uint32_t *VB = reinterpret_cast<const uint32_t *>(sm + FSmem::kVB);
  const int j0 = qtr * per, j1 = min(nt, j0 + per);
  for (int j = j0; j < j1; ++j) {
    const float vv = BITS ? (float)((VB[j * 4 + (c >> 5)] >> (c & 31)) & 1u) : Vs[j * kD + c];
    const float4 p0 = *reinterpret_cast<const float4 *>(P + j * kFMaxG);
    const float4 p1 = *reinterpret_cast<const float4 *>(P + j * kFMaxG + 4);
    o[0] = fmaf(p0.x, vv, o[0]); o[1] = fmaf(p0.y, vv, o[1]);
    o[2] = fmaf(p0.z, vv, o[2]); o[3] = fmaf(p0.w, vv, o[3]);
    if (a.g > 4) {
      o[4] = fmaf(p1.x, vv, o[4]); o[5] = fmaf(p1.y, vv, o[5]);
      o[6] = fmaf(p1.z, vv, o[6]); o[7] = fmaf(p1.w, vv, o[7]);
    }
  }
  for (int hq = 0; hq < a.g; ++hq) red[(qtr * kFMaxG + hq) * kD + c] = o[hq];
  __syncthreads();
  if (qtr == 0) {
    const float *UML = reinterpret_cast<const float *>(sm + FSmem::kUnitML);
    const uint16_t *VS = reinterpret_cast<const uint16_t *>(sm + FSmem::kVS);
    for (int hq = 0; hq < a.g; ++hq) {
      float s = ((red[hq * kD + c] + red[(kFMaxG + hq) * kD + c]) + red[(2 * kFMaxG + hq) * kD + c]) +
                red[(3 * kFMaxG + hq) * kD + c];
      if (BITS) s = __half2float(__ushort_as_half(VS[c])) * (2.0f * s - UML[2 * hq + 1]);
      red[hq * kD + c] = s;
    }
  }
  __syncthreads();
}

// Exact tokens [e0, e0 + nt) of the concatenated window + tail (nt <= 64):
// the loads (into registers), the fp32 staging, and the compute are split so
// the first chunk's loads can be issued at kernel start.
struct ExactRegs {
  uint2 k[4], v[4];
};
__device__ __forceinline__ void fused_exact_load(const FusedArgs &a, int64_t b, int h, int64_t e0, int nt,
                                                 ExactRegs &r) {
  const int tid = threadIdx.x;
  const int64_t tokw = (int64_t)a.n_kv * kD;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = tid + i * kFThreads, j = idx >> 5, qd = idx & 31;
    r.k[i] = r.v[i] = make_uint2(0u, 0u);
    if (j < nt) {
      const int64_t e = e0 + j;
      const uint16_t *kp, *vp;
      int64_t off;
      if (e < a.n_win) {
        off = (b * a.win_cap + e) * tokw + (int64_t)h * kD + qd * 4;
        kp = a.win_k; vp = a.win_v;
      } else {
        off = (b * a.tail_cap + (e - a.n_win)) * tokw + (int64_t)h * kD + qd * 4;
        kp = a.tail_k; vp = a.tail_v;
      }
      r.k[i] = __ldg(reinterpret_cast<const uint2 *>(kp + off));
      r.v[i] = __ldg(reinterpret_cast<const uint2 *>(vp + off));
    }
  }
}
__device__ __forceinline__ void fused_exact_store(unsigned char *sm, const ExactRegs &r) {
  float *Ks = reinterpret_cast<float *>(sm + FSmem::kKs);
  float *Vs = reinterpret_cast<float *>(sm + FSmem::kVs);
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = tid + i * kFThreads, j = idx >> 5, qd = idx & 31;
    const float2 k0 = __half22float2(*reinterpret_cast<const __half2 *>(&r.k[i].x));
    const float2 k1 = __half22float2(*reinterpret_cast<const __half2 *>(&r.k[i].y));
    const float2 v0 = __half22float2(*reinterpret_cast<const __half2 *>(&r.v[i].x));
    const float2 v1 = __half22float2(*reinterpret_cast<const __half2 *>(&r.v[i].y));
    *reinterpret_cast<float4 *>(Ks + j * kFKsStride + qd * 4) = make_float4(k0.x, k0.y, k1.x, k1.y);
    *reinterpret_cast<float4 *>(Vs + j * kD + qd * 4) = make_float4(v0.x, v0.y, v1.x, v1.y);
  }
}
// Computes on a chunk already staged in Ks/Vs.
__device__ void fused_exact_compute(const FusedArgs &a, unsigned char *sm, int nt) {
  const float *Ks = reinterpret_cast<const float *>(sm + FSmem::kKs);
  const float *Qs = reinterpret_cast<const float *>(sm + FSmem::kQs);
  float *S = reinterpret_cast<float *>(sm + FSmem::kS);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __syncthreads();
  for (int p = warp; p < a.g * 2; p += kFWarps) {
    const int hq = p >> 1, j = (p & 1) * 32 + lane;
    const float4 *kr = reinterpret_cast<const float4 *>(Ks + j * kFKsStride);
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
  fused_softmax(a, sm, nt);
  __syncthreads();
  fused_pv<false>(a, sm, kFChunk);
  fold_unit(a, sm, reinterpret_cast<const float *>(sm + FSmem::kRed), false);
}

// One selected tile (store index t): bulk copy, LUT scores, softmax, P.V in
// the transformed domain.
template <int TILE>
__device__ void fused_tile(const FusedArgs &a, unsigned char *sm, int64_t row, int64_t t, unsigned &phase) {
  uint32_t *KB = reinterpret_cast<uint32_t *>(sm + FSmem::kKB);
  const uint16_t *KS = reinterpret_cast<const uint16_t *>(sm + FSmem::kKS);
  float *LUT = reinterpret_cast<float *>(sm + FSmem::kLUT);
  const float *Qp = reinterpret_cast<const float *>(sm + FSmem::kQp);
  float *S = reinterpret_cast<float *>(sm + FSmem::kS);
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm + FSmem::kBars) + 1;
  int *flags = reinterpret_cast<int *>(sm + FSmem::kFlags);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tix = row * a.nt_cap + t;
  constexpr unsigned kBits = TILE * 16, kScl = kD * 2;
  if (tid == 0) {
    flags[1] = 1;
    mbar_expect_tx(bar, 2 * kBits + 2 * kScl);
    bulk_g2s(KB, a.kbits + tix * TILE * 4, kBits, bar);
    bulk_g2s(sm + FSmem::kVB, a.vbits + tix * TILE * 4, kBits, bar);
    bulk_g2s(sm + FSmem::kKS, a.kscale + tix * kD, kScl, bar);
    bulk_g2s(sm + FSmem::kVS, a.vscale + tix * kD, kScl, bar);
  }
  __syncthreads();
  if (!mbar_wait_bounded(bar, phase)) {
    atomicOr(a.err, 1u);
    flags[1] = 0;
    mbar_wait_bounded(bar, phase);
  }
  phase ^= 1u;
  __syncthreads();
  if (!flags[1]) return;  // uniform: the unit is dropped and reported
  for (int i = tid; i < a.g * 32; i += kFThreads) {
    const int hq = i >> 5, grp = i & 31;
    float av[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) av[r] = Qp[hq * kD + 4 * grp + r] * __half2float(__ushort_as_half(KS[4 * grp + r]));
    float *Lt = LUT + (hq * 32 + grp) * 16;
#pragma unroll
    for (int x = 0; x < 16; ++x) {
      float s = 0.0f;
#pragma unroll
      for (int r = 0; r < 4; ++r) s += ((x >> r) & 1) ? av[r] : -av[r];
      Lt[x] = s;
    }
  }
  __syncthreads();
  constexpr int NB = TILE / 32;
  for (int p = warp; p < a.g * NB; p += kFWarps) {
    const int hq = p / NB, j = (p - hq * NB) * 32 + lane;
    const uint4 w4 = reinterpret_cast<const uint4 *>(KB)[j];
    const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
    const float *Lh = LUT + hq * 32 * 16;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int grp = 0; grp < 32; ++grp) acc[grp & 3] += Lh[grp * 16 + ((w[grp >> 3] >> (4 * (grp & 7))) & 15u)];
    S[hq * kD + j] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
  __syncthreads();
  fused_softmax(a, sm, TILE);
  __syncthreads();
  fused_pv<true>(a, sm, TILE);
  fold_unit(a, sm, reinterpret_cast<const float *>(sm + FSmem::kRed), true);
}

template <int TILE>
__global__ void __launch_bounds__(kFThreads, 1) sd1_fused_kernel(FusedArgs a) {
  extern __shared__ __align__(128) unsigned char sm[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int CS = a.cs;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t row = b * a.n_kv + h;
  const int g = a.g;

  float *lee = reinterpret_cast<float *>(sm + FSmem::kLee);
  float *Qp = reinterpret_cast<float *>(sm + FSmem::kQp);
  float *Qs = reinterpret_cast<float *>(sm + FSmem::kQs);
  float *Qavg = reinterpret_cast<float *>(sm + FSmem::kQavg);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + FSmem::kBars);
  int *flags = reinterpret_cast<int *>(sm + FSmem::kFlags);
  int32_t *sel_s = reinterpret_cast<int32_t *>(sm + FSmem::kSel);
  float *M = reinterpret_cast<float *>(sm + FSmem::kAccM);
  float *L = reinterpret_cast<float *>(sm + FSmem::kAccL);
  float *oex = reinterpret_cast<float *>(sm + FSmem::kOex);
  float *otr = reinterpret_cast<float *>(sm + FSmem::kOtr);
  float *scores_s = reinterpret_cast<float *>(sm + FSmem::kFixed);
  const int nt_per = a.nt_per;
  const size_t slice_off = FSmem::kFixed + align_up((size_t)nt_per * 4, 128);
  uint32_t *slice_bits = reinterpret_cast<uint32_t *>(sm + slice_off);
  uint16_t *slice_scl = reinterpret_cast<uint16_t *>(sm + slice_off + (size_t)nt_per * TILE * 16);

  const int64_t t0 = (int64_t)rank * nt_per;
  const int nt_here = (int)clamp64(a.n_tiles - t0, 0, nt_per);

  KVR_TRACE_POINT(2, 0);
  // ---- phase 0: issue the slice copy and the query loads
  if (tid == 0) {
    flags[0] = 1;
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    if (nt_here > 0) {
      const int64_t tix = row * a.nt_cap + t0;
      mbar_expect_tx(&bars[0], (unsigned)nt_here * (TILE * 16 + kD * 2));
      bulk_g2s(slice_bits, a.kbits + tix * TILE * 4, (unsigned)nt_here * TILE * 16, &bars[0]);
      bulk_g2s(slice_scl, a.kscale + tix * kD, (unsigned)nt_here * kD * 2, &bars[0]);
    }
  }
  if (a.kind == KVR_DCT) load_lee(lee);
  const int64_t n_ex = a.n_win + a.n_tail;
  const int64_t ex_per = (n_ex + CS - 2) / (CS - 1);
  const int64_t ex_begin = (int64_t)(rank - 1) * ex_per;
  const int ex_nt0 = rank > 0 ? (int)clamp64(n_ex - ex_begin, 0, kFChunk < ex_per ? kFChunk : ex_per) : 0;
  ExactRegs ex_regs;
  if (ex_nt0 > 0) fused_exact_load(a, b, h, ex_begin, ex_nt0, ex_regs);
  float qv[kFMaxG][4];
  const int64_t qb = (b * a.n_q + (int64_t)h * g) * kD + lane * 4;
  if (warp < g) {
    const float4 x = cvt4(raw4(a.q, qb + (int64_t)warp * kD, a.q_dt), a.q_dt);
    qv[0][0] = x.x; qv[0][1] = x.y; qv[0][2] = x.z; qv[0][3] = x.w;
  } else if (warp == kFMaxG) {
#pragma unroll
    for (int i = 0; i < kFMaxG; ++i)
      if (i < g) {
        const float4 x = cvt4(raw4(a.q, qb + (int64_t)i * kD, a.q_dt), a.q_dt);
        qv[i][0] = x.x; qv[i][1] = x.y; qv[i][2] = x.z; qv[i][3] = x.w;
      }
  }
  for (int i = tid; i < g * kD; i += kFThreads) {
    oex[i] = 0.0f;
    otr[i] = 0.0f;
  }
  if (tid < g) {
    M[tid] = -INFINITY;
    L[tid] = 0.0f;
  }
  __syncthreads();

  KVR_TRACE_POINT(2, 1);
  // ---- phase 1: transformed queries
  float *buf = reinterpret_cast<float *>(sm + FSmem::kBuf) + (warp < kFMaxG + 1 ? warp : 0) * 2 * kD;
  if (warp < g) {
    float x[4] = {qv[0][0], qv[0][1], qv[0][2], qv[0][3]};
    reinterpret_cast<float4 *>(Qs + warp * kD)[lane] =
        make_float4(x[0] * a.inv_scale, x[1] * a.inv_scale, x[2] * a.inv_scale, x[3] * a.inv_scale);
    transform128(x, lane, a.kind, false, buf, lee);
    reinterpret_cast<float4 *>(Qp + warp * kD)[lane] =
        make_float4(x[0] * a.inv_scale, x[1] * a.inv_scale, x[2] * a.inv_scale, x[3] * a.inv_scale);
  } else if (warp == kFMaxG) {
    float acc[4] = {qv[0][0], qv[0][1], qv[0][2], qv[0][3]};
#pragma unroll
    for (int i = 1; i < kFMaxG; ++i)
      if (i < g)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r] = __fadd_rn(acc[r], qv[i][r]);
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] = __fdiv_rn(acc[r], (float)g);
    transform128(acc, lane, a.kind, false, buf, lee);
    reinterpret_cast<float4 *>(Qavg)[lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
  __syncthreads();

  KVR_TRACE_POINT(2, 2);
  if (ex_nt0 > 0) fused_exact_store(sm, ex_regs);  // stage region is free until the exact compute
  // ---- phase 2: score the slice
  if (nt_here > 0) {
    if (!mbar_wait_bounded(&bars[0], 0)) {
      atomicOr(a.err, 1u);
      flags[0] = 0;
      mbar_wait_bounded(&bars[0], 0);
    }
    __syncthreads();
    const bool ok = flags[0] != 0;
    for (int i0 = 2 * warp; i0 < nt_here; i0 += 2 * kFWarps) {
      uint4 kb[2][TILE / 32];
      uint16_t ks[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = min(i0 + u, nt_here - 1);
#pragma unroll
        for (int r = 0; r < TILE / 32; ++r)
          kb[u][r] = reinterpret_cast<const uint4 *>(slice_bits + (size_t)i * TILE * 4)[lane + 32 * r];
#pragma unroll
        for (int m = 0; m < 4; ++m) ks[u][m] = slice_scl[(size_t)i * kD + lane + 32 * m];
      }
      float sc[2];
      sd1_score_tile2<TILE>(Qavg, kb, ks, lane, sc);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i0 + u;
        const int64_t t = t0 + i;
        if (i < nt_here && lane == 0) scores_s[i] = (!ok || (t >= a.ex_t0 && t < a.ex_t1)) ? -INFINITY : sc[u];
      }
    }
  }
  __syncthreads();
  KVR_TRACE_POINT(2, 3);
  cluster_arrive();  // S1: slice scores are in shared memory

  if (rank == 0) {
    cluster_wait();
    // gather every slice's scores and select
    // all remote reads are issued before any is consumed (n_tiles <= 4096)
    float *gs = reinterpret_cast<float *>(sm + FSmem::kGather);
    {
      constexpr int kPer = kFMaxTiles / kFThreads;
      float v[kPer];
#pragma unroll
      for (int m = 0; m < kPer; ++m) {
        const int64_t k = tid + (int64_t)m * kFThreads;
        v[m] = 0.0f;
        if (k < a.n_tiles) v[m] = cluster.map_shared_rank(scores_s, (int)(k / nt_per))[k % nt_per];
      }
#pragma unroll
      for (int m = 0; m < kPer; ++m) {
        const int64_t k = tid + (int64_t)m * kFThreads;
        if (k < a.n_tiles) gs[k] = v[m];
      }
    }
    __syncthreads();
    KVR_TRACE_POINT(3, 1);
    const int kk = (int)clamp64(a.n_tiles, 0, a.k_sel);
    TopkSmem &tsm = *reinterpret_cast<TopkSmem *>(sm + FSmem::kTopk);
    unsigned long long *cand = reinterpret_cast<unsigned long long *>(sm + FSmem::kCand);
    if (kk > 0) {
      if (kk <= 32) {
        block_topk_warp32<kFThreads>(gs, a.n_tiles, kk, tsm.lists, cand);
      } else {
        block_topk<kFThreads>([&](int64_t i) -> float { return gs[i]; }, a.n_tiles, kk, cand, tsm);
      }
    }
    KVR_TRACE_POINT(3, 2);
    for (int j = tid; j < a.k_sel; j += kFThreads) {
      const int32_t v = j < kk ? (int32_t)key_index(cand[j]) : -1;
      sel_s[j] = v;
      if (a.sel_out) a.sel_out[row * a.k_sel + j] = v;
    }
    __syncthreads();
    KVR_TRACE_POINT(2, 6);
    cluster_arrive();  // S2: selection ready
    cluster_wait();
  } else {
    // exact window/tail share of ranks 1..CS-1 while rank 0 selects
    const int64_t e_begin = ex_begin, e_end = e_begin + ex_per < n_ex ? e_begin + ex_per : n_ex;
    // the first chunk was loaded at kernel start and staged after phase 1
    for (int64_t e = e_begin; e < e_end; e += kFChunk) {
      const int nt = (int)clamp64(e_end - e, 0, kFChunk);
      if (e != e_begin) {
        ExactRegs r2;
        fused_exact_load(a, b, h, e, nt, r2);
        __syncthreads();
        fused_exact_store(sm, r2);
      }
      __syncthreads();
      fused_exact_compute(a, sm, nt);
    }
    cluster_wait();
    cluster_arrive();
    cluster_wait();
  }

  KVR_TRACE_POINT(2, 4);
  // ---- phase 3: selected tiles, slot j -> rank j % CS
  {
    const int32_t *sel0 = cluster.map_shared_rank(sel_s, 0);
    unsigned phase = 0;
    for (int j = rank; j < a.k_sel; j += CS) {
      const int32_t t = sel0[j];  // uniform across the CTA
      if (t >= 0) fused_tile<TILE>(a, sm, row, t, phase);
    }
  }
  __syncthreads();
  KVR_TRACE_POINT(2, 5);
  cluster_arrive();  // S3: partials final

  if (rank == 0) {
    cluster_wait();
    KVR_TRACE_POINT(2, 6);
    float *W = reinterpret_cast<float *>(sm + FSmem::kS);    // [16][8]
    float *ML = reinterpret_cast<float *>(sm + FSmem::kP);   // [8][2] merged (M, L)
    float *Ex = reinterpret_cast<float *>(sm + FSmem::kKs);  // [8][128]
    float *Tr = Ex + kFMaxG * kD;                            // [8][128]
    for (int hq = warp; hq < g; hq += kFWarps) {
      float mr = -INFINITY, lr = 0.0f;
      if (lane < CS) {
        mr = cluster.map_shared_rank(M, lane)[hq];
        lr = cluster.map_shared_rank(L, lane)[hq];
      }
      const float mx = warp_max(mr);
      const float w = (mr == -INFINITY) ? 0.0f : expf(mr - mx);
      if (lane < CS) W[lane * kFMaxG + hq] = w;
      const float ls = warp_sum(w * lr);
      if (lane == 0) {
        ML[2 * hq] = mx;
        ML[2 * hq + 1] = ls;
      }
    }
    __syncthreads();
    for (int i = tid; i < g * kD; i += kFThreads) {
      const int hq = i >> 7;
      float e[16], t[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        e[r] = r < CS ? cluster.map_shared_rank(oex, r)[i] : 0.0f;
        t[r] = r < CS ? cluster.map_shared_rank(otr, r)[i] : 0.0f;
      }
      float ex = 0.0f, tr = 0.0f;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const float w = r < CS ? W[r * kFMaxG + hq] : 0.0f;
        ex = fmaf(w, e[r], ex);
        tr = fmaf(w, t[r], tr);
      }
      Ex[i] = ex;
      Tr[i] = tr;
    }
    __syncthreads();
    for (int hq = warp; hq < g; hq += kFWarps) {
      float x[4];
      const float4 t4 = reinterpret_cast<const float4 *>(Tr + hq * kD)[lane];
      x[0] = t4.x; x[1] = t4.y; x[2] = t4.z; x[3] = t4.w;
      transform128(x, lane, a.kind, true, reinterpret_cast<float *>(sm + FSmem::kBuf) + (hq % (kFMaxG + 1)) * 2 * kD, lee);
      const float4 e4 = reinterpret_cast<const float4 *>(Ex + hq * kD)[lane];
      const float Lh = ML[2 * hq + 1];
      const float inv = Lh > 0.0f ? 1.0f / Lh : 0.0f;
      const float y[4] = {(e4.x + x[0]) * inv, (e4.y + x[1]) * inv, (e4.z + x[2]) * inv, (e4.w + x[3]) * inv};
      const int64_t qh = b * a.n_q + (int64_t)h * g + hq;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t idx = qh * kD + lane * 4 + r;
        if (a.out_dt == KVR_F32) store_elem<KVR_F32>(a.out, idx, y[r]);
        else if (a.out_dt == KVR_F16) store_elem<KVR_F16>(a.out, idx, y[r]);
        else store_elem<KVR_BF16>(a.out, idx, y[r]);
      }
    }
    __syncthreads();
    KVR_TRACE_POINT(2, 7);
    cluster_arrive();  // S4: rank 0 is done reading the other CTAs
    cluster_wait();
  } else {
    cluster_wait();
    cluster_arrive();
    cluster_wait();
  }
}

// ------------------------------------------------------------------ host ----
size_t fused_smem_bytes(int tile, int nt_per) {
  return FSmem::kFixed + align_up((size_t)nt_per * 4, 128) + (size_t)nt_per * (tile * 16 + kD * 2);
}

// Cluster size usable for this kernel on the current device (16, 8, or 0).
// (one wave: every row's cluster co-resident).
template <int TILE>
static int pick_cluster(int64_t rows, int nt_per_16, int nt_per_8) {
  for (int cs : {16, 8}) {
    const int np = cs == 16 ? nt_per_16 : nt_per_8;
    const size_t sb = fused_smem_bytes(TILE, np);
    if (sb > 227 * 1024) continue;
    cudaFuncSetAttribute(sd1_fused_kernel<TILE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sb);
    if (cs == 16) cudaFuncSetAttribute(sd1_fused_kernel<TILE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(cs, 1, 1);
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = sb;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, sd1_fused_kernel<TILE>, &cfg) == cudaSuccess && n >= rows) return cs;
    cudaGetLastError();
  }
  return 0;
}

// Returns KVR_OK if launched, KVR_ENOTSUP if this configuration should use
// the two-kernel path instead.
int sd1_fused_launch(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint16_t *win_k,
                     const uint16_t *win_v, int64_t win_cap, int64_t n_win, const uint16_t *tail_k,
                     const uint16_t *tail_v, int64_t n_tail, const uint32_t *kbits, const uint16_t *kscale,
                     const uint32_t *vbits, const uint16_t *vscale, int64_t nt_cap, int64_t n_tiles, int tile,
                     int kind, int k_sel, int64_t ex_t0, int64_t ex_t1, float scale, void *out, int out_dtype,
                     int32_t *sel_out, unsigned *err, cudaStream_t st) {
  const int g = n_q / n_kv;
  if (g > kFMaxG || k_sel > kFMaxSel || n_tiles > kFMaxTiles || n_tiles < 1 || (n_win + n_tail) < 1)
    return KVR_ENOTSUP;
  const int np16 = (int)((n_tiles + 15) / 16), np8 = (int)((n_tiles + 7) / 8);
  int cs = 0;
  switch (tile) {
    case 32: cs = pick_cluster<32>((int64_t)batch * n_kv, np16, np8); break;
    case 64: cs = pick_cluster<64>((int64_t)batch * n_kv, np16, np8); break;
    case 128: cs = pick_cluster<128>((int64_t)batch * n_kv, np16, np8); break;
    default: return KVR_ENOTSUP;
  }
  if (cs == 0) return KVR_ENOTSUP;
  FusedArgs a{};
  a.q = q; a.q_dt = q_dtype; a.n_q = n_q; a.n_kv = n_kv; a.g = g;
  a.inv_scale = (float)(1.0 / (scale > 0.f ? (double)scale : sqrt((double)kD)));
  a.win_k = win_k; a.win_v = win_v; a.win_cap = win_cap; a.n_win = n_win;
  a.tail_k = tail_k; a.tail_v = tail_v; a.n_tail = n_tail; a.tail_cap = tile;
  a.kbits = kbits; a.kscale = kscale; a.vbits = vbits; a.vscale = vscale;
  a.nt_cap = nt_cap; a.n_tiles = n_tiles; a.ex_t0 = ex_t0; a.ex_t1 = ex_t1;
  a.kind = kind; a.k_sel = k_sel; a.cs = cs; a.nt_per = cs == 16 ? np16 : np8;
  a.out = out; a.out_dt = out_dtype; a.sel_out = sel_out; a.err = err;
  const size_t sb = fused_smem_bytes(tile, a.nt_per);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(cs, n_kv, batch);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = sb;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (tile) {
    case 32: e = cudaLaunchKernelEx(&cfg, sd1_fused_kernel<32>, a); break;
    case 64: e = cudaLaunchKernelEx(&cfg, sd1_fused_kernel<64>, a); break;
    default: e = cudaLaunchKernelEx(&cfg, sd1_fused_kernel<128>, a); break;
  }
  if (e != cudaSuccess) return set_error(KVR_ECUDA, "sd1 fused decode launch: %s", cudaGetErrorString(e));
  return KVR_OK;
}

}  // namespace kvr

#ifdef KVR_TRACE
extern "C" KVR_API int kvr_debug_trace_fused(unsigned long long *host, int n) {
  return cudaMemcpyFromSymbol(host, kvr::g_kvr_trace, sizeof(unsigned long long) * n) == cudaSuccess ? 0 : 2;
}
#endif
