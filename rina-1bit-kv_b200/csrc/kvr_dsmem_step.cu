// One-kernel sd1 decode step for few (b, h) rows (batch-1 decode), sm_100a.
//
// The split path (selection kernel -> attention kernel -> last-CTA merge
// through L2) is a chain of dependent phases: at batch 1 each layer spends
// ~20 us on launch hand-offs, global counters and L2 round trips while the
// layer's compressed bytes need ~1.2 us of HBM time.  Here every (b, h) row
// is ONE thread-block cluster of C CTAs (C = 16, or 8 where 16-CTA clusters
// cannot be placed) and the whole step runs inside it:
//
//  0. before the grid dependency wait (overlapping the previous kernel):
//     CTA r bulk-copies its range of the row's tiles (K bits + K scales, one
//     contiguous copy each) into shared memory as far as the staging buffer
//     holds them, and prefetches the rest and its exact rows into L2;
//  1. after the wait, CTA r cp.async-stages its share of the exact rows
//     (window ring + pending tail, fp16; consumed after the scan) and reads
//     q; warp 0 forms q' = T(group mean), warps 1..g the per-head T q_h, the
//     rest the scaled natural q;
//  2. scan: the CTA's tiles are scored from shared memory with the
//     selection kernel's arithmetic (sd1_score_tile2: identical scores);
//     warp 0 keeps the CTA's top-32 keys (score desc, index asc) in a list;
//  3. cluster barrier; every CTA reads the C lists over distributed shared
//     memory and finds the keys of its own ranks (r, r + C) by binary search
//     (rank of a key = number of larger keys in all lists) -- the global top
//     k_sel lies in the union of the per-CTA top k_sel lists, keys are unique,
//     so the selection equals the split path's exactly;
//  4. the chosen tiles' K/V bits + scales are bulk-copied in; meanwhile the
//     warps attend the CTA's exact rows (natural domain);
//  5. the chosen tiles are attended in the transformed domain (nibble LUT
//     scores, bit-serial P.V), folded with the exact part per warp;
//  6. each CTA folds its warps per query head and stores the (m, l, o_exact,
//     o_transformed) row into the receive buffer of the CTA that merges that
//     head (st.shared::cluster); cluster barrier; the merging CTAs combine
//     the C rows, inverse-transform the transformed part and write out.
//
// No global scratch but the error word; no atomics; two cluster barriers.
// Bounded waits on every mbarrier; a wait that gives up sets the error word,
// lets its copies land (bounded) and the CTA still arrives at both cluster
// barriers, so a failure never leaves a cluster waiting.
//
// Reference behaviour replaced (same as the split path): retrieval + exact
// softmax over window + retrieved tokens (modules/kvr_retrieval.py:317-412,
// kvr_hook.py:274-282, kvr_triton.py:93-104), with the 1-bit codec.
#include "kvr_common.cuh"
#include "kvr_sd1_score.cuh"
#include "kvr_topk.cuh"
#include "kvr_transform.cuh"

#include <cstdlib>
#include <mutex>

namespace kvr {

constexpr int kDsMaxG = 8;
constexpr int kDsList = 32;         // per-CTA list length (k_sel <= 32)
constexpr int kDsExStride = 272;    // bytes per staged fp16 row (256 + 16: conflict-free 16-byte loads)
constexpr int kDsPart = 4 + 2 * kD; // floats per partial row: m, l, pad, pad, o_exact[128], o_tr[128]
constexpr int kDsStageMaxBytes = 48 * 1024;
constexpr int kDsMaxExact = 96;     // exact rows per CTA
constexpr int kDsMaxTpc = 1024;
     // tiles per CTA (beyond the staged ones they are read from global)

struct DsArgs {
  const void *q;
  int q_dt, n_q, n_kv, g;
  float inv_scale;
  const uint16_t *win_k, *win_v;
  int64_t win_cap, n_win;
  const uint16_t *tail_k, *tail_v;
  int64_t n_tail;
  const uint32_t *kbits;
  const uint16_t *kscale;
  const uint32_t *vbits;
  const uint16_t *vscale;
  int64_t nt_cap, n_tiles;
  int tile, kind, k_sel;
  int64_t ex0, ex1;
  void *out;
  int out_dt;
  float *partial_out;
  int32_t *sel_out;
  unsigned *err;
  // fused store update (upd != 0, batch 1): q is pre-RoPE; the new token's
  // pre-RoPE k and v (n_kv x 128, q's dtype) go to window slot `slot`; the
  // slot's old row becomes tail row `evict_row` (-1: nothing is evicted);
  // q_out (optional) receives the rotated q
  int upd;
  const void *k_new, *v_new;
  const float *cos_row, *sin_row;
  void *q_out;
  int64_t slot, evict_row;
  int tpc, staged, epc;
  // shared-memory plan (bytes, set by the host)
  int o_lists, o_sc, o_region, o_lut, o_p, o_ex, o_tiles, o_wpart, smem;
};

// ---- cluster primitives (PTX)
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_shared(const void *p, unsigned cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(cta));
  return r;
}
__device__ __forceinline__ unsigned long long ld_cluster_u64(uint32_t addr) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_cluster_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float load_q1(const void *p, int64_t i, int dt) {
  if (dt == KVR_F32) return load1<KVR_F32>(p, i);
  if (dt == KVR_F16) return load1<KVR_F16>(p, i);
  return load1<KVR_BF16>(p, i);
}

// q rows of the cluster's g heads into Qn (rotated when the store update is
// fused; CTA 0 also writes them to q_out).  Every load of a thread is
// issued before any of them is used: one round trip.
template <int DT>
__device__ __forceinline__ void stage_q_rows(const DsArgs &a, int64_t qb, int g, int tid, unsigned my, float *Qn) {
  constexpr int kMaxPer = kDsMaxG * kD / 256;  // q elements per thread, at most
  float x[kMaxPer], p[kMaxPer], cs[kMaxPer], sn[kMaxPer];
  const int n = g * kD;
#pragma unroll
  for (int u = 0; u < kMaxPer; ++u) {
    const int i = tid + 256 * u;
    if (i < n) {
      const int c = i & (kD - 1);
      x[u] = load1<DT>(a.q, qb + i);
      if (a.upd) {
        p[u] = load1<DT>(a.q, qb + (c < kD / 2 ? i + kD / 2 : i - kD / 2));
        cs[u] = __ldg(a.cos_row + c);
        sn[u] = __ldg(a.sin_row + c);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < kMaxPer; ++u) {
    const int i = tid + 256 * u;
    if (i < n) {
      const int c = i & (kD - 1);
      const float v = a.upd ? rope_elem<DT>(x[u], p[u], c < kD / 2, cs[u], sn[u]) : x[u];
      Qn[i] = v;
      if (a.q_out != nullptr && my == 0) store_elem<DT>(a.q_out, qb + i, v);
    }
  }
}

// The new token's window row (head h) from the raw rows staged in shared
// memory (raw: [k (128 of DT)][v][cos row fp32][sin row fp32], 512 B each):
// lanes 0-15 rotate 8 K channels each, lanes 16-31 convert 8 V channels; the
// fp16 chunks go to the staged K / V rows and to the window slot in global
// memory.
template <int DT>
__device__ __forceinline__ void build_new_row(const unsigned char *raw, unsigned char *k_row, unsigned char *v_row,
                                              uint16_t *g_k, uint16_t *g_v, int lane) {
  const int kv = lane >> 4, c8 = (lane & 15) * 8;
  float x[kChunk8];
  uint4 out;
  if (kv) {
    load8<DT>(raw + 512, c8, x);
    out = pack_f16x8(x);
  } else {
    float p[kChunk8], cs[kChunk8], sn[kChunk8], r[kChunk8];
    load8<DT>(raw, c8, x);
    load8<DT>(raw, (c8 + kD / 2) % kD, p);
    load8<KVR_F32>(raw + 1024, c8, cs);
    load8<KVR_F32>(raw + 1536, c8, sn);
    const bool lo = c8 < kD / 2;
#pragma unroll
    for (int e = 0; e < kChunk8; ++e) r[e] = rope_elem<DT>(x[e], p[e], lo, cs[e], sn[e]);
    out = pack_f16x8(r);
  }
  *reinterpret_cast<uint4 *>((kv ? v_row : k_row) + c8 * 2) = out;
  *reinterpret_cast<uint4 *>((kv ? g_v : g_k) + c8) = out;
}

// number of keys > x in a descending list of n keys
__device__ __forceinline__ int count_greater(const unsigned long long *list, int n, unsigned long long x) {
  int lo = 0, hi = n;  // list[0, lo) > x, list[hi, n) <= x
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (list[mid] > x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// Stamp for phase studies (trace builds only): thread `owner` of the CTA.
#ifdef KVR_TRACE
#define DS_TRACE(id, point, owner)                                                 \
  do {                                                                             \
    if (threadIdx.x == (owner)) {                                                  \
      unsigned long long t_;                                                       \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                       \
      const unsigned blk_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z); \
      if (blk_ < 2048) g_kvr_trace[((id) * 2048 + blk_) * 8 + (point)] = t_;       \
    }                                                                              \
  } while (0)
#else
#define DS_TRACE(id, point, owner) ((void)0)
#endif

#define DS_FN __device__ __forceinline__

// Named barrier of the first 128 threads (warps 0-3: the selection group).
__device__ __forceinline__ void sel_group_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Descending top-32 of two descending 32-key lists held one key per lane.
__device__ __forceinline__ unsigned long long merge_top32(unsigned long long a, unsigned long long b_desc, int lane) {
  const unsigned long long b_rev = __shfl_sync(0xffffffffu, b_desc, 31 - lane);
  return warp_bitonic_merge_desc(a > b_rev ? a : b_rev, lane);
}

// Exact softmax partial of query head hq over the CTA's staged rows [0, n):
// (m, l) and o (channels 4 lane .. 4 lane + 3), scores q.k * inv_scale.
DS_FN void exact_rows(const unsigned char *ex, int epc, int n, const float *qn, float &m_out,
                                           float &l_out, float (&o)[4], int lane) {
  const float4 *q4 = reinterpret_cast<const float4 *>(qn);
  constexpr int R = kDsMaxExact / 32;
  float sj[R];
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int rows = n - 32 * r;  // rows of this pass (warp-uniform)
    sj[r] = -INFINITY;
    if (rows <= 0) continue;
    // a full pass gives each lane a row; a short one (fewer than 16 rows,
    // e.g. the few pending-tail rows past 32) splits each row's 16 chunks
    // over a group of lanes and reduces them, so it costs a fraction of a pass
    const int lpr = rows >= 16 ? 1 : rows > 8 ? 2 : rows > 4 ? 4 : rows > 2 ? 8 : 16;
    const int row = lane / lpr, part = lane - row * lpr, nch = 16 / lpr;
    float v = -INFINITY;
    if (row < rows) {
      const uint4 *kr = reinterpret_cast<const uint4 *>(ex + (32 * r + row) * kDsExStride);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
      for (int c = part * nch; c < (part + 1) * nch; ++c) {
        const uint4 w = kr[c];
        const float4 qa = q4[2 * c], qb4 = q4[2 * c + 1];
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
        const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&w.z));
        const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&w.w));
        acc[0] = fmaf(qa.x, f0.x, acc[0]); acc[1] = fmaf(qa.y, f0.y, acc[1]);
        acc[2] = fmaf(qa.z, f1.x, acc[2]); acc[3] = fmaf(qa.w, f1.y, acc[3]);
        acc[0] = fmaf(qb4.x, f2.x, acc[0]); acc[1] = fmaf(qb4.y, f2.y, acc[1]);
        acc[2] = fmaf(qb4.z, f3.x, acc[2]); acc[3] = fmaf(qb4.w, f3.y, acc[3]);
      }
      v = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    }
    if (lpr > 1) {
      for (int o = lpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      v = __shfl_sync(0xffffffffu, v, (lane * lpr) & 31);  // row `lane`'s sum, from its group
      if (lane >= rows) v = -INFINITY;
    }
    sj[r] = v;
    mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  o[0] = o[1] = o[2] = o[3] = 0.0f;
  m_out = mx;
  l_out = 0.0f;
  if (mx == -INFINITY) return;
  float l = 0.0f;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    sj[r] = (lane + 32 * r < n) ? expf(sj[r] - mx) : 0.0f;
    l += sj[r];
  }
  l_out = warp_sum(l);
  const unsigned char *vrows = ex + epc * kDsExStride + lane * 8;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int jn = min(32, n - 32 * r);
    for (int jj = 0; jj < jn; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, sj[r], jj);
      const uint2 w = *reinterpret_cast<const uint2 *>(vrows + (32 * r + jj) * kDsExStride);
      const float2 v0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
      const float2 v1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
      o[0] = fmaf(pj, v0.x, o[0]); o[1] = fmaf(pj, v0.y, o[1]);
      o[2] = fmaf(pj, v1.x, o[2]); o[3] = fmaf(pj, v1.y, o[3]);
    }
  }
}

template <int TILE, int C>
__global__ void __launch_bounds__(256, 2) sd1_dsmem_step_kernel(DsArgs a) {
  extern __shared__ __align__(128) unsigned char sm[];
  constexpr int TPL = TILE / 32;
  constexpr unsigned kTileBits = TILE * 16;
  constexpr int kTileBytes = 2 * kTileBits + 2 * kD * 2;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned my = cluster_rank();
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t row = b * a.n_kv + h;
  const int g = a.g;

  float *lee = reinterpret_cast<float *>(sm);                              // [128]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + 512);                  // [0] stage, [1] tiles
  int *flags = reinterpret_cast<int *>(sm + 528);                           // [0] stage ok, [1] tiles ok, [2..3] sel
  float *qp = reinterpret_cast<float *>(sm + 576);                          // [128] group-mean q'
  float *Qn = reinterpret_cast<float *>(sm + 576 + 512);                    // [g][128] q * inv_scale
  float *Qt = Qn + kDsMaxG * kD;                                            // [g][128] T q_h * inv_scale
  unsigned long long *lists = reinterpret_cast<unsigned long long *>(sm + a.o_lists);  // [C][32]
  float *sc = reinterpret_cast<float *>(sm + a.o_sc);                       // [tpc]
  unsigned char *region = sm + a.o_region;  // scan staging; then the receive buffer [C][kDsPart]
  float *recv = reinterpret_cast<float *>(region);
  float *lut = reinterpret_cast<float *>(sm + a.o_lut);                     // per warp [32][17]
  float *pbuf = reinterpret_cast<float *>(sm + a.o_p);                      // per warp [TILE]
  unsigned char *ex = sm + a.o_ex;                                          // [2][epc] rows
  unsigned char *tiles = sm + a.o_tiles;                                    // [2] x (KB, VB, KS, VS)
  float *wpart = reinterpret_cast<float *>(sm + a.o_wpart);                 // [8][kDsPart] warp rows
  float *xpart = wpart + 8 * kDsPart;                                       // [g][4 + 128] exact rows

  KVR_TRACE_POINT(0, 0);
#ifdef KVR_TRACE
  if (tid == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    const unsigned blk = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (blk < 2048) g_kvr_trace[(2 * 2048 + blk) * 8] = smid + 1;
  }
#endif
  // ---- 0. stage this CTA's store range and exact rows
  const int64_t t0 = (int64_t)my * a.tpc;
  const int n_mine = (int)max((int64_t)0, min(a.n_tiles, t0 + a.tpc) - t0);
  const int n_staged = min(n_mine, a.staged);
  const int64_t n_ex = a.n_win + a.n_tail;
  const int64_t e0 = (int64_t)my * a.epc;
  const int ex_mine = (int)max((int64_t)0, min(n_ex, e0 + a.epc) - e0);
  const int64_t tokw = (int64_t)a.n_kv * kD;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    flags[0] = 1;
    flags[1] = 1;
    if (n_staged > 0) {
      const int64_t tix = row * a.nt_cap + t0;
      mbar_expect_tx(&bars[0], (unsigned)n_staged * (kTileBits + kD * 2));
      bulk_g2s(region, a.kbits + tix * TILE * 4, (unsigned)n_staged * kTileBits, &bars[0]);
      bulk_g2s(region + a.staged * kTileBits, a.kscale + tix * kD, (unsigned)n_staged * kD * 2, &bars[0]);
    }
  }
  // L2 prefetch of what this CTA later reads from global memory: the tiles
  // beyond the staging buffer (read by the scan) and its window/tail row
  // slices (staged after the wait).  Hints only, so they may precede the wait.
  if (tid == 32 && n_mine > n_staged) {
    const int64_t tix = row * a.nt_cap + t0 + n_staged;
    prefetch_l2(a.kbits + tix * TILE * 4, (unsigned)(n_mine - n_staged) * kTileBits);
    prefetch_l2(a.kscale + tix * kD, (unsigned)(n_mine - n_staged) * kD * 2);
  }
  for (int i = tid; i < ex_mine * 2; i += 256) {
    const int j = i >> 1, kv = i & 1;
    const int64_t e = e0 + j;
    const uint16_t *src = e < a.n_win ? (kv ? a.win_v : a.win_k) + (b * a.win_cap + e) * tokw
                                      : (kv ? a.tail_v : a.tail_k) + (b * TILE + (e - a.n_win)) * tokw;
    prefetch_l2(src + (int64_t)h * kD, kD * 2);
  }
  if (a.kind == KVR_DCT) load_lee(lee);

  // ---- 1. queries and exact rows (the previous kernel may write both: the
  // per-layer store update writes q, the window slot and the tail).
  // Everything above reads only the store's tiles: a kernel that lets this
  // one start early (griddepcontrol.launch_dependents) must not write those
  // -- in this library the attention kernels and the store update do not.
  griddep_wait();
  asm volatile("griddepcontrol.launch_dependents;");
  // the exact rows are consumed after the scan: their copies overlap it
  // (fused store update: the slot's row is the new token's, built by the
  // exact-row warps after the first cluster barrier; the evicted tail row is
  // read from the slot, and its CTA waits for that copy before the barrier,
  // so the slot may be overwritten after it)
  const bool slot_here = a.upd && a.slot >= e0 && a.slot < e0 + ex_mine;
  const bool evict_here = a.upd && a.evict_row >= 0 && a.n_win + a.evict_row >= e0 &&
                          a.n_win + a.evict_row < e0 + ex_mine;
  unsigned char *raw = reinterpret_cast<unsigned char *>(wpart);  // free until the warp fold
  if (slot_here && tid < 128) {
    // the new row's raw inputs (k, v of q's dtype; the RoPE table rows)
    const int part = tid >> 5, c = tid & 31;
    const int esz = a.q_dt == KVR_F32 ? 4 : 2;
    const unsigned char *src = part == 0   ? static_cast<const unsigned char *>(a.k_new) + (int64_t)h * kD * esz
                               : part == 1 ? static_cast<const unsigned char *>(a.v_new) + (int64_t)h * kD * esz
                               : part == 2 ? reinterpret_cast<const unsigned char *>(a.cos_row)
                                           : reinterpret_cast<const unsigned char *>(a.sin_row);
    if (part >= 2 || c * 16 < kD * esz) cp_async16(raw + part * 512 + c * 16, src + c * 16);
  }
  for (int i = tid; i < ex_mine * 32; i += 256) {
    const int j = i >> 5, kv = (i >> 4) & 1, c = i & 15;
    const int64_t e = e0 + j;
    unsigned char *dst = ex + (kv * a.epc + j) * kDsExStride + c * 16;
    if (a.upd && e == a.slot) continue;  // built by the exact-row warps
    const bool evicted = a.upd && e - a.n_win == a.evict_row;
    const uint16_t *src = e < a.n_win || evicted
                              ? (kv ? a.win_v : a.win_k) + (b * a.win_cap + (evicted ? a.slot : e)) * tokw
                              : (kv ? a.tail_v : a.tail_k) + (b * TILE + (e - a.n_win)) * tokw;
    cp_async16(dst, src + (int64_t)h * kD + c * 8);
  }
  cp_async_commit();
  KVR_TRACE_POINT(0, 1);
  const int64_t qb = (b * a.n_q + (int64_t)h * g) * kD;
  // the row's g query heads, read (and rotated, when the store update is
  // fused) once, in one round trip: Qn holds them unscaled until the
  // transforms below have read them
  if (a.q_dt == KVR_F32) stage_q_rows<KVR_F32>(a, qb, g, tid, my, Qn);
  else if (a.q_dt == KVR_F16) stage_q_rows<KVR_F16>(a, qb, g, tid, my, Qn);
  else stage_q_rows<KVR_BF16>(a, qb, g, tid, my, Qn);
  __syncthreads();  // q rows, Lee factors, barrier init
  // task 0 (warp 0): group mean (ordered sum) -> q' for the scan; task 1 + i:
  // T q of head i for the tile attention (warp 0 also takes head 7 when
  // g = 8).  One transform call site keeps the kernel's code small (every
  // layer's launch fetches it again).
  {
    const bool dct = a.kind == KVR_DCT;
    for (int task = warp; task <= g; task += 8) {
      float x[4];
      const int src = task == 0 ? 0 : (task - 1) * kD;
#pragma unroll
      for (int s = 0; s < 4; ++s) x[s] = Qn[src + (dct ? lane + 32 * s : lane * 4 + s)];
      if (task == 0) {
        for (int i = 1; i < g; ++i)
#pragma unroll
          for (int s = 0; s < 4; ++s) x[s] = __fadd_rn(x[s], Qn[i * kD + (dct ? lane + 32 * s : lane * 4 + s)]);
#pragma unroll
        for (int s = 0; s < 4; ++s) x[s] = __fdiv_rn(x[s], (float)g);
      }
      if (dct) dct128_fwd_shfl(x, lane, lee);
      else wht128(x, lane);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int c = dct ? lane + 32 * s : lane * 4 + s;
        if (task == 0) qp[c] = x[s];
        else Qt[(task - 1) * kD + c] = x[s] * a.inv_scale;
      }
    }
  }
  __syncthreads();  // the transforms have read the unscaled rows
  for (int i = tid; i < g * kD; i += 256) Qn[i] *= a.inv_scale;
  __syncthreads();
  KVR_TRACE_POINT(0, 2);

  // ---- 2. scan of the CTA's tiles
  if (n_staged > 0 && !mbar_wait_bounded(&bars[0], 0)) {
    if (lane == 0) atomicOr(a.err, 1u);
    flags[0] = 0;
    mbar_wait_bounded(&bars[0], 0);
  }
  __syncthreads();
  DS_TRACE(1, 0, 0);
  const bool stage_ok = flags[0] != 0;
  const uint4 *skb = reinterpret_cast<const uint4 *>(region);
  const uint16_t *sks = reinterpret_cast<const uint16_t *>(region + a.staged * kTileBits);
  for (int p0 = 2 * warp; p0 < n_mine; p0 += 16) {
    uint4 kb[2][TPL];
    uint16_t ks[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int lt = min(p0 + u, n_mine - 1);  // a lone last tile is scored twice, stored once
      if (lt < n_staged) {
#pragma unroll
        for (int r = 0; r < TPL; ++r) kb[u][r] = skb[lt * TILE + lane + 32 * r];
#pragma unroll
        for (int m = 0; m < 4; ++m) ks[u][m] = sks[lt * kD + lane + 32 * m];
      } else {
        const int64_t tix = row * a.nt_cap + t0 + lt;
        const uint4 *src = reinterpret_cast<const uint4 *>(a.kbits + tix * TILE * 4);
#pragma unroll
        for (int r = 0; r < TPL; ++r) kb[u][r] = __ldg(src + lane + 32 * r);
#pragma unroll
        for (int m = 0; m < 4; ++m) ks[u][m] = __ldg(a.kscale + tix * kD + lane + 32 * m);
      }
    }
    float s2[2];
    sd1_score_tile2<TILE>(qp, kb, ks, lane, s2);
    if (lane == 0) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int lt = p0 + u;
        const int64_t t = t0 + lt;
        if (lt < n_mine) sc[lt] = (t >= a.ex0 && t < a.ex1) || !stage_ok ? -INFINITY : s2[u];
      }
    }
  }
  __syncthreads();
  KVR_TRACE_POINT(0, 3);
  if (warp == 0) {
    unsigned long long list = lane < n_mine ? make_key(sc[lane], t0 + lane) : 0ull;
    list = warp_sort_desc(list, lane);
    for (int c0 = 32; c0 < n_mine; c0 += 32) {
      const int i = c0 + lane;
      const unsigned long long key = i < n_mine ? make_key(sc[i], t0 + i) : 0ull;
      list = warp_fold_top32(list, warp_sort_desc(key, lane), lane);
    }
    lists[my * kDsList + lane] = list;
  }

  // ---- 3. global top-k: tree merge of the C lists (level 1 straight from
  // the owners' shared memory); meanwhile warps 4-7 attend the exact rows
  // the CTA that staged the evicted row (a copy of the slot's old row) has
  // it before the barrier; after it the slot may be overwritten
  if (evict_here) cp_async_wait<0>();
  cluster_sync_all();
  KVR_TRACE_POINT(0, 4);
  if (warp < C / 2) {
    const unsigned ca = 2 * warp, cb = 2 * warp + 1;
    const unsigned long long ka =
        ca == my ? lists[ca * kDsList + lane] : ld_cluster_u64(map_shared(&lists[ca * kDsList + lane], ca));
    const unsigned long long kb2 =
        cb == my ? lists[cb * kDsList + lane] : ld_cluster_u64(map_shared(&lists[cb * kDsList + lane], cb));
    // level-1 lists go to local scratch (the tile-attention P rows, free
    // until the tiles arrive); the owners' lists are never written again
    const unsigned long long m = merge_top32(ka, kb2, lane);
    reinterpret_cast<unsigned long long *>(pbuf)[warp * 32 + lane] = m;
  }
  __syncthreads();
  cp_async_wait<0>();  // this thread's exact-row copies
  __syncthreads();
  if (warp < 4) {
    // selection group: levels 2.. of the tree over the C/2 level-1 lists
    unsigned long long *l1 = reinterpret_cast<unsigned long long *>(pbuf);
    for (int n = C / 2; n > 1; n >>= 1) {
      unsigned long long m = 0ull;
      if (warp < n / 2) m = merge_top32(l1[(2 * warp) * 32 + lane], l1[(2 * warp + 1) * 32 + lane], lane);
      sel_group_sync();
      if (warp < n / 2) l1[warp * 32 + lane] = m;
      sel_group_sync();
    }
    if (warp == 0) {
      // l1[0..32) = global top-32 (descending; 0 = empty)
      const int k_eff = (int)min((int64_t)a.k_sel, a.n_tiles);
      const unsigned long long key = l1[lane];
      int sel[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = (int)my + u * C;
        const unsigned long long kr = __shfl_sync(0xffffffffu, key, r & 31);
        sel[u] = (r < k_eff && kr != 0ull) ? (int)key_index(kr) : -1;
        if (a.sel_out != nullptr && lane == 0 && r < a.k_sel) a.sel_out[row * a.k_sel + r] = sel[u];
      }
      const int n_sel = (sel[0] >= 0) + (sel[1] >= 0);
      if (lane == 0) {
        flags[2] = sel[0];
        flags[3] = sel[1];
        if (n_sel > 0) {
          mbar_expect_tx(&bars[1], (unsigned)n_sel * kTileBytes);
          for (int s = 0; s < n_sel; ++s) {
            const int64_t tix = row * a.nt_cap + sel[s];
            unsigned char *dst = tiles + s * kTileBytes;
            bulk_g2s(dst, a.kbits + tix * TILE * 4, kTileBits, &bars[1]);
            bulk_g2s(dst + kTileBits, a.vbits + tix * TILE * 4, kTileBits, &bars[1]);
            bulk_g2s(dst + 2 * kTileBits, a.kscale + tix * kD, kD * 2, &bars[1]);
            bulk_g2s(dst + 2 * kTileBits + kD * 2, a.vscale + tix * kD, kD * 2, &bars[1]);
          }
        }
      }
    }
    DS_TRACE(1, 1, 0);
  } else {
    // exact group: the exact rows of every head (fused store update: first
    // the new window row, and the evicted row goes to the tail)
    if (slot_here) {
      if (warp == 7) {
        unsigned char *kr = ex + (a.slot - e0) * kDsExStride, *vr = ex + (a.epc + a.slot - e0) * kDsExStride;
        // the fused entry point passes writable window and tail buffers
        uint16_t *gk = const_cast<uint16_t *>(a.win_k) + (b * a.win_cap + a.slot) * tokw + (int64_t)h * kD;
        uint16_t *gv = const_cast<uint16_t *>(a.win_v) + (b * a.win_cap + a.slot) * tokw + (int64_t)h * kD;
        if (a.q_dt == KVR_F32) build_new_row<KVR_F32>(raw, kr, vr, gk, gv, lane);
        else if (a.q_dt == KVR_F16) build_new_row<KVR_F16>(raw, kr, vr, gk, gv, lane);
        else build_new_row<KVR_BF16>(raw, kr, vr, gk, gv, lane);
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");  // warps 4-7
    }
    if (evict_here && warp == 6) {
      const int kv = lane >> 4, c = lane & 15;
      const int64_t j = a.n_win + a.evict_row - e0;
      uint16_t *dst = const_cast<uint16_t *>(kv ? a.tail_v : a.tail_k) + (b * TILE + a.evict_row) * tokw +
                      (int64_t)h * kD + c * 8;
      *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(ex + (kv * a.epc + j) * kDsExStride + c * 16);
    }
    const int wi = warp - 4;
    for (int hh = wi; hh < g; hh += 4) {
      float m, l, o[4];
      exact_rows(ex, a.epc, ex_mine, Qn + hh * kD, m, l, o, lane);
      float *xp = xpart + hh * (4 + kD);
      if (lane == 0) {
        xp[0] = m;
        xp[1] = l;
      }
      reinterpret_cast<float4 *>(xp + 4)[lane] = make_float4(o[0], o[1], o[2], o[3]);
    }
    DS_TRACE(1, 2, 128);
  }
  __syncthreads();
  KVR_TRACE_POINT(0, 5);
  const int sel0 = flags[2], sel1 = flags[3];
  const int n_sel = (sel0 >= 0) + (sel1 >= 0);

  // ---- 4. the chosen tiles (transformed domain): warp w takes query head
  // w % g and the tiles w / g, w / g + 8 / g, ...; the first part starts
  // from the head's exact partial
  if (n_sel > 0) {
    if (!mbar_wait_bounded(&bars[1], 0)) {
      if (lane == 0) atomicOr(a.err, 1u);
      flags[1] = 0;
      mbar_wait_bounded(&bars[1], 0);
    }
  }
  __syncthreads();
  DS_TRACE(1, 3, 0);
  const int nsplit = 8 / g;  // g in {1, 2, 4, 8}
  const int hq = warp % g, part = warp / g;
  float m_run = -INFINITY, l_run = 0.0f;
  float oe[4] = {0.f, 0.f, 0.f, 0.f};  // channels 4 lane .. 4 lane + 3 (natural)
  float ot[4] = {0.f, 0.f, 0.f, 0.f};  // channels lane + 32 s (transformed)
  if (part == 0) {
    const float *xp = xpart + hq * (4 + kD);
    m_run = xp[0];
    l_run = xp[1];
    const float4 v = reinterpret_cast<const float4 *>(xp + 4)[lane];
    oe[0] = v.x; oe[1] = v.y; oe[2] = v.z; oe[3] = v.w;
  }
  // work items per head: (tile, token half) when a head has at least two
  // warps per selected tile (halves the bit-serial P.V chain), else tiles
  const int nh = (TPL >= 2 && nsplit >= 2 * n_sel) ? 2 : 1;
  if (flags[1] != 0)
  for (int it = part; it < n_sel * nh; it += nsplit) {
    const int s = it / nh, hf = it - s * nh;
    const int r0 = hf * (TPL / nh), r1 = r0 + TPL / nh;  // token rows (lane + 32 r) of this item
    const unsigned char *tb = tiles + s * kTileBytes;
    const uint32_t *KB = reinterpret_cast<const uint32_t *>(tb);
    const uint32_t *VB = reinterpret_cast<const uint32_t *>(tb + kTileBits);
    const uint16_t *KS = reinterpret_cast<const uint16_t *>(tb + 2 * kTileBits);
    const uint16_t *VS = reinterpret_cast<const uint16_t *>(tb + 2 * kTileBits + kD * 2);
    float *L = lut + warp * 32 * 17;
    float *P = pbuf + warp * TILE;
    {
      const int grp = lane;
      float av[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) av[r] = Qt[hq * kD + 4 * grp + r] * __half2float(__ushort_as_half(KS[4 * grp + r]));
#pragma unroll
      for (int x = 0; x < 16; ++x) {
        float sum = 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) sum += ((x >> r) & 1) ? av[r] : -av[r];
        L[grp * 17 + x] = sum;  // row stride 17: conflict-free stores and lookups
      }
    }
    __syncwarp();
    float sj[TPL];
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < TPL; ++r) {
      sj[r] = -INFINITY;
      if (r < r0 || r >= r1) continue;
      const uint4 w4 = reinterpret_cast<const uint4 *>(KB)[lane + 32 * r];
      const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int grp = 0; grp < 32; ++grp) acc[grp & 3] += L[grp * 17 + ((w[grp >> 3] >> (4 * (grp & 7))) & 15u)];
      sj[r] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
      mx = fmaxf(mx, sj[r]);
    }
    mx = warp_max(mx);
    float l = 0.0f;
#pragma unroll
    for (int r = 0; r < TPL; ++r) {
      if (r < r0 || r >= r1) continue;
      const float p = expf(sj[r] - mx);
      P[lane + 32 * r] = p;
      l += p;
    }
    l = warp_sum(l);
    __syncwarp();
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t lane_bit = 1u << lane;
#pragma unroll 8
    for (int j = 32 * r0; j < 32 * r1; ++j) {
      const float pj = P[j];
      const uint4 v4 = reinterpret_cast<const uint4 *>(VB)[j];
      // channel lane + 32 m of token j set: add p_j (adding 0 otherwise is exact)
      if (v4.x & lane_bit) o[0] += pj;
      if (v4.y & lane_bit) o[1] += pj;
      if (v4.z & lane_bit) o[2] += pj;
      if (v4.w & lane_bit) o[3] += pj;
    }
    // fold (mx, l, o') into the warp state
    const float mn = fmaxf(m_run, mx);
    const float al = m_run == -INFINITY ? 0.0f : expf(m_run - mn);
    const float be = expf(mx - mn);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      oe[m] *= al;
      ot[m] = ot[m] * al + be * (__half2float(__ushort_as_half(VS[lane + 32 * m])) * (2.0f * o[m] - l));
    }
    l_run = l_run * al + l * be;
    m_run = mn;
    __syncwarp();
  }
  DS_TRACE(1, 4, 0);
  KVR_TRACE_POINT(0, 6);
  // ---- 6. fold the warps of each head; store the CTA row into the merging CTA
  {
    float *wp = wpart + warp * kDsPart;
    if (lane == 0) {
      wp[0] = m_run;
      wp[1] = l_run;
    }
    reinterpret_cast<float4 *>(wp + 4)[lane] = make_float4(oe[0], oe[1], oe[2], oe[3]);
#pragma unroll
    for (int m = 0; m < 4; ++m) wp[4 + kD + lane + 32 * m] = ot[m];
  }
  __syncthreads();
  if (warp < g) {
    // warp hq folds warps hq, hq + g, ... and stores into CTA hq's buffer, slot my
    float M = -INFINITY;
    for (int p = 0; p < nsplit; ++p) M = fmaxf(M, wpart[(hq + p * g) * kDsPart]);
    float wts[8], Lsum = 0.0f;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      wts[p] = 0.0f;
      if (p < nsplit) {
        const float mp = wpart[(hq + p * g) * kDsPart];
        wts[p] = mp == -INFINITY ? 0.0f : expf(mp - M);
        Lsum += wts[p] * wpart[(hq + p * g) * kDsPart + 1];
      }
    }
    const uint32_t dst = map_shared(recv + my * kDsPart, (unsigned)hq);
    for (int c4 = lane; c4 < 2 * kD / 4; c4 += 32) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < 8; ++p)
        if (p < nsplit) {
          const float4 v = reinterpret_cast<const float4 *>(wpart + (hq + p * g) * kDsPart + 4)[c4];
          acc.x = fmaf(wts[p], v.x, acc.x); acc.y = fmaf(wts[p], v.y, acc.y);
          acc.z = fmaf(wts[p], v.z, acc.z); acc.w = fmaf(wts[p], v.w, acc.w);
        }
      st_cluster_f4(dst + 16 + c4 * 16, acc);
    }
    if (lane == 0) st_cluster_f4(dst, make_float4(M, Lsum, 0.f, 0.f));
  }
  cluster_sync_all();
  KVR_TRACE_POINT(0, 7);
  if ((int)my >= g) return;

  // ---- merge of query head my over the C rows
  const int mh = (int)my;
  float *wl = wpart;  // [C] weights, then [2][128] sums (the warp rows are dead)
  if (warp == 0) {
    float M = -INFINITY;
    for (int s = lane; s < C; s += 32) M = fmaxf(M, recv[s * kDsPart]);
    M = warp_max(M);
    float Lsum = 0.0f;
    for (int s = lane; s < C; s += 32) {
      const float ms = recv[s * kDsPart];
      const float w = ms == -INFINITY ? 0.0f : expf(ms - M);
      wl[s] = w;
      Lsum += w * recv[s * kDsPart + 1];
    }
    Lsum = warp_sum(Lsum);
    if (lane == 0) {
      wl[C] = M;
      wl[C + 1] = Lsum;
    }
  }
  __syncthreads();
  DS_TRACE(1, 5, 0);
  {
    float acc = 0.0f;
#pragma unroll 4
    for (int s = 0; s < C; ++s) acc = fmaf(wl[s], recv[s * kDsPart + 4 + tid], acc);
    wl[64 + tid] = acc;  // [0, 128) exact, [128, 256) transformed
  }
  __syncthreads();
  DS_TRACE(1, 6, 0);
  if (warp != 0) return;
  const float M = wl[C], Lsum = wl[C + 1];
  const float *Ex = wl + 64, *Tr = wl + 64 + kD;
  const int64_t qh = b * a.n_q + (int64_t)h * g + mh;
  float y[4];
  int ch[4];
  if (a.kind == KVR_DCT) {
#pragma unroll
    for (int s = 0; s < 4; ++s) y[s] = Tr[lane + 32 * s];
    dct128_inv_shfl(y, lane, lee);
#pragma unroll
    for (int s = 0; s < 4; ++s) ch[s] = lane + 32 * s;
  } else {
#pragma unroll
    for (int r = 0; r < 4; ++r) y[r] = Tr[lane * 4 + r];
    wht128(y, lane);
#pragma unroll
    for (int r = 0; r < 4; ++r) ch[r] = lane * 4 + r;
  }
  if (a.partial_out) {
    float *pr = a.partial_out + qh * (kD + 2);
    if (lane == 0) {
      pr[0] = M;
      pr[1] = Lsum;
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) pr[2 + ch[s]] = Ex[ch[s]] + y[s];
  } else {
    const float inv = Lsum > 0.0f ? 1.0f / Lsum : 0.0f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int64_t idx = qh * kD + ch[s];
      const float v = (Ex[ch[s]] + y[s]) * inv;
      if (a.out_dt == KVR_F32) store_elem<KVR_F32>(a.out, idx, v);
      else if (a.out_dt == KVR_F16) store_elem<KVR_F16>(a.out, idx, v);
      else store_elem<KVR_BF16>(a.out, idx, v);
    }
  }
  DS_TRACE(1, 7, 0);
}

// ------------------------------------------------------------------ host ----
namespace {

int ds_plan(DsArgs &a, int C) {
  const int tile_bits = a.tile * 16;
  a.tpc = (int)((a.n_tiles + C - 1) / C);
  const int per_tile = tile_bits + kD * 2;
  // 16-CTA clusters: two CTAs per SM (this layer's and the next one's);
  // 8-CTA clusters use half the SMs per layer and may fill an SM alone
  a.staged = min(a.tpc, (C == 8 ? 2 : 1) * kDsStageMaxBytes / per_tile);
  a.epc = (int)((a.n_win + a.n_tail + C - 1) / C);
  if (a.tpc > kDsMaxTpc || a.epc > kDsMaxExact) return -1;
  size_t o = 576 + 512 + 2 * kDsMaxG * kD * 4;
  a.o_lists = (int)o;
  o += (size_t)C * kDsList * 8;
  a.o_sc = (int)o;
  o = align_up(o + (size_t)max(a.tpc, 1) * 4, 128);
  const size_t stage = (size_t)a.staged * per_tile;
  const size_t recv = (size_t)C * kDsPart * 4;
  // P rows per warp; before the tiles arrive they hold the C/2 level-1 lists
  const size_t lutp = (size_t)8 * 32 * 17 * 4 + std::max((size_t)8 * a.tile * 4, (size_t)(C / 2) * kDsList * 8);
  a.o_region = (int)o;
  // the receive buffer aliases the scan staging (written only after the
  // first cluster barrier, when every CTA's scan is done); LUT + P follow it
  a.o_lut = (int)(o + recv);
  a.o_p = a.o_lut + 8 * 32 * 17 * 4;
  o += std::max(stage, recv + lutp);
  o = align_up(o, 128);
  a.o_ex = (int)o;
  o += (size_t)2 * max(a.epc, 1) * kDsExStride;
  o = align_up(o, 128);
  a.o_tiles = (int)o;
  o += (size_t)2 * (2 * tile_bits + 2 * kD * 2);
  a.o_wpart = (int)o;
  o += (size_t)8 * kDsPart * 4 + (size_t)kDsMaxG * (4 + kD) * 4;
  a.smem = (int)align_up(o, 128);
  return a.smem <= 227 * 1024 ? 0 : -1;
}

template <int TILE, int C>
int ds_launch(DsArgs &a, int batch, cudaStream_t st, bool pdl, bool query_only, bool *fits) {
  auto *fn = sd1_dsmem_step_kernel<TILE, C>;
  static std::mutex mu;
  static int attr_dev[64] = {};  // bit 0: attributes set on this device
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && !attr_dev[dev]) {
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (C > 8) cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      attr_dev[dev] = 1;
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(C, a.n_kv, batch);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = a.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  if (query_only) {
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, fn, &cfg);
    if (e != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    *fits = n >= 1;
    return KVR_OK;
  }
  if (cudaLaunchKernelEx(&cfg, fn, a) != cudaSuccess) return check_launch("kvr_sd1_decode_step (cluster)");
  return check_launch("kvr_sd1_decode_step (cluster)");
}

template <int C>
int ds_dispatch(DsArgs &a, int batch, cudaStream_t st, bool pdl, bool query_only, bool *fits) {
  switch (a.tile) {
    case 32: return ds_launch<32, C>(a, batch, st, pdl, query_only, fits);
    case 64: return ds_launch<64, C>(a, batch, st, pdl, query_only, fits);
    default: return ds_launch<128, C>(a, batch, st, pdl, query_only, fits);
  }
}

// Cluster size usable on this device for this plan (cached per device,
// tile and C): 16 where a 16-CTA cluster can be placed, else 8, else 0.
int ds_pick_cluster(DsArgs &a, int batch, cudaStream_t st, int force_c) {
  static std::mutex mu;
  static int cache[64][3][2];  // [dev][tile][C16?]: 0 unknown, 1 yes, 2 no
  int dev = 0;
  cudaGetDevice(&dev);
  const int ti = a.tile == 32 ? 0 : a.tile == 64 ? 1 : 2;
  for (int C : {16, 8}) {
    if (force_c && C != force_c) continue;
    DsArgs t = a;
    if (ds_plan(t, C) != 0) continue;
    if (a.k_sel > 2 * C) continue;
    int known = 0;
    {
      std::lock_guard<std::mutex> lk(mu);
      if (dev >= 0 && dev < 64) known = cache[dev][ti][C == 16];
    }
    if (known == 0) {
      bool fits = false;
      // the smem plan differs per shape; query at the largest plan this
      // path accepts so that the cached answer covers every shape
      DsArgs big = t;
      big.smem = 227 * 1024;
      if (C == 16) ds_dispatch<16>(big, batch, st, false, true, &fits);
      else ds_dispatch<8>(big, batch, st, false, true, &fits);
      known = fits ? 1 : 2;
      std::lock_guard<std::mutex> lk(mu);
      if (dev >= 0 && dev < 64) cache[dev][ti][C == 16] = known;
    }
    if (known == 1) {
      a = t;
      return C;
    }
  }
  return 0;
}

}  // namespace

// Used by kvr_sd1_decode_step: returns KVR_ENOTSUP (without launching) when
// the shape is outside this path's limits.  force_c = 8 or 16 restricts the
// cluster size (tests of the 8-CTA fallback), 0 picks it.
int sd1_dsmem_step(const void *q, int q_dtype, int batch, int n_q, int n_kv, const uint16_t *win_k,
                   const uint16_t *win_v, int64_t win_cap, int64_t n_win, const uint16_t *tail_k,
                   const uint16_t *tail_v, int64_t n_tail, const uint32_t *kbits, const uint16_t *kscale,
                   const uint32_t *vbits, const uint16_t *vscale, int64_t nt_cap, int64_t n_tiles, int tile,
                   int kind, int k_sel, int64_t ex_t0, int64_t ex_t1, float scale, void *out, int out_dtype,
                   float *partial_out, int32_t *sel_out, unsigned *err, cudaStream_t st, bool pdl,
                   int force_c, const Sd1StepUpdate *upd) {
  const int g = n_kv > 0 ? n_q / n_kv : 0;
  if (!(g == 1 || g == 2 || g == 4 || g == 8) || n_q != g * n_kv) return KVR_ENOTSUP;
  if (k_sel < 0 || k_sel > kDsList) return KVR_ENOTSUP;
  if (n_tiles + n_win + n_tail <= 0) return KVR_ENOTSUP;
  if (n_tiles > 0 && (kbits == nullptr || kscale == nullptr || vbits == nullptr || vscale == nullptr))
    return KVR_ENOTSUP;
  const uintptr_t al = reinterpret_cast<uintptr_t>(win_k) | reinterpret_cast<uintptr_t>(win_v) |
                       reinterpret_cast<uintptr_t>(tail_k) | reinterpret_cast<uintptr_t>(tail_v) |
                       reinterpret_cast<uintptr_t>(kbits) | reinterpret_cast<uintptr_t>(kscale) |
                       reinterpret_cast<uintptr_t>(vbits) | reinterpret_cast<uintptr_t>(vscale);
  if (al % 16 != 0) return KVR_ENOTSUP;
  DsArgs a{};
  a.q = q; a.q_dt = q_dtype; a.n_q = n_q; a.n_kv = n_kv; a.g = g;
  a.inv_scale = (float)(1.0 / (scale > 0.f ? (double)scale : sqrt((double)kD)));
  a.win_k = win_k; a.win_v = win_v; a.win_cap = win_cap; a.n_win = n_win;
  a.tail_k = tail_k; a.tail_v = tail_v; a.n_tail = n_tail;
  a.kbits = kbits; a.kscale = kscale; a.vbits = vbits; a.vscale = vscale;
  a.nt_cap = nt_cap; a.n_tiles = n_tiles; a.tile = tile; a.kind = kind; a.k_sel = k_sel;
  a.ex0 = ex_t0; a.ex1 = ex_t1;
  a.out = out; a.out_dt = out_dtype; a.partial_out = partial_out; a.sel_out = sel_out; a.err = err;
  if (upd != nullptr) {
    if (batch != 1) return KVR_ENOTSUP;
    a.upd = 1;
    a.k_new = upd->k_new; a.v_new = upd->v_new; a.cos_row = upd->cos_row; a.sin_row = upd->sin_row;
    a.q_out = upd->q_out; a.slot = upd->slot; a.evict_row = upd->evict_row;
  } else {
    a.slot = a.evict_row = -1;
  }
  const int C = ds_pick_cluster(a, batch, st, force_c);
  if (C == 16) return ds_dispatch<16>(a, batch, st, pdl, false, nullptr);
  if (C == 8) return ds_dispatch<8>(a, batch, st, pdl, false, nullptr);
  return KVR_ENOTSUP;
}

}  // namespace kvr

#ifdef KVR_TRACE
extern "C" KVR_API int kvr_debug_trace_dsmem(unsigned long long *host, int n) {
  return cudaMemcpyFromSymbol(host, kvr::g_kvr_trace, sizeof(unsigned long long) * n) == cudaSuccess ? 0 : 2;
}
#endif
