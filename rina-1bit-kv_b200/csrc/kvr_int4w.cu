// int4w codec kernels (the reference-faithful path), window ring write and
// the per-row top-k entry point (sm_100a).
//
// Reference: modules/kvr_retrieval.py (int4 K + W-predicted V + int2 residual),
// modules/kvr_window.py (fp16 ring), modules/kvr_cuda.cu (native score kernel).
// Quantisers use correctly rounded division (__fdiv_rn) and round-half-even
// (rintf) exactly like torch.round(x / step), so the packed codes are
// bit-identical to the reference's.
#include "kvr_common.cuh"
#include "kvr_topk.cuh"

namespace kvr {

static int blocks_for(int64_t n, int per) {
  int64_t g = (n + per - 1) / per;
  if (g > 148 * 32) g = 148 * 32;
  return (int)(g < 1 ? 1 : g);
}

// ------------------------------------------------------------- absmax ----
template <int DT>
__global__ void absmax_kernel(const void *__restrict__ x, int64_t n, int64_t cols, int64_t rows_per,
                              unsigned *__restrict__ out_bits) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per, r1 = min(n, r0 + rows_per);
  float m = 0.0f;
  for (int64_t r = r0; r < r1; ++r) m = fmaxf(m, fabsf(load_elem<DT>(x, r * cols + c)));
  atomicMax(out_bits + c, __float_as_uint(m));  // non-negative floats order like their bits
}
__global__ void clamp_min_kernel(float *out, int64_t cols, float lo) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c < cols) out[c] = fmaxf(out[c], lo);
}

// ----------------------------------------------------------- encode K ----
// One thread per 8 consecutive elements of one (token, head) row -> 4 bytes.
template <int DT>
__global__ void encode_k_kernel(const void *__restrict__ k, int64_t n, int n_kv, int d, int64_t tok_stride,
                                const float *__restrict__ scales, uint8_t *__restrict__ out) {
  const int groups = d / 8;
  const int64_t total = n * n_kv * groups;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int gi = (int)(i % groups);
    const int64_t th = i / groups;
    const int h = (int)(th % n_kv);
    const int64_t t = th / n_kv;
    const int64_t src = t * tok_stride + (int64_t)h * d + gi * 8;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      int code[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int c = gi * 8 + e + q;
        const float step = __fdiv_rn(__fmul_rn(2.0f, __ldg(scales + h * d + c)), 16.0f);
        float r = rintf(__fdiv_rn(load_elem<DT>(k, src + e + q), step));
        r = fminf(fmaxf(r, -8.0f), 7.0f);
        code[q] = (int)r + 8;
      }
      word |= (uint32_t)((code[0] << 4) | code[1]) << (8 * (e / 2));
    }
    *reinterpret_cast<uint32_t *>(out + th * (d / 2) + gi * 4) = word;
  }
}

// -------------------------------------------------------- encode V res ----
// One thread per 16 elements -> 4 bytes.
template <int DT>
__global__ void encode_vres_kernel(const void *__restrict__ v, const float *__restrict__ vpred, int64_t n, int n_kv,
                                   int d, const float *__restrict__ vr, uint8_t *__restrict__ out) {
  const int groups = d / 16;
  const int64_t total = n * n_kv * groups;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int gi = (int)(i % groups);
    const int64_t th = i / groups;
    const int h = (int)(th % n_kv);
    const int64_t base = th * d + gi * 16;
    const float step = __fdiv_rn(__fmul_rn(2.0f, __ldg(vr + h)), 4.0f);
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      uint32_t byte = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float res = __fsub_rn(load_elem<DT>(v, base + e + q), __ldg(vpred + base + e + q));
        float r = rintf(__fdiv_rn(res, step));
        r = fminf(fmaxf(r, -2.0f), 1.0f);
        byte |= (uint32_t)((int)r + 2) << (6 - 2 * q);
      }
      word |= byte << (8 * (e / 4));
    }
    *reinterpret_cast<uint32_t *>(out + th * (d / 4) + gi * 4) = word;
  }
}

// ---------------------------------------- drop-in interleaved scores ----
// Drop-in for the reference's native score op (modules/kvr_cuda.cu:9-77):
// score[t, h] = sum_i q[h,2i]*k0r + q[h,2i+1]*k1r, / sqrt(d), where the int4
// pair (hi, lo) of byte i is dequantised as code*s/8 and rotated by the
// interleaved-pair tables cos/sin (n, d/2).
//
// Layout of the work: a warp owns 32 consecutive (token, head) pairs, which
// are 32 consecutive packed rows of d/2 bytes in memory.  The warp first
// copies those rows into its shared-memory slot with coalesced 16-byte loads
// (each load instruction covers 512 contiguous bytes), rows padded by 16 B so
// that the per-lane 16-byte reads that follow hit distinct banks; then each
// lane walks its own row 16 bytes at a time with float4 loads of q, the
// scales and the cos/sin rows (lanes of the same token share those rows, so
// the loads broadcast from L1).  The element order and every rounding step
// follow the reference expression — (code*s)/8, fmaf(ke, c, -(ko*s)),
// fmaf(ke, s, ko*c), score = fmaf(q_even, k0, fmaf(q_odd, k1, score)) in
// increasing i, then an IEEE division by sqrt(d) — so the scores are
// bit-identical to the reference kernel's.
template <int D>
__global__ void __launch_bounds__(256) compute_scores_kernel(const float *__restrict__ q,
                                                             const uint8_t *__restrict__ kp,
                                                             const float *__restrict__ sc,
                                                             const float *__restrict__ cs,
                                                             const float *__restrict__ sn, int n_kv,
                                                             int64_t n_stored, float *__restrict__ scores) {
  constexpr int kRow = D / 2;            // packed bytes per (token, head)
  constexpr int kChunks = kRow / 16;     // 16-byte pieces per row
  constexpr int kPitch = kRow + 16;      // padded smem row
  __shared__ __align__(16) uint8_t stage[8][32 * kPitch];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *my = stage[warp];
  const int64_t total = n_stored * n_kv;
  const float inv_div = __fsqrt_rn((float)D);
  for (int64_t base = ((int64_t)blockIdx.x * 8 + warp) * 32; base < total; base += (int64_t)gridDim.x * 8 * 32) {
    const int rows = (int)(total - base < 32 ? total - base : 32);
    const uint4 *src = reinterpret_cast<const uint4 *>(kp + base * kRow);
    for (int c = lane; c < rows * kChunks; c += 32) {
      const int r = c / kChunks, o = c - r * kChunks;
      *reinterpret_cast<uint4 *>(my + r * kPitch + o * 16) = __ldg(src + c);
    }
    __syncwarp();
    if (lane < rows) {
      const int64_t pair = base + lane;
      const int64_t t = pair / n_kv;
      const int h = (int)(pair - t * n_kv);
      const float4 *qh = reinterpret_cast<const float4 *>(q + (int64_t)h * D);
      const float4 *sh = reinterpret_cast<const float4 *>(sc + (int64_t)h * D);
      const float4 *ct = reinterpret_cast<const float4 *>(cs + t * kRow);
      const float4 *st = reinterpret_cast<const float4 *>(sn + t * kRow);
      float score = 0.0f;
#pragma unroll 1
      for (int c = 0; c < kChunks; ++c) {
        const uint4 w4 = *reinterpret_cast<const uint4 *>(my + lane * kPitch + c * 16);
        const uint32_t words[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int wq = 0; wq < 4; ++wq) {
          // bytes i = 16c + 4wq .. +3: elements 2i, 2i+1 -> q/scale float4 pairs, cos/sin one float4
          const int i0 = 16 * c + 4 * wq;
          const float4 cv4 = __ldg(ct + i0 / 4), sv4 = __ldg(st + i0 / 4);
          const float cvs[4] = {cv4.x, cv4.y, cv4.z, cv4.w}, svs[4] = {sv4.x, sv4.y, sv4.z, sv4.w};
#pragma unroll
          for (int b = 0; b < 4; b += 2) {
            const float4 qv = __ldg(qh + (i0 + b) / 2), sv = __ldg(sh + (i0 + b) / 2);
            const float qe[2] = {qv.x, qv.z}, qo[2] = {qv.y, qv.w};
            const float se[2] = {sv.x, sv.z}, so[2] = {sv.y, sv.w};
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint32_t byte = (words[wq] >> (8 * (b + u))) & 0xffu;
              const float hi = (float)((int)(byte >> 4) - 8), lo = (float)((int)(byte & 15u) - 8);
              const float ke = __fdiv_rn(__fmul_rn(hi, se[u]), 8.0f);
              const float ko = __fdiv_rn(__fmul_rn(lo, so[u]), 8.0f);
              const float cv = cvs[b + u], svv = svs[b + u];
              const float k0 = fmaf(ke, cv, -__fmul_rn(ko, svv));
              const float k1 = fmaf(ke, svv, __fmul_rn(ko, cv));
              score = fmaf(qe[u], k0, fmaf(qo[u], k1, score));
            }
          }
        }
      }
      scores[pair] = __fdiv_rn(score, inv_div);
    }
    __syncwarp();
  }
}

// ------------------------------------------------- group-mean queries ----
__device__ __forceinline__ void stage_qavg(const float *__restrict__ q, int n_q, int n_kv, int d, float *qa) {
  const int g = n_q / n_kv;
  for (int i = threadIdx.x; i < n_kv * d; i += blockDim.x) {
    const int h = i / d, c = i - h * d;
    float s = 0.0f;
    for (int j = 0; j < g; ++j) s += q[(int64_t)(h * g + j) * d + c];
    qa[i] = s / (float)g;
  }
}

// --------------------------------------------------- cosine token scores ----
// compute_all_scores (kvr_retrieval.py:265-289).  Persistent CTAs walk tiles
// of 32 tokens.  The tile's packed rows (32 * n_kv * 64 contiguous bytes) and
// its cos/sin rows (half rows when both halves of the table are equal) are
// brought into shared memory by cp.async, two tiles in flight, so the next
// tile streams in while this one is scored.  Warp w scores tokens 4w..4w+3
// of the tile, all (<= 8) heads at once: lane = (head lane/4, group lane%4);
// group g covers channels [16g, 16g+16) and their rotate_half partners
// [64+16g, 64+16g+16), so a lane rotates its own pairs with no shuffles.
// The dequantisation steps and the group-mean queries sit in a padded
// shared layout (the 8 lanes of a quarter-warp hit 8 distinct bank groups).
// Each element's arithmetic is the reference's: k = code*step, k_rot =
// k*cos + rotate_half(k)*sin (three roundings), then dot and norm.
constexpr int kTsTile = 32;
// Bins of the cosine scores over [-1, 1] for the fused top-k: a monotone map,
// so every score of a higher bin beats every score of a lower one.
constexpr int kCosBins = 4096;
__device__ __forceinline__ int cos_bin(float s) {
  const int b = (int)floorf((s + 1.0f) * (0.5f * kCosBins));
  return b < 0 ? 0 : (b >= kCosBins ? kCosBins - 1 : b);
}
__device__ __forceinline__ int ts_idx(int h, int c) { return h * 176 + c + (c >> 4) * 4; }
__global__ void __launch_bounds__(256) token_scores_kernel(
    const float *__restrict__ q, int n_q, const uint8_t *__restrict__ kp, const float *__restrict__ sc,
    const float *__restrict__ cs, const float *__restrict__ sn, int64_t rope_stride, int halves_equal, int n_kv,
    int64_t n_stored, float *__restrict__ scores, int64_t score_stride, int *__restrict__ hist, int64_t ex0,
    int64_t ex1) {
  constexpr int d = 128;
  __shared__ __align__(16) float qa[8 * 176];  // n_kv <= 8
  __shared__ __align__(16) float stp[8 * 176];
  __shared__ float qn_s[8];
  __shared__ float outb[8][kTsTile];           // [head][token]
  extern __shared__ __align__(16) unsigned char dsm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row_bytes = n_kv * (d / 2);
  const int cw = halves_equal ? 64 : 128;          // table floats kept per token
  const int k_bytes = kTsTile * row_bytes;
  const int t_bytes = kTsTile * cw * 4;
  const int stage_bytes = k_bytes + 2 * t_bytes;
  const int64_t tiles = (n_stored + kTsTile - 1) / kTsTile;

  auto issue = [&](int64_t tile, int stage) {
    unsigned char *base = dsm + stage * stage_bytes;
    const int64_t t0 = tile * kTsTile;
    const int nt = (int)(n_stored - t0 < kTsTile ? n_stored - t0 : kTsTile);
    const unsigned char *ksrc = kp + t0 * row_bytes;
    for (int p = tid; p < nt * row_bytes / 16; p += blockDim.x) cp_async16(base + p * 16, ksrc + p * 16);
    const int per = cw / 4;  // 16-byte pieces per table row
    for (int p = tid; p < nt * per; p += blockDim.x) {
      const int j = p / per, o = p - j * per;
      cp_async16(base + k_bytes + (j * cw + o * 4) * 4, cs + (t0 + j) * rope_stride + o * 4);
      cp_async16(base + k_bytes + t_bytes + (j * cw + o * 4) * 4, sn + (t0 + j) * rope_stride + o * 4);
    }
    cp_async_commit();
  };
  int64_t tile = blockIdx.x;
  if (tile < tiles) issue(tile, 0);
  const int g = n_q / n_kv;
  for (int i = tid; i < n_kv * d; i += blockDim.x) {
    const int h = i / d, c = i - h * d;
    float s = 0.0f;
    for (int j = 0; j < g; ++j) s += __ldg(q + (int64_t)(h * g + j) * d + c);
    qa[ts_idx(h, c)] = s / (float)g;
    stp[ts_idx(h, c)] = __fdiv_rn(__fmul_rn(2.0f, __ldg(sc + i)), 16.0f);
  }
  __syncthreads();
  if (warp < n_kv) {
    float s = 0.0f;
    for (int c = lane; c < d; c += 32) s = fmaf(qa[ts_idx(warp, c)], qa[ts_idx(warp, c)], s);
    s = warp_sum(s);
    if (lane == 0) qn_s[warp] = sqrtf(s) + 1e-8f;
  }
  const int h = lane >> 2, gq = lane & 3;
  const bool hv = h < n_kv;
  const int hh = hv ? h : 0;
  const int c_lo = gq * 16, c_hi = 64 + gq * 16;
  const int tc_hi = halves_equal ? c_lo : c_hi;
  const float4 *qlo = reinterpret_cast<const float4 *>(qa + ts_idx(hh, c_lo));
  const float4 *qhi = reinterpret_cast<const float4 *>(qa + ts_idx(hh, c_hi));
  const float4 *slo = reinterpret_cast<const float4 *>(stp + ts_idx(hh, c_lo));
  const float4 *shi = reinterpret_cast<const float4 *>(stp + ts_idx(hh, c_hi));
  for (int it = 0; tile < tiles; ++it, tile += gridDim.x) {
    const int st = it & 1;
    if (tile + gridDim.x < tiles) {
      issue(tile + gridDim.x, st ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const unsigned char *base = dsm + st * stage_bytes;
    const float *cst = reinterpret_cast<const float *>(base + k_bytes);
    const float *snt = reinterpret_cast<const float *>(base + k_bytes + t_bytes);
    const int64_t t0 = tile * kTsTile;
#pragma unroll 1
    for (int jj = 0; jj < kTsTile / 8; ++jj) {
      const int j = warp * (kTsTile / 8) + jj;
      const uint8_t *row = base + j * row_bytes + hh * (d / 2);
      const uint2 rlo = *reinterpret_cast<const uint2 *>(row + c_lo / 2);
      const uint2 rhi = *reinterpret_cast<const uint2 *>(row + c_hi / 2);
      const float4 *crl = reinterpret_cast<const float4 *>(cst + j * cw + c_lo);
      const float4 *srl = reinterpret_cast<const float4 *>(snt + j * cw + c_lo);
      const float4 *crh = reinterpret_cast<const float4 *>(cst + j * cw + tc_hi);
      const float4 *srh = reinterpret_cast<const float4 *>(snt + j * cw + tc_hi);
      float dot = 0.0f, nk = 0.0f;
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {  // channels c_lo + 4*g4 .. +3 and their partners c_hi + 4*g4 ..
        const float4 cl = crl[g4], sl = srl[g4], ch = crh[g4], sh = srh[g4];
        const float4 ql = qlo[g4], qh = qhi[g4], pl = slo[g4], ph = shi[g4];
        const uint32_t wl = ((g4 < 2 ? rlo.x : rlo.y) >> (16 * (g4 & 1))) & 0xffffu;
        const uint32_t wh = ((g4 < 2 ? rhi.x : rhi.y) >> (16 * (g4 & 1))) & 0xffffu;
        const float al[4] = {__fmul_rn((float)((int)((wl >> 4) & 15u) - 8), pl.x),
                             __fmul_rn((float)((int)(wl & 15u) - 8), pl.y),
                             __fmul_rn((float)((int)((wl >> 12) & 15u) - 8), pl.z),
                             __fmul_rn((float)((int)((wl >> 8) & 15u) - 8), pl.w)};
        const float ah[4] = {__fmul_rn((float)((int)((wh >> 4) & 15u) - 8), ph.x),
                             __fmul_rn((float)((int)(wh & 15u) - 8), ph.y),
                             __fmul_rn((float)((int)((wh >> 12) & 15u) - 8), ph.z),
                             __fmul_rn((float)((int)((wh >> 8) & 15u) - 8), ph.w)};
        const float cvl[4] = {cl.x, cl.y, cl.z, cl.w}, svl[4] = {sl.x, sl.y, sl.z, sl.w};
        const float cvh[4] = {ch.x, ch.y, ch.z, ch.w}, svh[4] = {sh.x, sh.y, sh.z, sh.w};
        const float qvl[4] = {ql.x, ql.y, ql.z, ql.w}, qvh[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // rotate_half: channel c < 64 pairs with -k[c+64], channel c+64 with +k[c]
          const float kl = __fadd_rn(__fmul_rn(al[e], cvl[e]), __fmul_rn(-ah[e], svl[e]));
          const float kh = __fadd_rn(__fmul_rn(ah[e], cvh[e]), __fmul_rn(al[e], svh[e]));
          dot = fmaf(qvl[e], kl, dot);
          nk = fmaf(kl, kl, nk);
          dot = fmaf(qvh[e], kh, dot);
          nk = fmaf(kh, kh, nk);
        }
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      nk += __shfl_xor_sync(0xffffffffu, nk, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      nk += __shfl_xor_sync(0xffffffffu, nk, 2);
      if (gq == 0 && hv) {
        float s = dot / (qn_s[hh] * (sqrtf(nk) + 1e-8f));
        if (s != s) s = -INFINITY;
        outb[hh][j] = s;
      }
    }
    __syncthreads();
    for (int e = tid; e < n_kv * kTsTile; e += blockDim.x) {
      const int h2 = e / kTsTile, j = e - h2 * kTsTile;
      if (t0 + j < n_stored) {
        const float sv = outb[h2][j];
        scores[(int64_t)h2 * score_stride + t0 + j] = sv;
        const int64_t t = t0 + j;
        if (hist != nullptr && !(t >= ex0 && t < ex1) && sv > -INFINITY)
          atomicAdd(hist + h2 * kCosBins + cos_bin(sv), 1);
      }
    }
  }
}

// --------------------------------------------------- cosine chunk scores ----
// One warp per (chunk, head); lane owns dims 4l..4l+3 (rotate_half partner in lane ^ 16).
__global__ void __launch_bounds__(256) chunk_scores_kernel(
    const float *__restrict__ q, int n_q, const uint8_t *__restrict__ kp, const float *__restrict__ sc,
    const float *__restrict__ cs, const float *__restrict__ sn, int64_t rope_stride, int halves_equal, int n_kv,
    int64_t n_chunks, int chunk, float *__restrict__ scores, int64_t score_stride) {
  constexpr int d = 128;
  __shared__ float qa[8 * d];
  stage_qavg(q, n_q, n_kv, d, qa);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t wi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < n_chunks * n_kv; wi += warps) {
    const int h = (int)(wi % n_kv);
    const int64_t ci = wi / n_kv;
    float step[4], acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 4; ++r) step[r] = __fdiv_rn(__fmul_rn(2.0f, __ldg(sc + h * d + lane * 4 + r)), 16.0f);
    const int coff = halves_equal ? ((lane * 4) & 63) : lane * 4;
    for (int j = 0; j < chunk; ++j) {
      const int64_t t = ci * chunk + j;
      const uint16_t two = __ldg(reinterpret_cast<const uint16_t *>(kp + (t * n_kv + h) * (d / 2) + lane * 2));
      float kx[4];
      kx[0] = (float)((int)((two >> 4) & 15) - 8) * step[0];
      kx[1] = (float)((int)(two & 15) - 8) * step[1];
      kx[2] = (float)((int)((two >> 12) & 15) - 8) * step[2];
      kx[3] = (float)((int)((two >> 8) & 15) - 8) * step[3];
      const float4 c4 = __ldg(reinterpret_cast<const float4 *>(cs + t * rope_stride + coff));
      const float4 s4 = __ldg(reinterpret_cast<const float4 *>(sn + t * rope_stride + coff));
      const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float partner = __shfl_xor_sync(0xffffffffu, kx[r], 16);
        const float rh = lane < 16 ? -partner : partner;
        acc[r] += __fadd_rn(__fmul_rn(kx[r], cv[r]), __fmul_rn(rh, sv[r]));
      }
    }
    float dot = 0.f, nk = 0.f, nq = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float m = acc[r] / (float)chunk;
      const float qv = qa[h * d + lane * 4 + r];
      dot = fmaf(qv, m, dot);
      nk = fmaf(m, m, nk);
      nq = fmaf(qv, qv, nq);
    }
    dot = warp_sum(dot);
    nk = warp_sum(nk);
    nq = warp_sum(nq);
    if (lane == 0) {
      float s = dot / ((sqrtf(nq) + 1e-8f) * (sqrtf(nk) + 1e-8f));
      if (s != s) s = -INFINITY;
      scores[(int64_t)h * score_stride + ci] = s;
    }
  }
}

// ----------------------------------------------------------------- top-k ----
constexpr int kTopkThreads = 1024;
// One CTA per row.  STAGE: the row is first copied into shared memory (one
// coalesced pass, exclusions and NaN mapped to -inf there), so the radix
// passes of block_topk re-read it on chip instead of from L2.
template <bool STAGE>
__global__ void __launch_bounds__(kTopkThreads) topk_rows_kernel(const float *__restrict__ scores, int64_t n,
                                                                 int64_t row_stride, int k, int64_t ex0,
                                                                 int64_t ex1, int64_t *__restrict__ idx,
                                                                 float *__restrict__ vals, int64_t ors,
                                                                 int64_t oes) {
  extern __shared__ __align__(16) unsigned char dyn[];
  TopkSmem &tsm = *reinterpret_cast<TopkSmem *>(dyn);
  unsigned long long *cand = reinterpret_cast<unsigned long long *>(dyn + align_up(sizeof(TopkSmem), 16));
  const float *row = scores + (int64_t)blockIdx.x * row_stride;
  if constexpr (STAGE) {
    int P = 1;
    while (P < k) P <<= 1;
    float *srow = reinterpret_cast<float *>(dyn + align_up(sizeof(TopkSmem), 16) + (size_t)P * 8);
    for (int64_t i = threadIdx.x; i < n; i += kTopkThreads) {
      const float v = __ldcs(row + i);
      srow[i] = (i >= ex0 && i < ex1) ? -INFINITY : v;
    }
    __syncthreads();
    block_topk<kTopkThreads>([&](int64_t i) -> float { return srow[i]; }, n, k, cand, tsm);
  } else {
    block_topk<kTopkThreads>(
        [&](int64_t i) -> float { return (i >= ex0 && i < ex1) ? -INFINITY : __ldg(row + i); }, n, k, cand, tsm);
  }
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int64_t o = (int64_t)blockIdx.x * ors + (int64_t)j * oes;
    idx[o] = key_index(cand[j]);
    if (vals) vals[o] = key_score(cand[j]);
  }
}

// Long rows (n in the tens of thousands, k up to ~1/8 of n): the row is staged
// in shared memory, then a 4096-bin histogram over the linear map of the
// finite scores' [min, max] range (a monotone map, so every key of a higher
// bin beats every key of a lower one) locates the bin holding the k-th
// largest score.  Keys of higher bins are taken outright; only that bin's
// keys go through the exact radix selection, then the k keys are sorted
// (score desc, index asc).  When the threshold bin is too crowded for the
// candidate buffer, or fewer than k scores are finite, the CTA falls back to
// the whole-row radix select.
constexpr int kHistBins = 4096;
constexpr int kHistCand = 4096;
struct HistSmem {
  int hist[kHistBins];
  float mn[32], mx[32];
  int thr_bin, above, n_cand, n_take, n_finite;
  float lo, scale;
};
__global__ void __launch_bounds__(kTopkThreads) topk_rows_hist_kernel(const float *__restrict__ scores, int64_t n,
                                                                      int64_t row_stride, int k, int64_t ex0,
                                                                      int64_t ex1, int64_t *__restrict__ idx,
                                                                      float *__restrict__ vals, int64_t ors,
                                                                      int64_t oes) {
  extern __shared__ __align__(16) unsigned char dyn[];
  TopkSmem &tsm = *reinterpret_cast<TopkSmem *>(dyn);
  size_t off = align_up(sizeof(TopkSmem), 16);
  HistSmem &hs = *reinterpret_cast<HistSmem *>(dyn + off);
  off += align_up(sizeof(HistSmem), 16);
  int P = 1;
  while (P < k) P <<= 1;
  unsigned long long *cand = reinterpret_cast<unsigned long long *>(dyn + off);   // P keys: the answer
  off += (size_t)P * 8;
  unsigned long long *cand2 = reinterpret_cast<unsigned long long *>(dyn + off);  // threshold-bin keys
  off += (size_t)kHistCand * 8;
  unsigned long long *cand3 = reinterpret_cast<unsigned long long *>(dyn + off);  // P keys: their top
  off += (size_t)P * 8;
  float *srow = reinterpret_cast<float *>(dyn + off);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float *row = scores + (int64_t)blockIdx.x * row_stride;
  float mn = INFINITY, mx = -INFINITY;
  int nf = 0;
  for (int64_t r0 = 0; r0 < n; r0 += 8 * kTopkThreads) {  // 8 loads in flight per thread
    float vv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t i = r0 + u * kTopkThreads + tid;
      vv[u] = i < n ? __ldcs(row + i) : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t i = r0 + u * kTopkThreads + tid;
      if (i >= n) continue;
      float v = vv[u];
      if ((i >= ex0 && i < ex1) || v != v) v = -INFINITY;
      srow[i] = v;
      if (v > -INFINITY && v < INFINITY) {
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
        ++nf;
      }
    }
  }
  for (int b = tid; b < kHistBins; b += kTopkThreads) hs.hist[b] = 0;
  mn = -warp_max(-mn);
  mx = warp_max(mx);
  nf = warp_sum_int(nf);
  if (lane == 0) {
    hs.mn[warp] = mn;
    hs.mx[warp] = mx;
  }
  if (tid == 0) {
    hs.n_finite = 0;
    hs.above = 0;
    hs.n_cand = 0;
  }
  __syncthreads();
  if (lane == 0) atomicAdd(&hs.n_finite, nf);
  if (tid == 0) {
    float a = INFINITY, b = -INFINITY;
    for (int w = 0; w < kTopkThreads / 32; ++w) {
      a = fminf(a, hs.mn[w]);
      b = fmaxf(b, hs.mx[w]);
    }
    hs.lo = a;
    hs.scale = (b > a) ? (float)(kHistBins - 1) / (b - a) : 0.0f;
  }
  __syncthreads();
  const float lo = hs.lo, scale = hs.scale;
  auto bin_of = [&](float v) -> int {
    int b = (int)((v - lo) * scale);
    return b < 0 ? 0 : (b >= kHistBins ? kHistBins - 1 : b);
  };
  bool fallback = hs.n_finite < k;
  if (!fallback) {
    for (int64_t i = tid; i < n; i += kTopkThreads) {
      const float v = srow[i];
      if (v > -INFINITY && v < INFINITY) atomicAdd(&hs.hist[bin_of(v)], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // suffix counts from the top bin down: lane l owns bins [128*(31-l), 128*(32-l))
      int s = 0;
      const int b_hi = kHistBins - 128 * lane;
      for (int b = b_hi - 1; b >= b_hi - 128; --b) s += hs.hist[b];
      int incl = s;
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int excl = incl - s;
      if (excl < k && k <= incl) {
        int cum = excl;
        for (int b = b_hi - 1; b >= b_hi - 128; --b) {
          if (cum + hs.hist[b] >= k) {
            hs.thr_bin = b;
            hs.above = cum;
            break;
          }
          cum += hs.hist[b];
        }
      }
    }
    __syncthreads();
    fallback = hs.hist[hs.thr_bin] > kHistCand;
  }
  if (fallback) {  // (uniform across the block)
    block_topk<kTopkThreads>([&](int64_t i) -> float { return srow[i]; }, n, k, cand, tsm);
  } else {
    const int thr = hs.thr_bin;
    __shared__ int n_above;
    __shared__ int wcount[kTopkThreads / 32];
    if (tid == 0) n_above = 0;
    __syncthreads();
    // keys of higher bins in any order (they are sorted below); keys of the
    // threshold bin in index order, so that block_topk's position tie-break
    // over cand2 is the index tie-break of the row
    int base_pos = 0;
    for (int64_t r0 = 0; r0 < n; r0 += kTopkThreads) {
      const int64_t i = r0 + tid;
      float v = -INFINITY;
      if (i < n) v = srow[i];
      const bool fin = v > -INFINITY && v < INFINITY;
      const int b = fin ? bin_of(v) : -1;
      if (b > thr) cand[atomicAdd(&n_above, 1)] = make_key(v, i);
      const bool in_thr = (b == thr);
      const unsigned bal = __ballot_sync(0xffffffffu, in_thr);
      if (lane == 0) wcount[warp] = __popc(bal);
      __syncthreads();
      int before = base_pos, total = 0;
      for (int w = 0; w < kTopkThreads / 32; ++w) {
        const int c = wcount[w];
        if (w < warp) before += c;
        total += c;
      }
      if (in_thr) cand2[before + __popc(bal & ((1u << lane) - 1u))] = make_key(v, i);
      base_pos += total;
      __syncthreads();
    }
    if (tid == 0) hs.n_cand = base_pos;
    __syncthreads();
    const int na = n_above, nc = hs.n_cand, need = k - na;
    block_topk<kTopkThreads>([&](int64_t i) -> float { return key_score(cand2[i]); }, nc, need, cand3, tsm);
    // cand3 holds positions in cand2 as its indices: map back to the row keys
    for (int j = tid; j < need; j += kTopkThreads) cand[na + j] = cand2[key_index(cand3[j])];
    for (int j = k + tid; j < P; j += kTopkThreads) cand[j] = 0ull;
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < P / 2; i += kTopkThreads) {
          const int a = 2 * i - (i & (stride - 1));
          const int b = a + stride;
          const bool desc = ((a & size) == 0);
          const unsigned long long x = cand[a], y = cand[b];
          if ((x < y) == desc) {
            cand[a] = y;
            cand[b] = x;
          }
        }
        __syncthreads();
      }
    }
  }
  for (int j = tid; j < k; j += blockDim.x) {
    const int64_t o = (int64_t)blockIdx.x * ors + (int64_t)j * oes;
    idx[o] = key_index(cand[j]);
    if (vals) vals[o] = key_score(cand[j]);
  }
}

// ------------------------------------------- fused token top-k (int4w) ----
// Histogram kernel: CTAs (segment, head) count the kept scores of a head into
// kCosBins bins (shared-memory histograms added into a global one).
// Split kernel: CTAs (segment, head) find the threshold bin (the bin holding
// the k-th largest kept score, from the top) and route their segment's keys:
// higher bins -> the head's "above" list (fewer than k), the threshold bin ->
// its candidate list.  Finalize kernel (one CTA per head): exact top of the
// candidates by key, joined with the above keys and sorted (score desc,
// index asc); it clears the head's histogram and counters for the next call.
// A head with fewer than k kept scores, or a threshold bin with more than
// kTkCand keys, is finished by the whole-row radix select instead.
constexpr int kTkCand = 4096;
constexpr int kTkSegs = 16;
struct TkRow {
  int above, cand, overflow, thr;
};

// The threshold bin of a head (the bin holding its k-th largest kept score,
// counting from the top) by a block scan of the histogram: thread t owns
// kCosBins / NT consecutive bins, thread 0 the highest.  Optionally leaves
// each bin's count (cnt_s) and the number of kept scores in higher bins
// (pos_s) in shared memory.  Returns -1 when fewer than k scores are kept.
template <int NT>
__device__ int tk_threshold_block(const int *__restrict__ hist, int k, int *above_out, int *pos_s = nullptr,
                                  int *cnt_s = nullptr) {
  constexpr int PER = kCosBins / NT;
  __shared__ int thr_s, above_s, wsum[NT / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hi = kCosBins - PER * tid;  // bins [hi - PER, hi), visited downwards
  int v[PER], sum = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    v[j] = __ldcg(hist + hi - 1 - j);
    sum += v[j];
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[warp] = incl;
  if (tid == 0) {
    thr_s = -1;
    above_s = 0;
  }
  __syncthreads();
  int cum = incl - sum;
  for (int w = 0; w < warp; ++w) cum += wsum[w];
  const bool mine = cum < k && k <= cum + sum;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    if (pos_s) {
      pos_s[hi - 1 - j] = cum;
      cnt_s[hi - 1 - j] = v[j];
    }
    if (mine && cum < k && k <= cum + v[j]) {
      thr_s = hi - 1 - j;
      above_s = cum;
    }
    cum += v[j];
  }
  __syncthreads();
  *above_out = above_s;
  return thr_s;
}

// Per-(segment, head) histogram of the kept scores in shared memory, added
// into the head's global histogram bin by bin (only non-empty bins).
__global__ void __launch_bounds__(256) tk_hist_kernel(const float *__restrict__ scores, int64_t n, int64_t ex0,
                                                      int64_t ex1, int *__restrict__ hist) {
  __shared__ int sh[kCosBins];
  const int h = blockIdx.y;
  for (int b = threadIdx.x; b < kCosBins; b += blockDim.x) sh[b] = 0;
  __syncthreads();
  const float *row = scores + (int64_t)h * n;
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * per, i1 = min(n, i0 + per);
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float v = __ldcg(row + i);
    if ((i >= ex0 && i < ex1) || !(v > -INFINITY)) continue;
    atomicAdd(&sh[cos_bin(v)], 1);
  }
  __syncthreads();
  for (int b = threadIdx.x; b < kCosBins; b += blockDim.x)
    if (sh[b]) atomicAdd(hist + (int64_t)h * kCosBins + b, sh[b]);
}

__global__ void __launch_bounds__(256) tk_split_kernel(const float *__restrict__ scores, int64_t n, int k,
                                                       int64_t ex0, int64_t ex1, const int *__restrict__ hist,
                                                       TkRow *__restrict__ rows, unsigned long long *__restrict__ above,
                                                       unsigned long long *__restrict__ cand) {
  const int h = blockIdx.y, lane = threadIdx.x & 31;
  int above_n;
  const int thr = tk_threshold_block<256>(hist + (int64_t)h * kCosBins, k, &above_n);
  if (thr < 0) return;  // finalize falls back to the whole-row select
  const float *row = scores + (int64_t)h * n;
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * per, i1 = min(n, i0 + per);
  TkRow &r = rows[h];
  // one atomic per warp and list: lanes take consecutive slots
  const int64_t i_end = i0 + (i1 - i0 + 31) / 32 * 32;
  for (int64_t i = i0 + threadIdx.x; i < i_end; i += blockDim.x) {
    float v = -INFINITY;
    if (i < i1 && !(i >= ex0 && i < ex1)) v = __ldcg(row + i);
    const bool kept = v > -INFINITY;
    const int b = kept ? cos_bin(v) : -1;
    const unsigned ma = __ballot_sync(0xffffffffu, kept && b > thr);
    const unsigned mc = __ballot_sync(0xffffffffu, kept && b == thr);
    const unsigned below = (1u << lane) - 1u;
    int base_a = 0, base_c = 0;
    if (lane == 0) {
      if (ma) base_a = atomicAdd(&r.above, __popc(ma));
      if (mc) base_c = atomicAdd(&r.cand, __popc(mc));
    }
    base_a = __shfl_sync(0xffffffffu, base_a, 0);
    base_c = __shfl_sync(0xffffffffu, base_c, 0);
    if (ma >> lane & 1u) above[(int64_t)h * k + base_a + __popc(ma & below)] = make_key(v, i);
    if (mc >> lane & 1u) {
      const int slot = base_c + __popc(mc & below);
      if (slot < kTkCand) cand[(int64_t)h * kTkCand + slot] = make_key(v, i);
      else r.overflow = 1;
    }
  }
}

// Shared-memory layout of the finalize kernel for top k (P = k rounded up to
// a power of two).
struct TkFinSmem {
  size_t keys, cand_s, cbuf, pos, cnt, fill, total;
  __host__ __device__ explicit TkFinSmem(int P) {
    keys = align_up(sizeof(TopkSmem), 16);
    cand_s = keys + (size_t)P * 8;
    cbuf = cand_s + (size_t)P * 8;
    pos = cbuf + (size_t)kTkCand * 8;
    cnt = pos + (size_t)kCosBins * 4;
    fill = cnt + (size_t)kCosBins * 4;
    total = fill + (size_t)kCosBins * 4;
  }
};

__global__ void __launch_bounds__(kTopkThreads) tk_finalize_kernel(const float *__restrict__ scores, int64_t n,
                                                                   int k, int64_t ex0, int64_t ex1,
                                                                   int *__restrict__ hist, TkRow *__restrict__ rows,
                                                                   const unsigned long long *__restrict__ above,
                                                                   const unsigned long long *__restrict__ cand,
                                                                   int64_t *__restrict__ idx, int n_kv) {
  extern __shared__ __align__(16) unsigned char dyn[];
  TopkSmem &tsm = *reinterpret_cast<TopkSmem *>(dyn);
  int P = 1;
  while (P < k) P <<= 1;
  const TkFinSmem L(P);
  unsigned long long *keys = reinterpret_cast<unsigned long long *>(dyn + L.keys);
  unsigned long long *cand_s = reinterpret_cast<unsigned long long *>(dyn + L.cand_s);  // the candidates' top
  unsigned long long *cbuf = reinterpret_cast<unsigned long long *>(dyn + L.cbuf);      // candidates staged
  int *pos_s = reinterpret_cast<int *>(dyn + L.pos);    // kept scores in higher bins
  int *cnt_s = reinterpret_cast<int *>(dyn + L.cnt);    // the bin's count
  int *fill_s = reinterpret_cast<int *>(dyn + L.fill);  // keys placed per bin
  const int h = blockIdx.x, tid = threadIdx.x;
  TkRow &r = rows[h];
  int above_n;
  const int thr = tk_threshold_block<kTopkThreads>(hist + (int64_t)h * kCosBins, k, &above_n, pos_s, cnt_s);
  const int na = r.above, nc = r.cand;
  const bool fallback = thr < 0 || r.overflow != 0 || na != above_n;
  if (fallback) {
    const float *row = scores + (int64_t)h * n;
    block_topk<kTopkThreads>([&](int64_t i) -> float { return (i >= ex0 && i < ex1) ? -INFINITY : __ldcg(row + i); },
                             n, k, keys, tsm);
    for (int j = tid; j < k; j += kTopkThreads) idx[(int64_t)j * n_kv + h] = key_index(keys[j]);
  } else {
    // The keys above the threshold bin, counting-sorted by bin (bins are
    // monotone in the score, pos_s gives each bin's first output slot), then
    // ranked inside their bin; the threshold bin's candidates ranked among
    // themselves fill the last k - na slots.  Keys are unique, so the ranks
    // give exactly the order (score desc, index asc).
    for (int b = tid; b < kCosBins; b += kTopkThreads) fill_s[b] = 0;
    for (int i = tid; i < nc; i += kTopkThreads) cbuf[i] = cand[(int64_t)h * kTkCand + i];
    __syncthreads();
    for (int i = tid; i < na; i += kTopkThreads) {
      const unsigned long long key = above[(int64_t)h * k + i];
      const int b = cos_bin(key_float((uint32_t)(key >> 32)));
      keys[pos_s[b] + atomicAdd(&fill_s[b], 1)] = key;
    }
    __syncthreads();
    for (int i = tid; i < na; i += kTopkThreads) {
      const unsigned long long key = keys[i];
      const int b = cos_bin(key_float((uint32_t)(key >> 32)));
      const int g0 = pos_s[b], g1 = g0 + cnt_s[b];
      int rk = 0;
      for (int j = g0; j < g1; ++j) rk += keys[j] > key ? 1 : 0;
      idx[(int64_t)(g0 + rk) * n_kv + h] = key_index(key);
    }
    const int need = k - na;
    const unsigned long long *pool = cbuf;
    int np = nc;
    if (nc > kTopkThreads) {
      // many ties in one bin: exact top `need` of the candidates first
      block_topk_keys<kTopkThreads>([&](int64_t i) -> unsigned long long { return cbuf[i]; }, nc, need, cand_s, tsm);
      pool = cand_s;
      np = need;
    }
    for (int i = tid; i < np; i += kTopkThreads) {
      const unsigned long long key = pool[i];
      int rk = 0;
      for (int j = 0; j < np; ++j) rk += pool[j] > key ? 1 : 0;
      if (rk < need) idx[(int64_t)(na + rk) * n_kv + h] = key_index(key);
    }
  }
  // leave the head's histogram and counters zeroed for the next call
  __syncthreads();
  for (int b = tid; b < kCosBins; b += kTopkThreads) hist[(int64_t)h * kCosBins + b] = 0;
  if (tid == 0) r = TkRow{0, 0, 0, 0};
}

// ---------------------------------------------------------------- gather ----
// One warp per (i, h): ret_k row (RoPE'd head h) and the all-heads x row.
__global__ void __launch_bounds__(256) gather_kernel(const uint8_t *__restrict__ kp, const float *__restrict__ sc,
                                                     const int64_t *__restrict__ top, int k, int n_kv,
                                                     const float *__restrict__ cs, const float *__restrict__ sn,
                                                     int64_t rope_stride, const float *__restrict__ kmean,
                                                     float *__restrict__ ret_k, float *__restrict__ x,
                                                     const int32_t *__restrict__ count) {
  constexpr int d = 128;
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t kv = count ? min((int64_t)k, (int64_t)__ldg(count)) : (int64_t)k;
  for (int64_t wi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < kv * n_kv; wi += warps) {
    const int h = (int)(wi % n_kv);
    const int64_t i = wi / n_kv;
    const int64_t t = top[i * n_kv + h];
    const int D = n_kv * d;
    // x[h, i, :] = deq K[t, all heads] - K_mean (only for the library V-predict path)
    float *xr = x ? x + ((int64_t)h * k + i) * D : nullptr;
    for (int e = lane * 4; xr && e < D; e += 128) {
      const int hh = e / d, c = e - hh * d;
      const uint16_t two = *reinterpret_cast<const uint16_t *>(kp + (t * n_kv + hh) * (d / 2) + c / 2);
      const int codes[4] = {(int)((two >> 4) & 15) - 8, (int)(two & 15) - 8, (int)((two >> 12) & 15) - 8,
                            (int)((two >> 8) & 15) - 8};
      float4 o;
      float *op = &o.x;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float step = __fdiv_rn(__fmul_rn(2.0f, sc[hh * d + c + r]), 16.0f);
        op[r] = __fsub_rn(__fmul_rn((float)codes[r], step), kmean[e + r]);
      }
      *reinterpret_cast<float4 *>(xr + e) = o;
    }
    // ret_k[i, h, :] = RoPE(deq K[t, h]) at position t
    const uint16_t two = *reinterpret_cast<const uint16_t *>(kp + (t * n_kv + h) * (d / 2) + lane * 2);
    const int codes[4] = {(int)((two >> 4) & 15) - 8, (int)(two & 15) - 8, (int)((two >> 12) & 15) - 8,
                          (int)((two >> 8) & 15) - 8};
    float kx[4], out4[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
      kx[r] = __fmul_rn((float)codes[r], __fdiv_rn(__fmul_rn(2.0f, sc[h * d + lane * 4 + r]), 16.0f));
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float partner = __shfl_xor_sync(0xffffffffu, kx[r], 16);
      const float rh = lane < 16 ? -partner : partner;
      out4[r] = __fadd_rn(__fmul_rn(kx[r], cs[t * rope_stride + lane * 4 + r]),
                          __fmul_rn(rh, sn[t * rope_stride + lane * 4 + r]));
    }
    *reinterpret_cast<float4 *>(ret_k + (i * n_kv + h) * d + lane * 4) = make_float4(out4[0], out4[1], out4[2], out4[3]);
  }
}

__global__ void vres_add_kernel(const float *__restrict__ vb, const uint8_t *__restrict__ vr,
                                const float *__restrict__ vrs, const int64_t *__restrict__ top, int k, int n_kv,
                                uint16_t *__restrict__ out) {
  constexpr int d = 128;
  const int64_t total = (int64_t)k * n_kv * d;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % d);
    const int64_t ih = e / d;
    const int h = (int)(ih % n_kv);
    const int64_t i = ih / n_kv;
    const int64_t t = top[i * n_kv + h];
    const uint8_t byte = vr[(t * n_kv + h) * (d / 4) + c / 4];
    const int code = (int)((byte >> (6 - 2 * (c & 3))) & 3) - 2;
    const float step = __fdiv_rn(__fmul_rn(2.0f, vrs[h]), 4.0f);
    const float v = __fadd_rn(vb[((int64_t)h * k + i) * d + c], __fmul_rn((float)code, step));
    out[e] = __half_as_ushort(__float2half_rn(v));
  }
}

// ---------------------------------------------------------------- window ----
template <int DT>
__global__ void window_write_kernel(const void *__restrict__ k, const void *__restrict__ v, int64_t first,
                                   int64_t count, int64_t row_elems, uint16_t *__restrict__ rk,
                                   uint16_t *__restrict__ rv, int64_t cap, int64_t pos) {
  const int64_t total = count * row_elems;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / row_elems, c = e - i * row_elems;
    const int64_t src = (first + i) * row_elems + c;
    const int64_t slot = (pos + first + i) % cap;
    rk[slot * row_elems + c] = __half_as_ushort(__float2half_rn(load_elem<DT>(k, src)));
    rv[slot * row_elems + c] = __half_as_ushort(__float2half_rn(load_elem<DT>(v, src)));
  }
}

}  // namespace kvr

using namespace kvr;

extern "C" int kvr_absmax_scales(const void *x, int dtype, int64_t n, int64_t cols, float clamp_min, float *out,
                                 kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(x && out && n > 0 && cols > 0 && valid_dtype(dtype), "kvr_absmax_scales: bad arguments");
  cudaStream_t st = as_cuda(stream);
  if (cudaMemsetAsync(out, 0, cols * 4, st) != cudaSuccess) return check_launch("kvr_absmax_scales memset");
  const int64_t rows_per = 256;
  dim3 grid((unsigned)((cols + 255) / 256), (unsigned)((n + rows_per - 1) / rows_per));
  unsigned *bits = reinterpret_cast<unsigned *>(out);
  if (dtype == KVR_F32) absmax_kernel<KVR_F32><<<grid, 256, 0, st>>>(x, n, cols, rows_per, bits);
  else if (dtype == KVR_F16) absmax_kernel<KVR_F16><<<grid, 256, 0, st>>>(x, n, cols, rows_per, bits);
  else absmax_kernel<KVR_BF16><<<grid, 256, 0, st>>>(x, n, cols, rows_per, bits);
  clamp_min_kernel<<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(out, cols, clamp_min);
  return check_launch("kvr_absmax_scales");
}

extern "C" int kvr_int4w_encode_k(const void *k, int dtype, int64_t n, int n_kv, int d, int64_t tok_stride,
                                  const float *k_scales, uint8_t *k_packed, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(k && k_scales && k_packed && valid_dtype(dtype), "kvr_int4w_encode_k: bad arguments");
  KVR_REQUIRE(n >= 0 && n_kv > 0 && d > 0 && d % 16 == 0, "kvr_int4w_encode_k: d must be a multiple of 16");
  if (n == 0) return KVR_OK;
  const int64_t total = n * n_kv * (d / 8);
  cudaStream_t st = as_cuda(stream);
  if (dtype == KVR_F32) encode_k_kernel<KVR_F32><<<blocks_for(total, 256), 256, 0, st>>>(k, n, n_kv, d, tok_stride, k_scales, k_packed);
  else if (dtype == KVR_F16) encode_k_kernel<KVR_F16><<<blocks_for(total, 256), 256, 0, st>>>(k, n, n_kv, d, tok_stride, k_scales, k_packed);
  else encode_k_kernel<KVR_BF16><<<blocks_for(total, 256), 256, 0, st>>>(k, n, n_kv, d, tok_stride, k_scales, k_packed);
  return check_launch("kvr_int4w_encode_k");
}

extern "C" int kvr_int4w_encode_vres(const void *v, int dtype, const float *v_pred, int64_t n, int n_kv, int d,
                                     const float *vr_scales, uint8_t *vr_packed, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(v && v_pred && vr_scales && vr_packed && valid_dtype(dtype), "kvr_int4w_encode_vres: bad arguments");
  KVR_REQUIRE(n >= 0 && n_kv > 0 && d > 0 && d % 16 == 0, "kvr_int4w_encode_vres: d must be a multiple of 16");
  if (n == 0) return KVR_OK;
  const int64_t total = n * n_kv * (d / 16);
  cudaStream_t st = as_cuda(stream);
  if (dtype == KVR_F32) encode_vres_kernel<KVR_F32><<<blocks_for(total, 256), 256, 0, st>>>(v, v_pred, n, n_kv, d, vr_scales, vr_packed);
  else if (dtype == KVR_F16) encode_vres_kernel<KVR_F16><<<blocks_for(total, 256), 256, 0, st>>>(v, v_pred, n, n_kv, d, vr_scales, vr_packed);
  else encode_vres_kernel<KVR_BF16><<<blocks_for(total, 256), 256, 0, st>>>(v, v_pred, n, n_kv, d, vr_scales, vr_packed);
  return check_launch("kvr_int4w_encode_vres");
}

extern "C" int kvr_compute_scores(const float *q_avg, const uint8_t *k_pack, const float *k_scales, const float *cos_tbl,
                                  const float *sin_tbl, int n_kv, int d, int64_t n_stored, float *scores,
                                  kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(q_avg && k_pack && k_scales && cos_tbl && sin_tbl && scores, "kvr_compute_scores: null pointer");
  KVR_REQUIRE(n_kv > 0 && n_stored >= 0, "kvr_compute_scores: bad shape");
  KVR_REQUIRE(d == 64 || d == 128 || d == 256, "kvr_compute_scores: head_dim must be 64, 128 or 256 (got %d)", d);
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KVR_REQUIRE(al16(q_avg) && al16(k_pack) && al16(k_scales) && al16(cos_tbl) && al16(sin_tbl),
              "kvr_compute_scores: all inputs must be 16-byte aligned");
  if (n_stored == 0) return KVR_OK;
  const int64_t warps = (n_stored * n_kv + 31) / 32;
  int64_t bl = (warps + 7) / 8;
  int blocks = (int)(bl < 148 * 8 ? bl : 148 * 8);
  cudaStream_t st = as_cuda(stream);
  if (d == 64) compute_scores_kernel<64><<<blocks, 256, 0, st>>>(q_avg, k_pack, k_scales, cos_tbl, sin_tbl, n_kv, n_stored, scores);
  else if (d == 128) compute_scores_kernel<128><<<blocks, 256, 0, st>>>(q_avg, k_pack, k_scales, cos_tbl, sin_tbl, n_kv, n_stored, scores);
  else compute_scores_kernel<256><<<blocks, 256, 0, st>>>(q_avg, k_pack, k_scales, cos_tbl, sin_tbl, n_kv, n_stored, scores);
  return check_launch("kvr_compute_scores");
}

extern "C" int kvr_int4w_token_scores(const float *q, int n_q, const uint8_t *k_packed, const float *k_scales,
                                      const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                                      int rope_halves_equal, int n_kv, int d, int64_t n_stored, float *scores,
                                      int64_t score_stride, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == 128, "kvr_int4w_token_scores: head_dim must be 128");
  KVR_REQUIRE(n_kv > 0 && n_kv <= 8 && n_q % n_kv == 0, "kvr_int4w_token_scores: need n_kv <= 8, n_q %% n_kv == 0");
  KVR_REQUIRE(q && k_packed && k_scales && cos_tbl && sin_tbl && scores, "kvr_int4w_token_scores: null pointer");
  KVR_REQUIRE(score_stride >= n_stored && rope_stride >= (rope_halves_equal ? 64 : 128), "kvr_int4w_token_scores: bad strides");
  if (n_stored <= 0) return KVR_OK;
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(k_packed) & 15) == 0 && (reinterpret_cast<uintptr_t>(cos_tbl) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sin_tbl) & 15) == 0 && rope_stride % 4 == 0,
              "kvr_int4w_token_scores: packed rows and rope tables must be 16-byte aligned");
  KVR_REQUIRE(rope_stride >= (rope_halves_equal ? 64 : 128), "kvr_int4w_token_scores: rope rows too short");
  const int cw = rope_halves_equal ? 64 : 128;
  const size_t smem = 2 * ((size_t)kTsTile * n_kv * 64 + 2 * (size_t)kTsTile * cw * 4);
  const int64_t tiles = (n_stored + kTsTile - 1) / kTsTile;
  static thread_local int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaFuncSetAttribute(token_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    attr_dev = dev;
  }
  int64_t blocks = tiles < 148 * 3 ? tiles : 148 * 3;
  token_scores_kernel<<<(unsigned)blocks, 256, smem, as_cuda(stream)>>>(
      q, n_q, k_packed, k_scales, cos_tbl, sin_tbl, rope_stride, rope_halves_equal, n_kv, n_stored, scores,
      score_stride, nullptr, 0, 0);
  return check_launch("kvr_int4w_token_scores");
}

extern "C" int kvr_int4w_chunk_scores(const float *q, int n_q, const uint8_t *k_packed, const float *k_scales,
                                      const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                                      int rope_halves_equal, int n_kv, int d, int64_t n_stored, int chunk,
                                      float *scores, int64_t score_stride, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == 128, "kvr_int4w_chunk_scores: head_dim must be 128");
  KVR_REQUIRE(n_kv > 0 && n_kv <= 8 && n_q % n_kv == 0 && chunk > 0, "kvr_int4w_chunk_scores: bad shape");
  KVR_REQUIRE(q && k_packed && k_scales && cos_tbl && sin_tbl && scores, "kvr_int4w_chunk_scores: null pointer");
  const int64_t n_chunks = n_stored / chunk;
  KVR_REQUIRE(score_stride >= n_chunks, "kvr_int4w_chunk_scores: bad score stride");
  if (n_chunks <= 0) return KVR_OK;
  chunk_scores_kernel<<<blocks_for(n_chunks * n_kv, 8), 256, 0, as_cuda(stream)>>>(
      q, n_q, k_packed, k_scales, cos_tbl, sin_tbl, rope_stride, rope_halves_equal, n_kv, n_chunks, chunk, scores,
      score_stride);
  return check_launch("kvr_int4w_chunk_scores");
}

extern "C" int kvr_topk_rows(const float *scores, int rows, int64_t n, int64_t row_stride, int k, int64_t ex_start,
                             int64_t ex_end, int64_t *idx, float *vals, int64_t out_row_stride,
                             int64_t out_elem_stride, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(scores && idx && rows >= 0, "kvr_topk_rows: bad arguments");
  KVR_REQUIRE(k >= 0 && k <= n && k <= 4096, "kvr_topk_rows: need 0 <= k <= min(n, 4096) (k=%d n=%lld)", k, (long long)n);
  KVR_REQUIRE(n < 0xffffffffll, "kvr_topk_rows: rows longer than 2^32-1");
  if (rows == 0 || k == 0) return KVR_OK;
  int P = 1;
  while (P < k) P <<= 1;
  const size_t base = align_up(sizeof(TopkSmem), 16) + (size_t)P * 8;
  const size_t staged = base + (size_t)n * 4;
  const size_t hist = align_up(sizeof(TopkSmem), 16) + align_up(sizeof(HistSmem), 16) + (size_t)P * 16 +
                      (size_t)kHistCand * 8 + (size_t)n * 4;
  cudaStream_t st = as_cuda(stream);
  if (n >= 8192 && (int64_t)k * 4 <= n && hist <= 220 * 1024) {
    cudaFuncSetAttribute(topk_rows_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist);
    topk_rows_hist_kernel<<<rows, kTopkThreads, hist, st>>>(scores, n, row_stride, k, ex_start, ex_end, idx, vals,
                                                             out_row_stride, out_elem_stride);
  } else if (staged <= 200 * 1024) {
    cudaFuncSetAttribute(topk_rows_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)staged);
    topk_rows_kernel<true><<<rows, kTopkThreads, staged, st>>>(scores, n, row_stride, k, ex_start, ex_end, idx, vals,
                                                               out_row_stride, out_elem_stride);
  } else {
    if (base > 48 * 1024)
      cudaFuncSetAttribute(topk_rows_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)base);
    topk_rows_kernel<false><<<rows, kTopkThreads, base, st>>>(scores, n, row_stride, k, ex_start, ex_end, idx, vals,
                                                              out_row_stride, out_elem_stride);
  }
  return check_launch("kvr_topk_rows");
}

extern "C" int kvr_int4w_gather(const uint8_t *k_packed, const float *k_scales, const int64_t *top, int k, int n_kv,
                                int d, const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                                const float *k_mean, float *ret_k, float *x, const int32_t *count,
                                kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == 128, "kvr_int4w_gather: head_dim must be 128");
  KVR_REQUIRE(k_packed && k_scales && top && cos_tbl && sin_tbl && ret_k && (x == nullptr || k_mean),
              "kvr_int4w_gather: null pointer");
  KVR_REQUIRE(k >= 0 && n_kv > 0, "kvr_int4w_gather: bad shape");
  if (k == 0) return KVR_OK;
  gather_kernel<<<blocks_for((int64_t)k * n_kv, 8), 256, 0, as_cuda(stream)>>>(
      k_packed, k_scales, top, k, n_kv, cos_tbl, sin_tbl, rope_stride, k_mean, ret_k, x, count);
  return check_launch("kvr_int4w_gather");
}

extern "C" int kvr_int4w_vres_add(const float *v_base, const uint8_t *vr_packed, const float *vr_scales,
                                  const int64_t *top, int k, int n_kv, int d, uint16_t *ret_v, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == 128, "kvr_int4w_vres_add: head_dim must be 128");
  KVR_REQUIRE(v_base && vr_packed && vr_scales && top && ret_v && k >= 0 && n_kv > 0, "kvr_int4w_vres_add: bad arguments");
  if (k == 0) return KVR_OK;
  vres_add_kernel<<<blocks_for((int64_t)k * n_kv * d, 256), 256, 0, as_cuda(stream)>>>(v_base, vr_packed, vr_scales,
                                                                                        top, k, n_kv, ret_v);
  return check_launch("kvr_int4w_vres_add");
}

extern "C" int kvr_window_write(const void *k, const void *v, int dtype, int64_t n, int n_kv, int d, uint16_t *ring_k,
                                uint16_t *ring_v, int64_t cap, int64_t pos, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(k && v && ring_k && ring_v && valid_dtype(dtype), "kvr_window_write: bad arguments");
  KVR_REQUIRE(n >= 0 && cap > 0 && pos >= 0 && n_kv > 0 && d > 0, "kvr_window_write: bad shape");
  if (n == 0) return KVR_OK;
  const int64_t count = n < cap ? n : cap;
  const int64_t first = n - count;
  const int64_t row = (int64_t)n_kv * d;
  cudaStream_t st = as_cuda(stream);
  const int blocks = blocks_for(count * row, 256);
  if (dtype == KVR_F32) window_write_kernel<KVR_F32><<<blocks, 256, 0, st>>>(k, v, first, count, row, ring_k, ring_v, cap, pos);
  else if (dtype == KVR_F16) window_write_kernel<KVR_F16><<<blocks, 256, 0, st>>>(k, v, first, count, row, ring_k, ring_v, cap, pos);
  else window_write_kernel<KVR_BF16><<<blocks, 256, 0, st>>>(k, v, first, count, row, ring_k, ring_v, cap, pos);
  return check_launch("kvr_window_write");
}

// Workspace: a fixed header (histograms and counters of up to 8 heads, which
// must start at zero and are left at zero) at the same offsets whatever the
// shapes, so one workspace can serve calls of different shapes; then the
// per-call regions (rewritten before they are read).
constexpr size_t kTkHdrHist = 0;
constexpr size_t kTkHdrRows = (size_t)8 * kCosBins * 4;
constexpr size_t kTkHdr = kTkHdrRows + 256;

extern "C" size_t kvr_int4w_token_topk_workspace_bytes(int n_kv, int64_t n_stored, int k) {
  if (n_kv <= 0 || n_stored <= 0 || k <= 0) return kTkHdr;
  return kTkHdr + align_up((size_t)n_kv * k * 8, 256) + align_up((size_t)n_kv * kTkCand * 8, 256) +
         align_up((size_t)n_kv * n_stored * 4, 256);
}

extern "C" int kvr_int4w_token_topk(const float *q, int n_q, const uint8_t *k_packed, const float *k_scales,
                                    const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                                    int rope_halves_equal, int n_kv, int d, int64_t n_stored, int k, int64_t ex_start,
                                    int64_t ex_end, int64_t *idx, void *workspace, size_t workspace_bytes,
                                    kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == 128, "kvr_int4w_token_topk: head_dim must be 128");
  KVR_REQUIRE(n_kv > 0 && n_kv <= 8 && n_q % n_kv == 0, "kvr_int4w_token_topk: need n_kv <= 8, n_q %% n_kv == 0");
  KVR_REQUIRE(q && k_packed && k_scales && cos_tbl && sin_tbl && idx && workspace, "kvr_int4w_token_topk: null pointer");
  KVR_REQUIRE(n_stored > 0 && k > 0 && k <= n_stored && k <= 4096 && n_stored < 0xffffffffll,
              "kvr_int4w_token_topk: need 0 < k <= min(n_stored, 4096)");
  KVR_REQUIRE(workspace_bytes >= kvr_int4w_token_topk_workspace_bytes(n_kv, n_stored, k),
              "kvr_int4w_token_topk: workspace too small");
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "kvr_int4w_token_topk: workspace alignment");
  char *p = reinterpret_cast<char *>(workspace);
  int *hist = reinterpret_cast<int *>(p + kTkHdrHist);
  TkRow *rows = reinterpret_cast<TkRow *>(p + kTkHdrRows);
  p += kTkHdr;
  unsigned long long *above = reinterpret_cast<unsigned long long *>(p);
  p += align_up((size_t)n_kv * k * 8, 256);
  unsigned long long *cand = reinterpret_cast<unsigned long long *>(p);
  p += align_up((size_t)n_kv * kTkCand * 8, 256);
  float *scores = reinterpret_cast<float *>(p);
  // scores + histogram (the same launch as kvr_int4w_token_scores)
  KVR_REQUIRE((reinterpret_cast<uintptr_t>(k_packed) & 15) == 0 && (reinterpret_cast<uintptr_t>(cos_tbl) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sin_tbl) & 15) == 0 && rope_stride % 4 == 0 &&
                  rope_stride >= (rope_halves_equal ? 64 : 128),
              "kvr_int4w_token_topk: packed rows and rope tables must be 16-byte aligned");
  const int cw = rope_halves_equal ? 64 : 128;
  const size_t smem = 2 * ((size_t)kTsTile * n_kv * 64 + 2 * (size_t)kTsTile * cw * 4);
  const int64_t tiles = (n_stored + kTsTile - 1) / kTsTile;
  cudaStream_t st = as_cuda(stream);
  static thread_local int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  int P = 1;
  while (P < k) P <<= 1;
  const size_t fin_smem = TkFinSmem(P).total;
  if (attr_dev != dev) {
    cudaFuncSetAttribute(token_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    cudaFuncSetAttribute(tk_finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TkFinSmem(4096).total);
    attr_dev = dev;
  }
  const int64_t blocks = tiles < 148 * 3 ? tiles : 148 * 3;
  token_scores_kernel<<<(unsigned)blocks, 256, smem, st>>>(q, n_q, k_packed, k_scales, cos_tbl, sin_tbl, rope_stride,
                                                          rope_halves_equal, n_kv, n_stored, scores, n_stored, nullptr,
                                                          0, 0);
  dim3 sg((unsigned)kTkSegs, (unsigned)n_kv);
  tk_hist_kernel<<<sg, 256, 0, st>>>(scores, n_stored, ex_start, ex_end, hist);
  tk_split_kernel<<<sg, 256, 0, st>>>(scores, n_stored, k, ex_start, ex_end, hist, rows, above, cand);
  tk_finalize_kernel<<<n_kv, kTopkThreads, fin_smem, st>>>(scores, n_stored, k, ex_start, ex_end, hist, rows, above,
                                                           cand, idx, n_kv);
  return check_launch("kvr_int4w_token_topk");
}
