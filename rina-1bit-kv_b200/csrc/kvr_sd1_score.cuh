// Warp-level sd1 tile selection score (shared by the selection kernel and the
// fused decode kernel).  Spec: oracle/sd1_ref.py tile_scores — bit-exact.
#pragma once

#include "kvr_common.cuh"

namespace kvr {

// qp: transformed group-mean query (128 fp32, shared memory); kb: this lane's
// TILE/32 token rows (16 bytes = 4 words each, token lane + 32 r); ks: fp16
// scales of channels lane + 32 m.  Lane c of the ballots owns channels
// c, 32 + c, 64 + c, 96 + c, i.e. bit c of words 0..3.
//   w_c = q'_c * s_c, M = max|w|, wq = rint(w * (127/M)),
//   S_j = 2 * sum_c wq_c bit_jc - sum_c wq_c  (bit planes + popcount),
//   score = float(max_j S_j) * (M / 127).
template <int TILE>
__device__ __forceinline__ float sd1_score_tile(const float *qp, const uint4 (&kb)[TILE / 32], const uint16_t (&ks)[4],
                                                int lane) {
  constexpr int TPL = TILE / 32;
  int wq[4];
  float w[4], mx = 0.0f;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    w[m] = __fmul_rn(qp[lane + 32 * m], __half2float(__ushort_as_half(ks[m])));
    mx = fmaxf(mx, fabsf(w[m]));
  }
  mx = warp_max(mx);
  const float inv = mx > 0.0f ? __fdiv_rn(127.0f, mx) : 0.0f;
  int wsum = 0;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    wq[m] = __float2int_rn(__fmul_rn(w[m], inv));
    wsum += wq[m];
  }
  wsum = warp_sum_int(wsum);
  uint32_t plane[8][4];
#pragma unroll
  for (int p = 0; p < 8; ++p)
#pragma unroll
    for (int m = 0; m < 4; ++m) plane[p][m] = __ballot_sync(0xffffffffu, (wq[m] >> p) & 1);
  int best = INT_MIN;
#pragma unroll
  for (int r = 0; r < TPL; ++r) {
    const uint32_t bw[4] = {kb[r].x, kb[r].y, kb[r].z, kb[r].w};
    int P = 0;
#pragma unroll
    for (int p = 0; p < 7; ++p) {
      int cnt = 0;
#pragma unroll
      for (int m = 0; m < 4; ++m) cnt += __popc(plane[p][m] & bw[m]);
      P += cnt << p;
    }
    int c7 = 0;
#pragma unroll
    for (int m = 0; m < 4; ++m) c7 += __popc(plane[7][m] & bw[m]);
    P -= c7 << 7;
    best = max(best, 2 * P - wsum);
  }
  best = warp_max_int(best);
  return __fmul_rn((float)best, __fdiv_rn(mx, 127.0f));
}

// Two tiles at once, their dependency chains interleaved (same arithmetic
// and results as two sd1_score_tile calls).
template <int TILE>
__device__ __forceinline__ void sd1_score_tile2(const float *qp, const uint4 (&kb)[2][TILE / 32],
                                                const uint16_t (&ks)[2][4], int lane, float (&out)[2]) {
  constexpr int TPL = TILE / 32;
  int wq[2][4];
  float w[2][4], mx[2] = {0.0f, 0.0f};
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float qv = qp[lane + 32 * m];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      w[u][m] = __fmul_rn(qv, __half2float(__ushort_as_half(ks[u][m])));
      mx[u] = fmaxf(mx[u], fabsf(w[u][m]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < 2; ++u) mx[u] = fmaxf(mx[u], __shfl_xor_sync(0xffffffffu, mx[u], o));
  int wsum[2] = {0, 0};
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const float inv = mx[u] > 0.0f ? __fdiv_rn(127.0f, mx[u]) : 0.0f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      wq[u][m] = __float2int_rn(__fmul_rn(w[u][m], inv));
      wsum[u] += wq[u][m];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < 2; ++u) wsum[u] += __shfl_xor_sync(0xffffffffu, wsum[u], o);
  int best[2] = {INT_MIN, INT_MIN};
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    uint32_t plane[8][4];
#pragma unroll
    for (int p = 0; p < 8; ++p)
#pragma unroll
      for (int m = 0; m < 4; ++m) plane[p][m] = __ballot_sync(0xffffffffu, (wq[u][m] >> p) & 1);
#pragma unroll
    for (int r = 0; r < TPL; ++r) {
      const uint32_t bw[4] = {kb[u][r].x, kb[u][r].y, kb[u][r].z, kb[u][r].w};
      int P = 0;
#pragma unroll
      for (int p = 0; p < 7; ++p) {
        int cnt = 0;
#pragma unroll
        for (int m = 0; m < 4; ++m) cnt += __popc(plane[p][m] & bw[m]);
        P += cnt << p;
      }
      int c7 = 0;
#pragma unroll
      for (int m = 0; m < 4; ++m) c7 += __popc(plane[7][m] & bw[m]);
      P -= c7 << 7;
      best[u] = max(best[u], 2 * P - wsum[u]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < 2; ++u) best[u] = max(best[u], __shfl_xor_sync(0xffffffffu, best[u], o));
#pragma unroll
  for (int u = 0; u < 2; ++u) out[u] = __fmul_rn((float)best[u], __fdiv_rn(mx[u], 127.0f));
}

}  // namespace kvr
