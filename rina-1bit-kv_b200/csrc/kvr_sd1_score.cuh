// Warp-level sd1 tile selection score (shared by the selection kernel and the
// fused decode kernel).  Spec: oracle/sd1_ref.py tile_scores — bit-exact.
#pragma once

#include "kvr_common.cuh"

namespace kvr {

// P = sum_{p<7} 2^p popc(plane_p & x) - 2^7 popc(plane_7 & x) over the 4
// words of one token row.  Planes 6 and 7 go through one carry-save full
// adder each (three popcounts instead of four: popc(a)+popc(b)+popc(c) =
// popc(a^b^c) + 2 popc(maj(a,b,c))), which moves work from the popcount unit
// to the logic pipe where that pays: the scan is bound by the two together.
__device__ __forceinline__ int sd1_plane_dot(const uint32_t (&plane)[8][4], const uint32_t (&bw)[4]) {
  int P = 0;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const uint32_t a = plane[p][0] & bw[0], b = plane[p][1] & bw[1], c = plane[p][2] & bw[2],
                   d = plane[p][3] & bw[3];
    int cnt;
    if (p >= 6) {
      const uint32_t sum = a ^ b ^ c, carry = (a & b) | (c & (a ^ b));
      cnt = __popc(sum) + __popc(d) + 2 * __popc(carry);
    } else {
      cnt = __popc(a) + __popc(b) + __popc(c) + __popc(d);
    }
    P += p == 7 ? -(cnt << 7) : (cnt << p);
  }
  return P;
}

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
    best = max(best, 2 * sd1_plane_dot(plane, bw) - wsum);
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
      best[u] = max(best[u], 2 * sd1_plane_dot(plane, bw) - wsum[u]);
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
