// Warp-level orthonormal transforms along head_dim (d = 128) for the sd1 codec.
//
// Register layout: lane L holds elements 4L .. 4L+3 of the vector in x[0..3].
// Every arithmetic step uses explicit round-to-nearest intrinsics so the
// results are bit-identical to the CPU specification (operation order fixed,
// no FMA contraction):
//   * Walsh-Hadamard: butterfly stages of stride 1, 2, 4, ..., 64 with
//     (a, b) -> (a + b, a - b), then x * fp32(1/sqrt(128));
//   * DCT-II: Lee's recursive factorisation (split levels M = 128..2:
//     a_j = x_j + x_{M-1-j}, b_j = (x_j - x_{M-1-j}) * f_M[j]; merge levels
//     M = 2..128: y_{2k} = A_k, y_{2k+1} = B_k + B_{k+1}), then the
//     orthonormal scaling sqrt(1/128) for k = 0 and sqrt(2/128) otherwise;
//   * DCT-III (inverse): the transposed flow graph of the above.
// The DCT variants stage through a 256-float per-warp shared buffer; the
// Hadamard runs entirely in registers with xor shuffles.
#pragma once

#include "kvr_common.cuh"
#include "kvr_lee_table.h"

namespace kvr {

constexpr int kD = 128;
constexpr uint32_t kInvSqrt128Bits = 0x3db504f3u;  // fp32(1/sqrt(128)) == fp32(sqrt(1/128))

__device__ __forceinline__ void wht128(float (&x)[4], int lane) {
  float a0 = x[0], a1 = x[1], a2 = x[2], a3 = x[3];
  // stride 1
  x[0] = __fadd_rn(a0, a1); x[1] = __fsub_rn(a0, a1);
  x[2] = __fadd_rn(a2, a3); x[3] = __fsub_rn(a2, a3);
  // stride 2
  a0 = x[0]; a1 = x[1]; a2 = x[2]; a3 = x[3];
  x[0] = __fadd_rn(a0, a2); x[2] = __fsub_rn(a0, a2);
  x[1] = __fadd_rn(a1, a3); x[3] = __fsub_rn(a1, a3);
  // strides 4..64 live across lanes (lane mask 1..16)
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float p = __shfl_xor_sync(0xffffffffu, x[r], m);
      x[r] = upper ? __fsub_rn(p, x[r]) : __fadd_rn(x[r], p);
    }
  }
  const float c = __uint_as_float(kInvSqrt128Bits);
#pragma unroll
  for (int r = 0; r < 4; ++r) x[r] = __fmul_rn(x[r], c);
}

// Loads the Lee factors into shared memory (call by all threads of a block,
// followed by a __syncthreads before first use).
__device__ __forceinline__ void load_lee(float *lee_s) {
  for (int i = threadIdx.x; i < kD - 1; i += blockDim.x) lee_s[i] = __uint_as_float(__ldg(kLeeBitsGlobal + i));
}

// Lee levels as compile-time steps (block size M is a template constant, so
// every index below is shift/mask arithmetic).
template <int M>
__device__ __forceinline__ void lee_split(const float *in, float *out, const float *lee, int lane) {
  constexpr int half = M / 2;
  const float *f = lee + half - 1;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int p = lane + 32 * q;
    const int o = (p / half) * M, j = p % half;
    const float xa = in[o + j], xb = in[o + M - 1 - j];
    out[o + j] = __fadd_rn(xa, xb);
    out[o + half + j] = __fmul_rn(__fsub_rn(xa, xb), f[j]);
  }
}
template <int M>
__device__ __forceinline__ void lee_merge(const float *in, float *out, int lane) {
  constexpr int half = M / 2;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int i = lane + 32 * q;
    const int o = (i / M) * M, r = i % M;
    float v;
    if ((r & 1) == 0) {
      v = in[o + (r >> 1)];
    } else {
      const int k = r >> 1;
      v = in[o + half + k];
      if (k < half - 1) v = __fadd_rn(v, in[o + half + k + 1]);
    }
    out[i] = v;
  }
}
template <int M>
__device__ __forceinline__ void lee_merge_t(const float *in, float *out, int lane) {
  constexpr int half = M / 2;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int i = lane + 32 * q;
    const int o = (i / M) * M, r = i % M;
    float v;
    if (r < half) {
      v = in[o + 2 * r];
    } else {
      const int k = r - half;
      v = in[o + 2 * k + 1];
      if (k > 0) v = __fadd_rn(v, in[o + 2 * k - 1]);
    }
    out[i] = v;
  }
}
template <int M>
__device__ __forceinline__ void lee_split_t(const float *in, float *out, const float *lee, int lane) {
  constexpr int half = M / 2;
  const float *f = lee + half - 1;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int p = lane + 32 * q;
    const int o = (p / half) * M, j = p % half;
    const float a = in[o + j], fb = __fmul_rn(in[o + half + j], f[j]);
    out[o + j] = __fadd_rn(a, fb);
    out[o + M - 1 - j] = __fsub_rn(a, fb);
  }
}

// buf: 256 floats owned by this warp.  lee: the 127 factors (shared memory).
__device__ __forceinline__ void dct128_fwd(float (&x)[4], int lane, float *buf, const float *lee) {
  float *A = buf, *B = buf + kD;
  reinterpret_cast<float4 *>(A)[lane] = make_float4(x[0], x[1], x[2], x[3]);
  __syncwarp();
  lee_split<128>(A, B, lee, lane); __syncwarp();
  lee_split<64>(B, A, lee, lane); __syncwarp();
  lee_split<32>(A, B, lee, lane); __syncwarp();
  lee_split<16>(B, A, lee, lane); __syncwarp();
  lee_split<8>(A, B, lee, lane); __syncwarp();
  lee_split<4>(B, A, lee, lane); __syncwarp();
  lee_split<2>(A, B, lee, lane); __syncwarp();
  lee_merge<2>(B, A, lane); __syncwarp();
  lee_merge<4>(A, B, lane); __syncwarp();
  lee_merge<8>(B, A, lane); __syncwarp();
  lee_merge<16>(A, B, lane); __syncwarp();
  lee_merge<32>(B, A, lane); __syncwarp();
  lee_merge<64>(A, B, lane); __syncwarp();
  lee_merge<128>(B, A, lane); __syncwarp();
  const float4 r4 = reinterpret_cast<const float4 *>(A)[lane];
  __syncwarp();
  const float c0 = __uint_as_float(kDctC0Bits), c1 = __uint_as_float(kDctC1Bits);
  x[0] = __fmul_rn(r4.x, lane == 0 ? c0 : c1);
  x[1] = __fmul_rn(r4.y, c1);
  x[2] = __fmul_rn(r4.z, c1);
  x[3] = __fmul_rn(r4.w, c1);
}

__device__ __forceinline__ void dct128_inv(float (&x)[4], int lane, float *buf, const float *lee) {
  const float c0 = __uint_as_float(kDctC0Bits), c1 = __uint_as_float(kDctC1Bits);
  float *A = buf, *B = buf + kD;
  reinterpret_cast<float4 *>(A)[lane] = make_float4(__fmul_rn(x[0], lane == 0 ? c0 : c1), __fmul_rn(x[1], c1),
                                                     __fmul_rn(x[2], c1), __fmul_rn(x[3], c1));
  __syncwarp();
  lee_merge_t<128>(A, B, lane); __syncwarp();
  lee_merge_t<64>(B, A, lane); __syncwarp();
  lee_merge_t<32>(A, B, lane); __syncwarp();
  lee_merge_t<16>(B, A, lane); __syncwarp();
  lee_merge_t<8>(A, B, lane); __syncwarp();
  lee_merge_t<4>(B, A, lane); __syncwarp();
  lee_merge_t<2>(A, B, lane); __syncwarp();
  lee_split_t<2>(B, A, lee, lane); __syncwarp();
  lee_split_t<4>(A, B, lee, lane); __syncwarp();
  lee_split_t<8>(B, A, lee, lane); __syncwarp();
  lee_split_t<16>(A, B, lee, lane); __syncwarp();
  lee_split_t<32>(B, A, lee, lane); __syncwarp();
  lee_split_t<64>(A, B, lee, lane); __syncwarp();
  lee_split_t<128>(B, A, lee, lane); __syncwarp();
  const float4 r4 = reinterpret_cast<const float4 *>(A)[lane];
  __syncwarp();
  x[0] = r4.x; x[1] = r4.y; x[2] = r4.z; x[3] = r4.w;
}

// kind: KVR_HADAMARD or KVR_DCT; the Hadamard is its own inverse.
__device__ __forceinline__ void transform128(float (&x)[4], int lane, int kind, bool inverse, float *buf,
                                             const float *lee) {
  if (kind == KVR_HADAMARD) {
    wht128(x, lane);
  } else if (inverse) {
    dct128_inv(x, lane, buf, lee);
  } else {
    dct128_fwd(x, lane, buf, lee);
  }
}

// ---- one thread per vector: all 128 elements in registers (x[0..127]).
// Same operations in the same order as the warp versions above (so the same
// bits), with every index a compile-time constant: no shuffles, no shared
// memory, factors read as constant-bank operands.  Used by the encoder,
// where each thread transforms one token vector.
__device__ __forceinline__ float lee_factor(int i) { return __uint_as_float(kLeeBits[i]); }

__device__ __forceinline__ void wht128_reg(float (&x)[kD]) {
#pragma unroll
  for (int m = 1; m < kD; m <<= 1) {
#pragma unroll
    for (int i = 0; i < kD; ++i) {
      if ((i & m) == 0) {
        const float a = x[i], b = x[i + m];
        x[i] = __fadd_rn(a, b);
        x[i + m] = __fsub_rn(a, b);
      }
    }
  }
  const float c = __uint_as_float(kInvSqrt128Bits);
#pragma unroll
  for (int i = 0; i < kD; ++i) x[i] = __fmul_rn(x[i], c);
}

template <int M>
__device__ __forceinline__ void lee_split_reg(const float (&in)[kD], float (&out)[kD]) {
  constexpr int half = M / 2;
#pragma unroll
  for (int o = 0; o < kD; o += M) {
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float xa = in[o + j], xb = in[o + M - 1 - j];
      out[o + j] = __fadd_rn(xa, xb);
      out[o + half + j] = __fmul_rn(__fsub_rn(xa, xb), lee_factor(half - 1 + j));
    }
  }
}
template <int M>
__device__ __forceinline__ void lee_merge_reg(const float (&in)[kD], float (&out)[kD]) {
  constexpr int half = M / 2;
#pragma unroll
  for (int o = 0; o < kD; o += M) {
#pragma unroll
    for (int k = 0; k < half; ++k) {
      out[o + 2 * k] = in[o + k];
      out[o + 2 * k + 1] = k < half - 1 ? __fadd_rn(in[o + half + k], in[o + half + k + 1]) : in[o + half + k];
    }
  }
}

__device__ __forceinline__ void dct128_fwd_reg(float (&x)[kD]) {
  float y[kD];
  lee_split_reg<128>(x, y);
  lee_split_reg<64>(y, x);
  lee_split_reg<32>(x, y);
  lee_split_reg<16>(y, x);
  lee_split_reg<8>(x, y);
  lee_split_reg<4>(y, x);
  lee_split_reg<2>(x, y);
  lee_merge_reg<2>(y, x);
  lee_merge_reg<4>(x, y);
  lee_merge_reg<8>(y, x);
  lee_merge_reg<16>(x, y);
  lee_merge_reg<32>(y, x);
  lee_merge_reg<64>(x, y);
  lee_merge_reg<128>(y, x);
  const float c0 = __uint_as_float(kDctC0Bits), c1 = __uint_as_float(kDctC1Bits);
  x[0] = __fmul_rn(x[0], c0);
#pragma unroll
  for (int i = 1; i < kD; ++i) x[i] = __fmul_rn(x[i], c1);
}

// ---- quad form: 4 lanes per vector, 32 elements per lane in registers.
// Lane t (= lane & 3) of a quad enters and leaves holding elements
// 32t .. 32t+31 in order; the 8 quads of a warp transform 8 vectors at once
// (all 32 lanes must call).  Only the two outermost Lee levels on each side
// cross lanes: for the forward split levels the lanes hold their blocks in
// orientations chosen so that the partner element sits in the SAME register
// of the xor partner (one shuffle per element, no index arithmetic); the
// 128-point merge goes through `scr` (128 floats per quad, private to the
// quad).  Every value is produced by the same operation on the same operands
// as in the specification, so the results are bit-identical to dct128_fwd /
// dct128_inv.  Latency: ~1 k instructions per lane, no block barriers.
template <int N, int M>
__device__ __forceinline__ void lee_split_n(float (&v)[N]) {
  constexpr int half = M / 2;
  float y[N];
#pragma unroll
  for (int o = 0; o < N; o += M) {
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float xa = v[o + j], xb = v[o + M - 1 - j];
      y[o + j] = __fadd_rn(xa, xb);
      y[o + half + j] = __fmul_rn(__fsub_rn(xa, xb), lee_factor(half - 1 + j));
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = y[i];
}
template <int N, int M>
__device__ __forceinline__ void lee_merge_n(float (&v)[N]) {
  constexpr int half = M / 2;
  float y[N];
#pragma unroll
  for (int o = 0; o < N; o += M) {
#pragma unroll
    for (int k = 0; k < half; ++k) {
      y[o + 2 * k] = v[o + k];
      y[o + 2 * k + 1] = k < half - 1 ? __fadd_rn(v[o + half + k], v[o + half + k + 1]) : v[o + half + k];
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = y[i];
}
// transposed levels (inverse)
template <int N, int M>
__device__ __forceinline__ void lee_merge_t_n(float (&v)[N]) {
  constexpr int half = M / 2;
  float y[N];
#pragma unroll
  for (int o = 0; o < N; o += M) {
#pragma unroll
    for (int k = 0; k < half; ++k) {
      y[o + k] = v[o + 2 * k];
      y[o + half + k] = k > 0 ? __fadd_rn(v[o + 2 * k + 1], v[o + 2 * k - 1]) : v[o + 1];
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = y[i];
}
template <int N, int M>
__device__ __forceinline__ void lee_split_t_n(float (&v)[N]) {
  constexpr int half = M / 2;
  float y[N];
#pragma unroll
  for (int o = 0; o < N; o += M) {
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float a = v[o + j], fb = __fmul_rn(v[o + half + j], lee_factor(half - 1 + j));
      y[o + j] = __fadd_rn(a, fb);
      y[o + M - 1 - j] = __fsub_rn(a, fb);
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = y[i];
}

__device__ __forceinline__ void quad_reverse_if(float (&v)[32], bool rev) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float a = v[i], b = v[31 - i];
    v[i] = rev ? b : a;
    v[31 - i] = rev ? a : b;
  }
}

__device__ __forceinline__ void dct128_fwd_quad(float (&v)[32], int lane, float *scr) {
  const int t = lane & 3;
  // split 128 (partner: t ^ 3).  Lanes 1 and 3 hold their block reversed, so
  // register i of a lane and register i of its partner form a pair (j, 127-j).
  quad_reverse_if(v, (t & 1) != 0);
  {
    const bool ra = t < 2;  // lanes 0, 1 keep a_j = x_j + x_{127-j}; lanes 2, 3 form b_j
    const float sg = ra ? 1.0f : -1.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float r = __shfl_xor_sync(0xffffffffu, v[i], 3);
      // b-role: lane 3 holds x_{127-i} (pairs with x_i: factor index i),
      // lane 2 holds x_{64+i} (pairs with x_{63-i}: factor index 63-i)
      const float f = t == 3 ? lee_factor(63 + i) : lee_factor(126 - i);
      const float sum = __fadd_rn(r, v[i] * sg);  // a: x_j + x_{127-j}; b: x_j - x_{127-j}
      v[i] = __fmul_rn(sum, ra ? 1.0f : f);
    }
  }
  // now lane 0: [0,32), lane 1: [32,64) reversed, lane 3: [64,96), lane 2: [96,128) reversed
  // split 64 (partner: t ^ 1); lanes 0 and 3 hold the first halves
  {
    const bool fa = t == 0 || t == 3;
    const float sg = fa ? 1.0f : -1.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float r = __shfl_xor_sync(0xffffffffu, v[i], 1);
      const float sum = __fadd_rn(r, v[i] * sg);
      v[i] = __fmul_rn(sum, fa ? 1.0f : lee_factor(31 + i));
    }
  }
  // lane 0: [0,32), lane 1: [32,64), lane 3: [64,96), lane 2: [96,128), all in order
  lee_split_n<32, 32>(v);
  lee_split_n<32, 16>(v);
  lee_split_n<32, 8>(v);
  lee_split_n<32, 4>(v);
  lee_split_n<32, 2>(v);
  lee_merge_n<32, 2>(v);
  lee_merge_n<32, 4>(v);
  lee_merge_n<32, 8>(v);
  lee_merge_n<32, 16>(v);
  lee_merge_n<32, 32>(v);
  // merge 64 (partner t ^ 1): first-half lanes (A) emit block positions 0..31,
  // second-half lanes (B) emit 32..63
  {
    const bool first = t == 0 || t == 3;
    float rcv[17];
#pragma unroll
    for (int k = 0; k < 17; ++k) {
      const float send = first ? v[16 + k < 32 ? 16 + k : 31] : v[k];
      rcv[k] = __shfl_xor_sync(0xffffffffu, send, 1);
    }
    float o[32];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      o[2 * k] = first ? v[k] : rcv[k];
      const float bf = __fadd_rn(rcv[k], rcv[k + 1]);
      const float bs = k < 15 ? __fadd_rn(v[16 + k], v[17 + k]) : v[31];
      o[2 * k + 1] = first ? bf : bs;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = o[i];
  }
  // merge 128 and the orthonormal scaling through the quad's scratch
  const int quad_base = (lane >> 2) * kD;
  float *q = scr + quad_base;
  const int bpos = t == 2 ? 96 : (t == 3 ? 64 : 32 * t);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    reinterpret_cast<float4 *>(q + bpos)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  __syncwarp();
  const float c0 = __uint_as_float(kDctC0Bits), c1 = __uint_as_float(kDctC1Bits);
  float A[16], B[17];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 a4 = reinterpret_cast<const float4 *>(q + 16 * t)[i];
    const float4 b4 = reinterpret_cast<const float4 *>(q + 64 + 16 * t)[i];
    A[4 * i] = a4.x; A[4 * i + 1] = a4.y; A[4 * i + 2] = a4.z; A[4 * i + 3] = a4.w;
    B[4 * i] = b4.x; B[4 * i + 1] = b4.y; B[4 * i + 2] = b4.z; B[4 * i + 3] = b4.w;
  }
  B[16] = t < 3 ? q[64 + 16 * t + 16] : 0.0f;
  __syncwarp();
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    v[2 * m] = __fmul_rn(A[m], (t == 0 && m == 0) ? c0 : c1);
    const float bo = (t == 3 && m == 15) ? B[15] : __fadd_rn(B[m], B[m + 1]);
    v[2 * m + 1] = __fmul_rn(bo, c1);
  }
}

__device__ __forceinline__ void dct128_inv_quad(float (&v)[32], int lane, float *scr) {
  const int t = lane & 3;
  const float c0 = __uint_as_float(kDctC0Bits), c1 = __uint_as_float(kDctC1Bits);
  const int quad_base = (lane >> 2) * kD;
  float *q = scr + quad_base;
  // scaling, then the transposed merges 128 and 64 read from the scratch:
  // y -> new (new_k = y_2k, B_j = new_{64+j} = y_{2j+1} + y_{2j-1}) -> the
  // 64-blocks; lane t takes block positions 32t .. 32t+31 of the result
#pragma unroll
  for (int i = 0; i < 8; ++i)
    reinterpret_cast<float4 *>(q + 32 * t)[i] =
        make_float4(__fmul_rn(v[4 * i], (t == 0 && i == 0) ? c0 : c1), __fmul_rn(v[4 * i + 1], c1),
                    __fmul_rn(v[4 * i + 2], c1), __fmul_rn(v[4 * i + 3], c1));
  __syncwarp();
  if (t == 0) {
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = q[4 * k];
  } else if (t == 1) {
    v[0] = q[2];
#pragma unroll
    for (int k = 1; k < 32; ++k) v[k] = __fadd_rn(q[4 * k + 2], q[4 * k - 2]);
  } else {
    // B_j = y_{2j+1} + y_{2j-1} (B_0 = y_1)
    float Bv[65];
    Bv[0] = q[1];
#pragma unroll
    for (int j = 1; j < 64; ++j) Bv[j] = __fadd_rn(q[2 * j + 1], q[2 * j - 1]);
    if (t == 2) {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = Bv[2 * k];
    } else {
      v[0] = Bv[1];
#pragma unroll
      for (int k = 1; k < 32; ++k) v[k] = __fadd_rn(Bv[2 * k + 1], Bv[2 * k - 1]);
    }
  }
  __syncwarp();
  lee_merge_t_n<32, 32>(v);
  lee_merge_t_n<32, 16>(v);
  lee_merge_t_n<32, 8>(v);
  lee_merge_t_n<32, 4>(v);
  lee_merge_t_n<32, 2>(v);
  lee_split_t_n<32, 2>(v);
  lee_split_t_n<32, 4>(v);
  lee_split_t_n<32, 8>(v);
  lee_split_t_n<32, 16>(v);
  lee_split_t_n<32, 32>(v);
  // transposed split 64 (partner t ^ 1): lanes 0, 2 hold a, lanes 1, 3 hold b
  {
    const bool first = (t & 1) == 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float r = __shfl_xor_sync(0xffffffffu, v[i], 1);
      const float a = first ? v[i] : r, b = first ? r : v[i];
      const float fb = __fmul_rn(b, lee_factor(31 + i));
      v[i] = first ? __fadd_rn(a, fb) : __fsub_rn(a, fb);  // second lanes: position 63-i
    }
  }
  // lane 0: [0,32), lane 1: [32,64) reversed, lane 2: [64,96), lane 3: [96,128) reversed
  // transposed split 128 (partner t ^ 2): lanes 0, 1 hold a, lanes 2, 3 hold b
  {
    const bool ha = t < 2;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float r = __shfl_xor_sync(0xffffffffu, v[i], 2);
      const float a = ha ? v[i] : r, b = ha ? r : v[i];
      const float fb = __fmul_rn(b, (t & 1) ? lee_factor(126 - i) : lee_factor(63 + i));
      v[i] = ha ? __fadd_rn(a, fb) : __fsub_rn(a, fb);
    }
  }
  // lane 0: [0,32), lane 1: [32,64) reversed, lane 2: [96,128) reversed, lane 3: [64,96)
  const bool rev = t == 1 || t == 2;
  const int bpos = t == 2 ? 96 : (t == 3 ? 64 : 32 * t);
#pragma unroll
  for (int i = 0; i < 32; ++i) q[bpos + (rev ? 31 - i : i)] = v[i];
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 x4 = reinterpret_cast<const float4 *>(q + 32 * t)[i];
    v[4 * i] = x4.x; v[4 * i + 1] = x4.y; v[4 * i + 2] = x4.z; v[4 * i + 3] = x4.w;
  }
  __syncwarp();
}

// ---- strided warp form: lane l holds elements l, 32+l, 64+l, 96+l in
// x[0..3] (the layout the tile scoring reads q' in).  Every Lee level moves
// data register to register with shuffles: the 128- and 64-point levels pair
// slot s with slot s' at lane 31-l (one xor-31 shuffle), the levels of 32
// points and less stay inside a slot (at most three shuffles with computed
// source lanes).  No shared-memory round trips, no warp barriers; the same
// operations on the same operands as the specification (bit-identical to
// dct128_fwd / dct128_inv).  lee: the 127 Lee factors (any memory).
__device__ __forceinline__ float shf_(float v, int src) { return __shfl_sync(0xffffffffu, v, src); }
__device__ __forceinline__ float shx_(float v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }

template <int M>
__device__ __forceinline__ void lee_split_shfl(float (&x)[4], int lane, const float *lee) {
  constexpr int half = M / 2;
  const int q = lane & (M - 1);
  const bool first = q < half;
  const float f = lee[half - 1 + (q & (half - 1))];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const float v = x[s];
    const float r1 = shx_(v, M - 1), r2 = shx_(v, half), r3 = shx_(v, half - 1);
    const float A = first ? v : r2, B = first ? r1 : r3;
    x[s] = first ? __fadd_rn(A, B) : __fmul_rn(__fsub_rn(A, B), f);
  }
}
template <int M>
__device__ __forceinline__ void lee_merge_shfl(float (&x)[4], int lane) {
  constexpr int half = M / 2;
  const int q = lane & (M - 1), base = lane & ~(M - 1), k = q >> 1;
  const bool even = (q & 1) == 0, last = q == M - 1;
  const int s1 = base + k, s2 = base + half + k, s3 = min(base + half + k + 1, base + M - 1);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const float v = x[s];
    const float r1 = shf_(v, s1), r2 = shf_(v, s2), r3 = shf_(v, s3);
    x[s] = even ? r1 : (last ? r2 : __fadd_rn(r2, r3));
  }
}

__device__ __forceinline__ void dct128_fwd_shfl(float (&x)[4], int lane, const float *lee) {
  {  // split 128: slot pairs (0,3), (1,2) at mirrored lanes
    const float b3 = shx_(x[3], 31), b2 = shx_(x[2], 31);
    const float f0 = lee[63 + lane], f1 = lee[95 + lane];
    const float n0 = __fadd_rn(x[0], b3), n1 = __fadd_rn(x[1], b2);
    const float n2 = __fmul_rn(__fsub_rn(x[0], b3), f0), n3 = __fmul_rn(__fsub_rn(x[1], b2), f1);
    x[0] = n0; x[1] = n1; x[2] = n2; x[3] = n3;
  }
  {  // split 64: slot pairs (0,1), (2,3)
    const float f = lee[31 + lane];
#pragma unroll
    for (int s = 0; s < 4; s += 2) {
      const float a = x[s], b = shx_(x[s + 1], 31);
      x[s] = __fadd_rn(a, b);
      x[s + 1] = __fmul_rn(__fsub_rn(a, b), f);
    }
  }
  lee_split_shfl<32>(x, lane, lee);
  lee_split_shfl<16>(x, lane, lee);
  lee_split_shfl<8>(x, lane, lee);
  lee_split_shfl<4>(x, lane, lee);
  lee_split_shfl<2>(x, lane, lee);
  lee_merge_shfl<2>(x, lane);
  lee_merge_shfl<4>(x, lane);
  lee_merge_shfl<8>(x, lane);
  lee_merge_shfl<16>(x, lane);
  lee_merge_shfl<32>(x, lane);
  const int k = lane >> 1;
  const bool even = (lane & 1) == 0;
  {  // merge 64 on slots (0,1) and (2,3)
#pragma unroll
    for (int s = 0; s < 4; s += 2) {
      const float A = x[s], B = x[s + 1];
      const float a1 = shf_(A, k), a2 = shf_(B, k), a3 = shf_(B, k + 1);
      const float b1 = shf_(A, 16 + k), b2 = shf_(B, 16 + k), b3 = shf_(B, min(17 + k, 31));
      x[s] = even ? a1 : __fadd_rn(a2, a3);
      x[s + 1] = even ? b1 : (lane == 31 ? b2 : __fadd_rn(b2, b3));
    }
  }
  {  // merge 128
    float y[4];
    const float p96 = shf_(x[3], 0);
#pragma unroll
    for (int sp = 0; sp < 4; ++sp) {
      const float A = x[sp >> 1], B = x[2 + (sp >> 1)];
      const int o = 16 * (sp & 1);
      const float r1 = shf_(A, o + k), r2 = shf_(B, o + k);
      float r3 = shf_(B, min(o + k + 1, 31));
      float odd;
      if (sp == 1) {
        r3 = lane == 31 ? p96 : r3;
        odd = __fadd_rn(r2, r3);
      } else if (sp == 3) {
        odd = lane == 31 ? r2 : __fadd_rn(r2, r3);
      } else {
        odd = __fadd_rn(r2, r3);
      }
      y[sp] = even ? r1 : odd;
    }
    const float c0 = __uint_as_float(kDctC0Bits), c1 = __uint_as_float(kDctC1Bits);
    x[0] = __fmul_rn(y[0], lane == 0 ? c0 : c1);
    x[1] = __fmul_rn(y[1], c1);
    x[2] = __fmul_rn(y[2], c1);
    x[3] = __fmul_rn(y[3], c1);
  }
}

template <int M>
__device__ __forceinline__ void lee_merge_t_shfl(float (&x)[4], int lane) {
  constexpr int half = M / 2;
  const int q = lane & (M - 1), base = lane & ~(M - 1), kk = q & (half - 1);
  const bool lo = q < half, k0 = kk == 0;
  const int s1 = base + 2 * kk, s2 = base + 2 * kk + 1, s3 = base + max(2 * kk - 1, 0);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const float v = x[s];
    const float r1 = shf_(v, s1), r2 = shf_(v, s2), r3 = shf_(v, s3);
    x[s] = lo ? r1 : (k0 ? r2 : __fadd_rn(r2, r3));
  }
}
template <int M>
__device__ __forceinline__ void lee_split_t_shfl(float (&x)[4], int lane, const float *lee) {
  constexpr int half = M / 2;
  const int q = lane & (M - 1);
  const bool lo = q < half;
  const int j = lo ? q : M - 1 - q;
  const float f = lee[half - 1 + j];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const float v = x[s];
    const float ra = shx_(v, M - 1), rbl = shx_(v, half), rbh = shx_(v, half - 1);
    const float a = lo ? v : ra;
    const float fb = __fmul_rn(lo ? rbl : rbh, f);
    x[s] = lo ? __fadd_rn(a, fb) : __fsub_rn(a, fb);
  }
}

__device__ __forceinline__ void dct128_inv_shfl(float (&x)[4], int lane, const float *lee) {
  const float c0 = __uint_as_float(kDctC0Bits), c1 = __uint_as_float(kDctC1Bits);
  x[0] = __fmul_rn(x[0], lane == 0 ? c0 : c1);
  x[1] = __fmul_rn(x[1], c1);
  x[2] = __fmul_rn(x[2], c1);
  x[3] = __fmul_rn(x[3], c1);
  const int e = (2 * lane) & 31, o1 = (2 * lane + 1) & 31, o2 = (2 * lane - 1) & 31;
  const bool low16 = lane < 16, le16 = lane <= 16;
  {  // transposed merge 128
    float y[4];
#pragma unroll
    for (int sp = 0; sp < 2; ++sp) {
      const float ra = shf_(x[2 * sp], e), rb = shf_(x[2 * sp + 1], e);
      y[sp] = low16 ? ra : rb;
    }
#pragma unroll
    for (int sp = 2; sp < 4; ++sp) {
      const int slo = 2 * (sp - 2), shi = slo + 1;
      const float r1a = shf_(x[slo], o1), r1b = shf_(x[shi], o1);
      const float p1 = low16 ? r1a : r1b;
      const float r2a = shf_(x[slo], o2), r2b = shf_(x[shi], o2);
      const float r2c = shf_(x[slo > 0 ? slo - 1 : 0], 31);
      const float p2 = lane == 0 ? r2c : (le16 ? r2a : r2b);
      float v = __fadd_rn(p1, p2);
      if (sp == 2) v = lane == 0 ? p1 : v;
      y[sp] = v;
    }
    x[0] = y[0]; x[1] = y[1]; x[2] = y[2]; x[3] = y[3];
  }
  {  // transposed merge 64 on slots (0,1) and (2,3)
#pragma unroll
    for (int s = 0; s < 4; s += 2) {
      const float A = x[s], B = x[s + 1];
      const float ra = shf_(A, e), rb = shf_(B, e);
      const float r1a = shf_(A, o1), r1b = shf_(B, o1);
      const float r2a = shf_(A, o2), r2b = shf_(B, o2);
      const float p1 = low16 ? r1a : r1b, p2 = le16 ? r2a : r2b;
      x[s] = low16 ? ra : rb;
      x[s + 1] = lane == 0 ? p1 : __fadd_rn(p1, p2);
    }
  }
  lee_merge_t_shfl<32>(x, lane);
  lee_merge_t_shfl<16>(x, lane);
  lee_merge_t_shfl<8>(x, lane);
  lee_merge_t_shfl<4>(x, lane);
  lee_merge_t_shfl<2>(x, lane);
  lee_split_t_shfl<2>(x, lane, lee);
  lee_split_t_shfl<4>(x, lane, lee);
  lee_split_t_shfl<8>(x, lane, lee);
  lee_split_t_shfl<16>(x, lane, lee);
  lee_split_t_shfl<32>(x, lane, lee);
  {  // transposed split 64
    const float f = lee[31 + lane];
#pragma unroll
    for (int s = 0; s < 4; s += 2) {
      const float a = x[s], fb = __fmul_rn(x[s + 1], f);
      const float d = __fsub_rn(a, fb);
      x[s] = __fadd_rn(a, fb);
      x[s + 1] = shx_(d, 31);
    }
  }
  {  // transposed split 128
    const float fb0 = __fmul_rn(x[2], lee[63 + lane]), fb1 = __fmul_rn(x[3], lee[95 + lane]);
    const float s0 = __fadd_rn(x[0], fb0), s1 = __fadd_rn(x[1], fb1);
    const float d0 = __fsub_rn(x[0], fb0), d1 = __fsub_rn(x[1], fb1);
    x[0] = s0;
    x[1] = s1;
    x[2] = shx_(d1, 31);
    x[3] = shx_(d0, 31);
  }
}

}  // namespace kvr
