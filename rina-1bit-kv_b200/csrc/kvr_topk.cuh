// Block-wide exact top-k by MSB radix select over 64-bit composite keys.
//
// key(i) = (float_key(score_i) << 32) | (0xffffffff - i): larger score first,
// then smaller index first.  Keys are unique, so the k largest keys are
// exactly the k entries the (score desc, index asc) rule selects and no tie
// handling is needed.  The select walks the key 8 bits at a time from the
// top and stops as soon as the chosen digit bucket holds exactly the number
// of entries still needed (usually after the 32 score bits, or earlier).
#pragma once

#include "kvr_common.cuh"

namespace kvr {

struct TopkSmem {
  unsigned long long prefix, mask;
  int remaining, bin_count, n_out;
  int hist[256];
};

__device__ __forceinline__ unsigned long long make_key(float s, int64_t i) {
  return ((unsigned long long)float_key(s) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
}
__device__ __forceinline__ int64_t key_index(unsigned long long key) {
  return (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
}
__device__ __forceinline__ float key_score(unsigned long long key) { return key_float((uint32_t)(key >> 32)); }

// score_of(i) -> float for 0 <= i < n (exclusions already mapped to -inf).
// cand: shared array of at least next_pow2(k) keys.  On return (after a
// __syncthreads) cand[0..k) holds the selected keys in descending order.
// Must be called by all NT threads of the block.
template <int NT, typename ScoreFn>
__device__ void block_topk(ScoreFn score_of, int64_t n, int k, unsigned long long *cand, TopkSmem &sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    sm.prefix = 0ull;
    sm.mask = 0ull;
    sm.remaining = k;
    sm.bin_count = -1;
    sm.n_out = 0;
  }
  __syncthreads();
  for (int pass = 0; pass < 8; ++pass) {
    const int shift = 56 - 8 * pass;
    for (int b = tid; b < 256; b += NT) sm.hist[b] = 0;
    __syncthreads();
    const unsigned long long prefix = sm.prefix, mask = sm.mask;
    for (int64_t i = tid; i < n; i += NT) {
      const unsigned long long key = make_key(score_of(i), i);
      if ((key & mask) == prefix) atomicAdd(&sm.hist[(key >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending)
      int c[8], s = 0;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        c[r] = sm.hist[255 - 8 * lane - r];
        s += c[r];
      }
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int excl = incl - s;
      const int rem = sm.remaining;
      if (excl < rem && rem <= incl) {
        int cum = excl;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if (cum + c[r] >= rem) {
            const unsigned long long digit = (unsigned long long)(255 - 8 * lane - r);
            sm.prefix = prefix | (digit << shift);
            sm.mask = mask | (0xffull << shift);
            sm.remaining = rem - cum;
            sm.bin_count = c[r];
            break;
          }
          cum += c[r];
        }
      }
    }
    __syncthreads();
    if (sm.bin_count == sm.remaining) break;
  }
  const unsigned long long prefix = sm.prefix, mask = sm.mask;
  for (int64_t i = tid; i < n; i += NT) {
    const unsigned long long key = make_key(score_of(i), i);
    if ((key & mask) >= prefix) {
      const int slot = atomicAdd(&sm.n_out, 1);
      if (slot < k) cand[slot] = key;
    }
  }
  __syncthreads();
  int P = 1;
  while (P < k) P <<= 1;
  for (int i = k + tid; i < P; i += NT) cand[i] = 0ull;
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P / 2; i += NT) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long a = cand[lo], b = cand[hi];
        if ((a < b) == desc) {
          cand[lo] = b;
          cand[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

}  // namespace kvr
