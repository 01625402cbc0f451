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
  unsigned long long prefix, mask, result;
  int remaining, bin_count, n_out;
  int hist[256];
  unsigned long long lists[512];  // per-warp top-32 lists (up to 16 warps)
};

__device__ __forceinline__ unsigned long long make_key(float s, int64_t i) {
  return ((unsigned long long)float_key(s) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
}
__device__ __forceinline__ int64_t key_index(unsigned long long key) {
  return (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
}
__device__ __forceinline__ float key_score(unsigned long long key) { return key_float((uint32_t)(key >> 32)); }

// The m-th largest key (1 <= m <= n) of the n entries: the same MSB-first
// digit walk as block_topk, stopping as soon as the chosen bin holds a single
// key (or after all 64 bits).  Must be called by all NT threads; every
// thread gets the result.
template <int NT, typename ScoreFn>
__device__ unsigned long long block_kth_largest(ScoreFn score_of, int64_t n, int m, TopkSmem &sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    sm.prefix = 0ull;
    sm.mask = 0ull;
    sm.remaining = m;
    sm.bin_count = -1;
  }
  for (int b = tid; b < 256; b += NT) sm.hist[b] = 0;
  __syncthreads();
  int pass = 0;
  for (; pass < 8; ++pass) {
    const int shift = 56 - 8 * pass;
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
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int excl = incl - s;
      const int rem = sm.remaining;
      __syncwarp();
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
#pragma unroll
      for (int r = 0; r < 8; ++r) sm.hist[8 * lane + r] = 0;  // ready for the next pass
    }
    __syncthreads();
    if (sm.bin_count == 1) break;
  }
  if (pass == 8) return sm.prefix;  // all 64 bits fixed
  const unsigned long long prefix = sm.prefix, mask = sm.mask;
  for (int64_t i = tid; i < n; i += NT) {
    const unsigned long long key = make_key(score_of(i), i);
    if ((key & mask) == prefix) sm.result = key;  // exactly one entry matches
  }
  __syncthreads();
  return sm.result;
}

// key_of(i) -> the unique 64-bit key of entry i (0 <= i < n); the k largest
// keys are selected.  cand: shared array of at least next_pow2(k) keys.  On
// return (after a __syncthreads) cand[0..k) holds them in descending order.
// Must be called by all NT threads of the block.
template <int NT, typename KeyFn>
__device__ void block_topk_keys(KeyFn key_of, int64_t n, int k, unsigned long long *cand, TopkSmem &sm) {
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
      const unsigned long long key = key_of(i);
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
  for (int64_t base = 0; base < n; base += NT) {
    const int64_t i = base + tid;
    unsigned long long key = 0ull;
    bool take = false;
    if (i < n) {
      key = key_of(i);
      take = (key & mask) >= prefix;
    }
    // one atomic per warp for the slots of its selected keys
    const unsigned ballot = __ballot_sync(0xffffffffu, take);
    int first = 0;
    if (ballot && lane == __ffs(ballot) - 1) first = atomicAdd(&sm.n_out, __popc(ballot));
    first = __shfl_sync(0xffffffffu, first, __ffs(ballot ? ballot : 1u) - 1);
    if (take) {
      const int slot = first + __popc(ballot & ((1u << lane) - 1u));
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

// score_of(i) -> float for 0 <= i < n (exclusions already mapped to -inf);
// keys (score, ~index): score descending, then index ascending.
template <int NT, typename ScoreFn>
__device__ void block_topk(ScoreFn score_of, int64_t n, int k, unsigned long long *cand, TopkSmem &sm) {
  block_topk_keys<NT>([&](int64_t i) -> unsigned long long { return make_key(score_of(i), i); }, n, k, cand, sm);
}

// Top-k (k <= 32) of a row held in shared memory by warp-level bitonic
// networks: each warp keeps a descending top-32 list in registers (one key
// per lane) and folds in its slice 32 keys at a time (sort the new keys,
// max against the reversed list, bitonic merge); warp 0 then folds the
// other warps' lists.  One block barrier; no shared-memory atomics.
// row_s: n scores; lists: 32 * (NT/32) keys of scratch; cand: >= k keys.
__device__ __forceinline__ unsigned long long warp_bitonic_merge_desc(unsigned long long key, int lane) {
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, stride);
    const bool lower = (lane & stride) == 0;
    key = lower ? (key > other ? key : other) : (key < other ? key : other);
  }
  return key;
}
__device__ __forceinline__ unsigned long long warp_sort_desc(unsigned long long key, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, stride);
      const bool keep_max = ((lane & stride) == 0) == ((lane & size) == 0 || size == 32);
      key = keep_max ? (key > other ? key : other) : (key < other ? key : other);
    }
  }
  return key;
}
// list and incoming both descending; returns the descending top 32 of the union
__device__ __forceinline__ unsigned long long warp_fold_top32(unsigned long long list, unsigned long long sorted_new,
                                                             int lane) {
  const unsigned long long rev = __shfl_sync(0xffffffffu, sorted_new, 31 - lane);
  return warp_bitonic_merge_desc(list > rev ? list : rev, lane);
}

template <int NT>
__device__ void block_topk_warp32(const float *row_s, int64_t n, int k, unsigned long long *lists,
                                  unsigned long long *cand) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t per = ((n + NW - 1) / NW + 31) / 32 * 32;  // slice per warp, multiple of 32
  unsigned long long list = 0ull;
  for (int64_t c0 = warp * per; c0 < (warp + 1) * per && c0 < n; c0 += 32) {
    const int64_t i = c0 + lane;
    const unsigned long long key = i < n ? make_key(row_s[i], i) : 0ull;
    list = warp_fold_top32(list, warp_sort_desc(key, lane), lane);
  }
  lists[warp * 32 + lane] = list;
  __syncthreads();
  // tree: in round s, warp w (w % 2s == 0) folds in the list of warp w + s
  for (int s = 1; s < NW; s <<= 1) {
    if ((warp % (2 * s)) == 0 && warp + s < NW) {
      const unsigned long long other = lists[(warp + s) * 32 + (31 - lane)];  // reversed: ascending
      list = warp_bitonic_merge_desc(list > other ? list : other, lane);
      lists[warp * 32 + lane] = list;
    }
    __syncthreads();
  }
  if (warp == 0 && lane < k) cand[lane] = list;
  __syncthreads();
}

}  // namespace kvr
