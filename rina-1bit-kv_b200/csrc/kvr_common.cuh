// Shared helpers of the kvr_b200 native library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <climits>
#include <cstdio>

#include "kvr_b200.h"

namespace kvr {

// ---------------------------------------------------------------- errors ----
// Sets the calling thread's last-error message and returns `code`.
int set_error(int code, const char *fmt, ...);
void clear_error();

#define KVR_REQUIRE(cond, ...)                              \
  do {                                                      \
    if (!(cond)) return ::kvr::set_error(KVR_EINVAL, __VA_ARGS__); \
  } while (0)

// Checks the launch that was just issued.
int check_launch(const char *what);

inline bool valid_dtype(int dt) { return dt == KVR_F32 || dt == KVR_F16 || dt == KVR_BF16; }
inline size_t dtype_size(int dt) { return dt == KVR_F32 ? 4 : 2; }
inline cudaStream_t as_cuda(kvr_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------- device utils ----
template <int DT>
__device__ __forceinline__ float load_elem(const void *p, int64_t i) {
  if constexpr (DT == KVR_F32) {
    return __ldg(reinterpret_cast<const float *>(p) + i);
  } else if constexpr (DT == KVR_F16) {
    return __half2float(reinterpret_cast<const __half *>(p)[i]);
  } else {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
  }
}

// Loads 4 consecutive elements starting at element i (i must be a multiple of 4
// and the row 8/16-byte aligned) and widens them to fp32 exactly.
template <int DT>
__device__ __forceinline__ void load4(const void *p, int64_t i, float (&x)[4]) {
  if constexpr (DT == KVR_F32) {
    float4 v = __ldg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + i));
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else {
    uint2 u = __ldg(reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(p) + i));
    uint32_t w[2] = {u.x, u.y};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint16_t lo = w[j] & 0xffff, hi = w[j] >> 16;
      if constexpr (DT == KVR_F16) {
        x[2 * j] = __half2float(__ushort_as_half(lo));
        x[2 * j + 1] = __half2float(__ushort_as_half(hi));
      } else {
        x[2 * j] = __bfloat162float(__ushort_as_bfloat16(lo));
        x[2 * j + 1] = __bfloat162float(__ushort_as_bfloat16(hi));
      }
    }
  }
}

template <int DT>
__device__ __forceinline__ void store_elem(void *p, int64_t i, float v) {
  if constexpr (DT == KVR_F32) {
    reinterpret_cast<float *>(p)[i] = v;
  } else if constexpr (DT == KVR_F16) {
    reinterpret_cast<__half *>(p)[i] = __float2half_rn(v);
  } else {
    reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_max_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Order-preserving map float -> uint32 (larger float -> larger key).  NaN maps
// to the key of -inf, -0.0 to the key of +0.0.
__device__ __forceinline__ uint32_t float_key(float f) {
  if (f != f) f = -INFINITY;
  if (f == 0.0f) f = 0.0f;
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// Every workspace starts with the same fixed header, so that no change of
// shapes between calls can move a counter onto stale data:
//   [0, 256)                         error word
//   [kWsSelCounters, +4*kWsMaxRows)  per-(b, h) counters of the selection kernel
//   [kWsAttnCounters, +4*kWsMaxRows) per-(b, h) counters of the attention kernel
// The counters are zero on entry and reset to zero by the kernel that used them.
constexpr int kWsMaxRows = 4096;  // batch * n_kv
constexpr size_t kWsSelCounters = 256;
constexpr size_t kWsAttnCounters = kWsSelCounters + 4 * kWsMaxRows;
constexpr size_t kWsHeader = kWsAttnCounters + 4 * kWsMaxRows;

// Optional phase timestamps for latency studies (compiled only with -DKVR_TRACE).
#ifdef KVR_TRACE
static __device__ unsigned long long g_kvr_trace[1 << 16];  // one copy per translation unit
__device__ __forceinline__ void kvr_trace(int kernel, int point) {
  if (threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const unsigned blk = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (blk < 2048) g_kvr_trace[(kernel * 2048 + blk) * 8 + point] = t;
  }
}
#define KVR_TRACE_POINT(k, p) ::kvr::kvr_trace(k, p)
#else
#define KVR_TRACE_POINT(k, p) ((void)0)
#endif

// Bound on device-side spin iterations (each iteration also sleeps ~64 ns).
constexpr uint32_t kSpinLimit = 1u << 22;

// One element as fp32.
template <int DT>
__device__ __forceinline__ float load1(const void *p, int64_t i) {
  if constexpr (DT == KVR_F32) return __ldg(reinterpret_cast<const float *>(p) + i);
  else if constexpr (DT == KVR_F16) return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(p) + i)));
  else return __bfloat162float(__ushort_as_bfloat16(__ldg(reinterpret_cast<const unsigned short *>(p) + i)));
}

// Raw 4-element load (16 bytes for fp32, 8 bytes for 16-bit types) and its
// widening to fp32; split so that many loads can be in flight at once.
__device__ __forceinline__ uint4 raw4(const void *p, int64_t i, int dt) {
  if (dt == KVR_F32) return __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const float *>(p) + i));
  const uint2 u = __ldg(reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(p) + i));
  return make_uint4(u.x, u.y, 0u, 0u);
}
__device__ __forceinline__ float4 cvt4(uint4 r, int dt) {
  if (dt == KVR_F32) return make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z),
                                        __uint_as_float(r.w));
  if (dt == KVR_F16) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&r.x));
    const float2 c = __half22float2(*reinterpret_cast<const __half2 *>(&r.y));
    return make_float4(a.x, a.y, c.x, c.y);
  }
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r.x));
  const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r.y));
  return make_float4(a.x, a.y, c.x, c.y);
}

// Programmatic dependent launch: wait for the preceding grid (a no-op when
// the kernel was not launched as a dependent), and let dependents start.
// Exact K/V segments (fp16 rows of kD channels: the window ring and the
// pending tail) of every (b, h) row, for a kernel that stages them in L2
// ahead of the attention kernel that reads them.
struct RowPrefetch {
  const uint16_t *k[2], *v[2];
  int64_t n[2], batch_stride[2], tok_stride;
};

// RoPE with the rotate_half convention in the arithmetic of an eager model
// in dtype DT (modules/kvr_generator.py:91-94).
template <int DT>
__device__ __forceinline__ float round_dt(float x) {
  if constexpr (DT == KVR_F32) return x;
  else if constexpr (DT == KVR_F16) return __half2float(__float2half_rn(x));
  else return __bfloat162float(__float2bfloat16_rn(x));
}

// x * c + rotate_half(x) * s with each op rounded to DT; x_i and its partner
// x_p (i +/- d/2) are the DT values, c and s the table entries rounded to DT.
template <int DT>
__device__ __forceinline__ float rope_elem(float x, float partner, bool low_half, float c, float s) {
  const float cr = round_dt<DT>(c), sr = round_dt<DT>(s);
  const float rh = low_half ? -partner : partner;
  const float a = round_dt<DT>(__fmul_rn(x, cr));
  const float b = round_dt<DT>(__fmul_rn(rh, sr));
  return round_dt<DT>(__fadd_rn(a, b));
}

// Eight consecutive elements of a row in dtype DT, as fp32 (16-byte loads and
// stores; the address must be 16-byte aligned).
constexpr int kChunk8 = 8;

template <int DT>
__device__ __forceinline__ void load8(const void *base, int64_t i, float (&x)[kChunk8]) {
  if constexpr (DT == KVR_F32) {
    const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + i);
    const float4 u = p[0], w = p[1];
    x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
    x[4] = w.x; x[5] = w.y; x[6] = w.z; x[7] = w.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + i);
    const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint16_t lo = (uint16_t)(wd[j] & 0xffffu), hi = (uint16_t)(wd[j] >> 16);
      if constexpr (DT == KVR_F16) {
        x[2 * j] = __half2float(__ushort_as_half(lo));
        x[2 * j + 1] = __half2float(__ushort_as_half(hi));
      } else {
        x[2 * j] = __bfloat162float(__ushort_as_bfloat16(lo));
        x[2 * j + 1] = __bfloat162float(__ushort_as_bfloat16(hi));
      }
    }
  }
}

template <int DT>
__device__ __forceinline__ uint16_t bits_dt(float x) {
  if constexpr (DT == KVR_F16) return __half_as_ushort(__float2half_rn(x));
  else return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

template <int DT>
__device__ __forceinline__ void store8(void *base, int64_t i, const float (&x)[kChunk8]) {
  if constexpr (DT == KVR_F32) {
    float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(base) + i);
    p[0] = make_float4(x[0], x[1], x[2], x[3]);
    p[1] = make_float4(x[4], x[5], x[6], x[7]);
  } else {
    uint32_t wd[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) wd[j] = (uint32_t)bits_dt<DT>(x[2 * j]) | ((uint32_t)bits_dt<DT>(x[2 * j + 1]) << 16);
    *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(base) + i) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
}

__device__ __forceinline__ uint4 pack_f16x8(const float (&x)[kChunk8]) {
  uint32_t wd[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    wd[j] = (uint32_t)bits_dt<KVR_F16>(x[2 * j]) | ((uint32_t)bits_dt<KVR_F16>(x[2 * j + 1]) << 16);
  return make_uint4(wd[0], wd[1], wd[2], wd[3]);
}

// The per-layer store update fused into the batch-1 decode step (host side):
// the new token's pre-RoPE k and v rows (n_kv x 128, q's dtype), the RoPE
// table rows of its position, the window slot it lands in, the tail row the
// slot's old row moves to (-1: none) and an optional output for rotated q.
struct Sd1StepUpdate {
  const void *k_new, *v_new;
  const float *cos_row, *sin_row;
  void *q_out;
  int64_t slot, evict_row;
};

// L2 prefetch of `bytes` (a multiple of 16) at a 16-byte aligned address: a
// hint only, nothing is read into the CTA, so it may run before a grid
// dependency wait on data the previous kernel still writes.
__device__ __forceinline__ void prefetch_l2(const void *p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- mbarrier + bulk copy (PTX)
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned phase) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Bounded wait; returns false if it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned phase, uint32_t limit = kSpinLimit) {
  for (uint32_t it = 0; it < limit; ++it) {
    if (mbar_try_wait(bar, phase)) return true;
    __nanosleep(64);
  }
  return false;
}



}  // namespace kvr
