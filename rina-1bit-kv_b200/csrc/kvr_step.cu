// Per-layer decode store update, fused (sm_100a): what one decode step of
// modules/kvr_generator.py:78-98 does between the q/k/v projections and the
// attention, in one launch:
//   * RoPE of q and k at the step position (rotate_half, kvr_retrieval.py:27-33),
//     every elementwise op rounded to the model dtype the way the eager
//     reference computes it (cos/sin rounded to the dtype, q*c, rot(q)*s and
//     their sum each rounded);
//   * eviction when the window is full (kvr_hook.py:136-148): the slot about
//     to be overwritten moves into the 1-bit store's pending tail; its K is
//     already post-RoPE at the evicted token's own position, so the row is
//     copied as it is (the reference un-rotates it and the 1-bit append
//     rotates it back at the same position);
//   * the window ring write of the new post-RoPE K and V (kvr_window.py:19-25),
//     in fp16.
// One CTA; the evicted row is read before the new row overwrites its slot.
// write_kv = 0 only rotates q (the generator's first step, whose token is
// already in the window from the prefill).
#include "kvr_common.cuh"

namespace kvr {

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

template <int DT>
__global__ void __launch_bounds__(256) decode_store_update_kernel(
    const void *__restrict__ q, const void *__restrict__ k, const void *__restrict__ v, int n_q, int n_kv,
    const float *__restrict__ cos_row, const float *__restrict__ sin_row, void *__restrict__ q_out,
    uint16_t *__restrict__ win_k, uint16_t *__restrict__ win_v, int64_t slot, uint16_t *__restrict__ tail_k,
    uint16_t *__restrict__ tail_v, int64_t tail_row, int write_kv) {
  constexpr int d = 128, h2 = d / 2;
  const int row_elems = n_kv * d;
  // 1. eviction: the slot's fp16 K/V rows move to the tail
  if (tail_k != nullptr) {
    const uint4 *sk = reinterpret_cast<const uint4 *>(win_k + slot * row_elems);
    const uint4 *sv = reinterpret_cast<const uint4 *>(win_v + slot * row_elems);
    uint4 *dk = reinterpret_cast<uint4 *>(tail_k + tail_row * row_elems);
    uint4 *dv = reinterpret_cast<uint4 *>(tail_v + tail_row * row_elems);
    for (int i = threadIdx.x; i < row_elems / 8; i += blockDim.x) {
      dk[i] = sk[i];
      dv[i] = sv[i];
    }
    __syncthreads();
  }
  // 2. q: RoPE in the model dtype
  for (int i = threadIdx.x; i < n_q * d; i += blockDim.x) {
    const int c = i & (d - 1);
    const bool lo = c < h2;
    const float x = load1<DT>(q, i), p = load1<DT>(q, lo ? i + h2 : i - h2);
    store_elem<DT>(q_out, i, rope_elem<DT>(x, p, lo, __ldg(cos_row + c), __ldg(sin_row + c)));
  }
  // 3. k, v: RoPE'd K and V into the window slot, as fp16
  for (int i = threadIdx.x; write_kv && i < row_elems; i += blockDim.x) {
    const int c = i & (d - 1);
    const bool lo = c < h2;
    const float x = load1<DT>(k, i), p = load1<DT>(k, lo ? i + h2 : i - h2);
    const float kr = rope_elem<DT>(x, p, lo, __ldg(cos_row + c), __ldg(sin_row + c));
    win_k[slot * row_elems + i] = __half_as_ushort(__float2half_rn(kr));
    win_v[slot * row_elems + i] = __half_as_ushort(__float2half_rn(load1<DT>(v, i)));
  }
}

}  // namespace kvr

using namespace kvr;

extern "C" int kvr_decode_store_update(const void *q, const void *k, const void *v, int dtype, int n_q, int n_kv,
                                       int d, const float *cos_tbl, const float *sin_tbl, int64_t rope_stride,
                                       int64_t pos, void *q_out, uint16_t *win_k, uint16_t *win_v, int64_t win_cap,
                                       int64_t slot, uint16_t *tail_k, uint16_t *tail_v, int64_t tail_row,
                                       int write_kv, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(d == 128, "kvr_decode_store_update: head_dim must be 128");
  KVR_REQUIRE(valid_dtype(dtype), "kvr_decode_store_update: bad dtype");
  KVR_REQUIRE(q && k && v && cos_tbl && sin_tbl && q_out && win_k && win_v, "kvr_decode_store_update: null pointer");
  KVR_REQUIRE(n_kv > 0 && n_q > 0 && n_q % n_kv == 0, "kvr_decode_store_update: bad head counts");
  KVR_REQUIRE(slot >= 0 && slot < win_cap && pos >= 0 && rope_stride >= d, "kvr_decode_store_update: bad slot/pos");
  KVR_REQUIRE((tail_k == nullptr) == (tail_v == nullptr) && (tail_k == nullptr || tail_row >= 0),
              "kvr_decode_store_update: bad tail");
  KVR_REQUIRE(((reinterpret_cast<uintptr_t>(win_k) | reinterpret_cast<uintptr_t>(win_v) |
                reinterpret_cast<uintptr_t>(tail_k) | reinterpret_cast<uintptr_t>(tail_v)) & 15) == 0,
              "kvr_decode_store_update: window/tail buffers must be 16-byte aligned");
  const float *cr = cos_tbl + pos * rope_stride, *sr = sin_tbl + pos * rope_stride;
  cudaStream_t st = as_cuda(stream);
  if (dtype == KVR_F32)
    decode_store_update_kernel<KVR_F32><<<1, 256, 0, st>>>(q, k, v, n_q, n_kv, cr, sr, q_out, win_k, win_v, slot,
                                                           tail_k, tail_v, tail_row, write_kv);
  else if (dtype == KVR_F16)
    decode_store_update_kernel<KVR_F16><<<1, 256, 0, st>>>(q, k, v, n_q, n_kv, cr, sr, q_out, win_k, win_v, slot,
                                                           tail_k, tail_v, tail_row, write_kv);
  else
    decode_store_update_kernel<KVR_BF16><<<1, 256, 0, st>>>(q, k, v, n_q, n_kv, cr, sr, q_out, win_k, win_v, slot,
                                                            tail_k, tail_v, tail_row, write_kv);
  return check_launch("kvr_decode_store_update");
}
