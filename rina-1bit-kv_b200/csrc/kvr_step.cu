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
// One thread per 8-channel chunk of a head row (n_q x 16 chunks of q, then
// n_kv x 16 chunks of k/v), so every thread makes one round trip to memory:
// its vector loads are issued together.  The thread that owns a window-slot
// chunk reads the old (evicted) chunk before it writes the new one.
// Launched as a programmatic dependent: it waits for the previous kernel
// (griddepcontrol.wait) before touching memory, then lets the next kernel
// start.  The next kernel may only read, before its own wait, what this
// kernel does not write: the 1-bit store's tiles (the one-kernel decode step
// stages those early, and the window rows and q only after its wait).
// write_kv = 0 only rotates q (the generator's first step, whose token is
// already in the window from the prefill).
#include "kvr_common.cuh"

namespace kvr {

template <int DT>
__global__ void __launch_bounds__(128) decode_store_update_kernel(
    const void *__restrict__ q, const void *__restrict__ k, const void *__restrict__ v, int n_q, int n_kv,
    const float *__restrict__ cos_row, const float *__restrict__ sin_row, void *__restrict__ q_out,
    uint16_t *__restrict__ win_k, uint16_t *__restrict__ win_v, int64_t slot, uint16_t *__restrict__ tail_k,
    uint16_t *__restrict__ tail_v, int64_t tail_row, int write_kv) {
  constexpr int d = 128, cpr = d / kChunk8;  // 16 chunks per head row
  griddep_wait();
  asm volatile("griddepcontrol.launch_dependents;");
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const bool is_q = t < n_q * cpr;
  if (!is_q && (t >= (n_q + n_kv) * cpr || (!write_kv && tail_k == nullptr))) return;
  const int u = is_q ? t : t - n_q * cpr;  // chunk index within q or within the k/v row
  const int head = u / cpr, cc = u % cpr;
  const int pc = (cc + cpr / 2) % cpr;     // the rotate_half partner chunk
  const bool lo = cc < cpr / 2;
  const int64_t off = (int64_t)head * d + cc * kChunk8, poff = (int64_t)head * d + pc * kChunk8;
  const void *src = is_q ? q : k;
  float x[kChunk8], p[kChunk8], c[kChunk8], s[kChunk8], vv[kChunk8];
  load8<DT>(src, off, x);
  load8<DT>(src, poff, p);
  load8<KVR_F32>(cos_row, cc * kChunk8, c);
  load8<KVR_F32>(sin_row, cc * kChunk8, s);
  uint4 old_k, old_v;
  const int64_t row_elems = (int64_t)n_kv * d;
  uint4 *wk = nullptr, *wv = nullptr;
  if (!is_q) {
    load8<DT>(v, off, vv);
    wk = reinterpret_cast<uint4 *>(win_k + slot * row_elems + off);
    wv = reinterpret_cast<uint4 *>(win_v + slot * row_elems + off);
    if (tail_k != nullptr) {
      old_k = *wk;
      old_v = *wv;
    }
  }
  float r[kChunk8];
#pragma unroll
  for (int e = 0; e < kChunk8; ++e) r[e] = rope_elem<DT>(x[e], p[e], lo, c[e], s[e]);
  if (is_q) {
    store8<DT>(q_out, off, r);
    return;
  }
  // eviction: the slot's fp16 K/V chunk moves to the tail, then the new one lands
  if (tail_k != nullptr) {
    *reinterpret_cast<uint4 *>(tail_k + tail_row * row_elems + off) = old_k;
    *reinterpret_cast<uint4 *>(tail_v + tail_row * row_elems + off) = old_v;
  }
  if (write_kv) {
    *wk = pack_f16x8(r);
    *wv = pack_f16x8(vv);
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
                reinterpret_cast<uintptr_t>(tail_k) | reinterpret_cast<uintptr_t>(tail_v) |
                reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                reinterpret_cast<uintptr_t>(q_out) | reinterpret_cast<uintptr_t>(cos_tbl) |
                reinterpret_cast<uintptr_t>(sin_tbl)) & 15) == 0 && rope_stride % 4 == 0,
              "kvr_decode_store_update: buffers must be 16-byte aligned (and the table row stride a multiple of 4)");
  const float *cr = cos_tbl + pos * rope_stride, *sr = sin_tbl + pos * rope_stride;
  cudaStream_t st = as_cuda(stream);
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)(((n_q + n_kv) * (d / kChunk8) + 127) / 128));
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dtype == KVR_F32)
    cudaLaunchKernelEx(&cfg, decode_store_update_kernel<KVR_F32>, q, k, v, n_q, n_kv, cr, sr, q_out, win_k,
                       win_v, slot, tail_k, tail_v, tail_row, write_kv);
  else if (dtype == KVR_F16)
    cudaLaunchKernelEx(&cfg, decode_store_update_kernel<KVR_F16>, q, k, v, n_q, n_kv, cr, sr, q_out, win_k,
                       win_v, slot, tail_k, tail_v, tail_row, write_kv);
  else
    cudaLaunchKernelEx(&cfg, decode_store_update_kernel<KVR_BF16>, q, k, v, n_q, n_kv, cr, sr, q_out, win_k,
                       win_v, slot, tail_k, tail_v, tail_row, write_kv);
  return check_launch("kvr_decode_store_update");
}
