// Sequence-split exchange over NVLink peer memory (sm_100a), in place of
// the NCCL all-gathers of the candidate lists and of the partial
// attention rows.
//
// Every rank owns one exchange buffer in its own HBM (kvr_peer_alloc) and
// maps the buffers of the other ranks of the node (CUDA IPC handles, passed
// around by the host).  An exchange is one kernel per rank: each CTA writes
// its slice of this rank's data into the same slice of every rank's buffer
// with plain stores (NVLink for the peers), makes them visible system-wide,
// raises its flag in every buffer, waits (bounded) for the flags of every
// rank for its slice, and merges the slice from its own, local buffer.  No
// kernel ever loads from a peer's memory, and no TMA or multicast is used.
//
// Ordering: data stores -> __threadfence_system() by every writer thread ->
// block barrier -> thread 0 stores the flag with release semantics at system
// scope; the waiter polls with acquire loads at system scope, then a block
// barrier orders the CTA's reads after it.  Flags carry the exchange epoch
// (a per-slice counter kept in the local header and advanced by the kernel,
// so the same launch can be replayed from a CUDA graph); data is double
// buffered by epoch parity, which is enough because a rank cannot start
// exchange e+2 before every rank has finished reading exchange e.
//
// Waits are bounded: on timeout the kernel sets the error word of the
// buffer (kvr_workspace_status reads it) and returns; nothing spins forever.
#include <cstring>

#include "kvr_common.cuh"
#include "kvr_topk.cuh"

namespace kvr {

namespace peer {
constexpr int kMaxRanks = 8;
constexpr int kMaxSlices = 64;   // CTAs of one exchange kind
constexpr int kMaxRows = 64;     // candidate rows (batch * kv heads)
constexpr int kMaxK = 64;        // candidates per row and rank
constexpr int kMaxQRows = 1024;  // partial rows (batch * q heads)
constexpr int kRowF = 130;       // [m, l, o_0 .. o_127]
constexpr int kQRowsPerCta = 8;
constexpr uint32_t kPeerSpinLimit = 1u << 20;  // polls (each ~0.1-1 us) before a wait gives up
// header: err word, epochs[2][slices], flags[2][ranks][slices]
constexpr size_t kOffEpoch = 256;
constexpr size_t kOffFlags = kOffEpoch + 2 * kMaxSlices * 4;
constexpr size_t kOffCand = (kOffFlags + 2 * kMaxRanks * kMaxSlices * 4 + 255) / 256 * 256;
constexpr size_t kCandBytes = 2ull * kMaxRanks * kMaxRows * kMaxK * 8;  // [parity][rank][row][k] (score, idx)
constexpr size_t kOffPart = kOffCand + kCandBytes;
constexpr size_t kPartBytes = 2ull * kMaxRanks * kMaxQRows * kRowF * 4;  // [parity][rank][row][130]
constexpr size_t kBytes = kOffPart + kPartBytes;
}  // namespace peer

struct PeerBufs {
  unsigned char *p[peer::kMaxRanks];  // every rank's buffer as mapped here (p[rank] is local)
  int n, rank;
};

__device__ __forceinline__ void st_release_sys(unsigned *addr, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *addr) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ unsigned *peer_flag(unsigned char *base, int kind, int src, int slice) {
  return reinterpret_cast<unsigned *>(base + peer::kOffFlags) + (kind * peer::kMaxRanks + src) * peer::kMaxSlices +
         slice;
}

// Publish this rank's slice to every rank, then wait for every rank's slice.
// Returns false (error word set) if a wait timed out.  Called by all threads.
__device__ bool publish_and_wait(const PeerBufs &pb, int kind, int slice, unsigned epoch) {
  __threadfence_system();
  __syncthreads();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    for (int r = 0; r < pb.n; ++r) st_release_sys(peer_flag(pb.p[r], kind, pb.rank, slice), epoch);
    int ok = 1;
    for (int r = 0; r < pb.n && ok; ++r) {
      const unsigned *f = peer_flag(pb.p[pb.rank], kind, r, slice);
      uint32_t it = 0;
      while ((int)(ld_acquire_sys(f) - epoch) < 0) {
        if (++it > peer::kPeerSpinLimit) {
          ok = 0;
          atomicOr(reinterpret_cast<unsigned *>(pb.p[pb.rank]), 4u);
          break;
        }
        __nanosleep(32);
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// kind 0: candidates.  CTA = one (b, h) row.
__global__ void __launch_bounds__(256) peer_candidates_kernel(PeerBufs pb, const float *__restrict__ scores,
                                                              const int32_t *__restrict__ idx, int rows, int k_local,
                                                              int k_sel, int64_t tile_base, int64_t n_local,
                                                              int32_t *__restrict__ gsel,
                                                              int32_t *__restrict__ lsel) {
  __shared__ unsigned long long keys[peer::kMaxRanks * peer::kMaxK];
  __shared__ int n_valid;
  const int row = blockIdx.x;
  unsigned *epoch_p = reinterpret_cast<unsigned *>(pb.p[pb.rank] + peer::kOffEpoch) + row;
  const unsigned epoch = *epoch_p + 1u;
  const int par = epoch & 1;
  // this rank's candidates of the row -> slot [par][rank][row] of every buffer
  for (int j = threadIdx.x; j < k_local; j += blockDim.x) {
    const float s = scores[(int64_t)row * k_local + j];
    const int32_t t = idx[(int64_t)row * k_local + j];
    const uint2 v = make_uint2(__float_as_uint(s), (unsigned)t);
    for (int r = 0; r < pb.n; ++r) {
      uint2 *dst = reinterpret_cast<uint2 *>(pb.p[r] + peer::kOffCand) +
                   ((size_t)(par * peer::kMaxRanks + pb.rank) * peer::kMaxRows + row) * peer::kMaxK + j;
      *dst = v;
    }
  }
  const bool ok = publish_and_wait(pb, 0, row, epoch);
  if (threadIdx.x == 0) {
    n_valid = 0;
    *epoch_p = epoch;
  }
  __syncthreads();
  const int n = pb.n * k_local;
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    const int r = c / k_local, j = c - r * k_local;
    const uint2 v = *reinterpret_cast<const uint2 *>(pb.p[pb.rank] + peer::kOffCand +
                                                     (((size_t)(par * peer::kMaxRanks + r) * peer::kMaxRows + row) *
                                                          peer::kMaxK + j) * 8);
    const float s = __uint_as_float(v.x);
    const int32_t t = (int32_t)v.y;
    const bool valid = ok && t >= 0 && s > -INFINITY;
    keys[c] = valid ? make_key(s, t) : 0ull;
    if (valid) atomicAdd(&n_valid, 1);
  }
  __syncthreads();
  const int nv = n_valid;
  for (int j = threadIdx.x; j < k_sel; j += blockDim.x)
    if (j >= nv) {
      if (gsel) gsel[(int64_t)row * k_sel + j] = -1;
      lsel[(int64_t)row * k_sel + j] = -1;
    }
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    const unsigned long long kc = keys[c];
    if (kc == 0ull) continue;
    int rank = 0;
    for (int e = 0; e < n; ++e) rank += keys[e] > kc;
    if (rank < k_sel) {
      const int64_t t = key_index(kc);
      if (gsel) gsel[(int64_t)row * k_sel + rank] = (int32_t)t;
      const int64_t loc = t - tile_base;
      lsel[(int64_t)row * k_sel + rank] = (loc >= 0 && loc < n_local) ? (int32_t)loc : -1;
    }
  }
}

// kind 1: partial rows [m, l, o].  CTA = kQRowsPerCta query rows; 8 warps,
// warp w owns row w of the slice: writes it to every rank, then merges it.
__global__ void __launch_bounds__(256) peer_lse_kernel(PeerBufs pb, const float *__restrict__ part, int n_rows,
                                                       void *__restrict__ out, int out_dt) {
  const int slice = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = slice * peer::kQRowsPerCta + warp;
  unsigned *epoch_p = reinterpret_cast<unsigned *>(pb.p[pb.rank] + peer::kOffEpoch) + peer::kMaxSlices + slice;
  const unsigned epoch = *epoch_p + 1u;
  const int par = epoch & 1;
  auto slot = [&](unsigned char *base, int src, int r) {
    return reinterpret_cast<float *>(base + peer::kOffPart) +
           ((size_t)(par * peer::kMaxRanks + src) * peer::kMaxQRows + r) * peer::kRowF;
  };
  if (row < n_rows) {
    const float *src = part + (int64_t)row * peer::kRowF;
    for (int r = 0; r < pb.n; ++r) {
      float *dst = slot(pb.p[r], pb.rank, row);
      for (int i = lane; i < peer::kRowF; i += 32) dst[i] = src[i];
    }
  }
  const bool ok = publish_and_wait(pb, 1, slice, epoch);
  if (threadIdx.x == 0) *epoch_p = epoch;
  if (row >= n_rows) return;
  // log-sum-exp merge of the ranks' rows (same arithmetic as kvr_lse_merge)
  float M = -INFINITY;
  for (int r = 0; r < pb.n; ++r) M = fmaxf(M, ok ? slot(pb.p[pb.rank], r, row)[0] : -INFINITY);
  float L = 0.0f, o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < pb.n && ok; ++r) {
    const float *pr = slot(pb.p[pb.rank], r, row);
    const float m = pr[0];
    const float w = (m == -INFINITY) ? 0.0f : expf(m - M);
    L = fmaf(w, pr[1], L);
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = fmaf(w, pr[2 + lane * 4 + j], o[j]);
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t i = (int64_t)row * 128 + lane * 4 + j;
    if (out_dt == KVR_F32) store_elem<KVR_F32>(out, i, o[j] * inv);
    else if (out_dt == KVR_F16) store_elem<KVR_F16>(out, i, o[j] * inv);
    else store_elem<KVR_BF16>(out, i, o[j] * inv);
  }
}

static int fill_bufs(PeerBufs &pb, void *const *bufs, int n_ranks, int rank) {
  KVR_REQUIRE(n_ranks > 0 && n_ranks <= peer::kMaxRanks && rank >= 0 && rank < n_ranks,
              "peer exchange: 1..%d ranks", peer::kMaxRanks);
  pb.n = n_ranks;
  pb.rank = rank;
  for (int r = 0; r < peer::kMaxRanks; ++r) pb.p[r] = r < n_ranks ? static_cast<unsigned char *>(bufs[r]) : nullptr;
  for (int r = 0; r < n_ranks; ++r) KVR_REQUIRE(bufs[r] != nullptr, "peer exchange: null buffer of rank %d", r);
  return KVR_OK;
}

}  // namespace kvr

using namespace kvr;

extern "C" size_t kvr_peer_buffer_bytes(void) { return peer::kBytes; }

extern "C" int kvr_peer_alloc(void **buf) {
  clear_error();
  KVR_REQUIRE(buf, "kvr_peer_alloc: null out pointer");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, peer::kBytes);
  if (e != cudaSuccess) return set_error(KVR_ECUDA, "kvr_peer_alloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, peer::kBytes);
  if (e != cudaSuccess) return set_error(KVR_ECUDA, "kvr_peer_alloc: %s", cudaGetErrorString(e));
  *buf = p;
  return KVR_OK;
}

extern "C" int kvr_peer_free(void *buf) {
  clear_error();
  if (buf && cudaFree(buf) != cudaSuccess) return check_launch("kvr_peer_free");
  return KVR_OK;
}

extern "C" int kvr_peer_handle(void *buf, void *handle_out) {
  clear_error();
  KVR_REQUIRE(buf && handle_out, "kvr_peer_handle: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, buf);
  if (e != cudaSuccess) return set_error(KVR_ECUDA, "kvr_peer_handle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  return KVR_OK;
}

extern "C" size_t kvr_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int kvr_peer_open(const void *handle, void **buf) {
  clear_error();
  KVR_REQUIRE(handle && buf, "kvr_peer_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(KVR_ECUDA, "kvr_peer_open: %s", cudaGetErrorString(e));
  *buf = p;
  return KVR_OK;
}

extern "C" int kvr_peer_close(void *buf) {
  clear_error();
  if (buf && cudaIpcCloseMemHandle(buf) != cudaSuccess) return check_launch("kvr_peer_close");
  return KVR_OK;
}

extern "C" int kvr_peer_merge_candidates(void *const *bufs, int n_ranks, int rank, const float *scores,
                                         const int32_t *idx, int rows, int k_local, int k_sel, int64_t tile_base,
                                         int64_t n_local, int32_t *global_sel, int32_t *local_sel,
                                         kvr_stream_t stream) {
  clear_error();
  PeerBufs pb{};
  int rc = fill_bufs(pb, bufs, n_ranks, rank);
  if (rc) return rc;
  KVR_REQUIRE(scores && idx && local_sel, "kvr_peer_merge_candidates: null pointer");
  KVR_REQUIRE(rows > 0 && rows <= peer::kMaxRows && k_local > 0 && k_local <= peer::kMaxK && k_sel > 0,
              "kvr_peer_merge_candidates: rows <= %d, k_local <= %d", peer::kMaxRows, peer::kMaxK);
  peer_candidates_kernel<<<rows, 256, 0, as_cuda(stream)>>>(pb, scores, idx, rows, k_local, k_sel, tile_base,
                                                            n_local, global_sel, local_sel);
  return check_launch("kvr_peer_merge_candidates");
}

extern "C" int kvr_peer_lse_merge(void *const *bufs, int n_ranks, int rank, const float *partials, int n_rows, int d,
                                  void *out, int out_dtype, kvr_stream_t stream) {
  clear_error();
  PeerBufs pb{};
  int rc = fill_bufs(pb, bufs, n_ranks, rank);
  if (rc) return rc;
  KVR_REQUIRE(d == 128, "kvr_peer_lse_merge: head_dim must be 128");
  KVR_REQUIRE(partials && out && valid_dtype(out_dtype), "kvr_peer_lse_merge: bad arguments");
  KVR_REQUIRE(n_rows > 0 && n_rows <= peer::kMaxQRows && (n_rows + peer::kQRowsPerCta - 1) / peer::kQRowsPerCta <=
                                                             peer::kMaxSlices,
              "kvr_peer_lse_merge: n_rows <= %d", peer::kMaxQRows);
  const int ctas = (n_rows + peer::kQRowsPerCta - 1) / peer::kQRowsPerCta;
  peer_lse_kernel<<<ctas, 256, 0, as_cuda(stream)>>>(pb, partials, n_rows, out, out_dtype);
  return check_launch("kvr_peer_lse_merge");
}
