// Sequence split across GPUs: merge of the gathered per-rank tile candidates
// into the global top-k (sm_100a).
//
// Each rank scores the tiles it owns and keeps its local top k per (b, h)
// row; after the all-gather every rank holds N lists of k (score, global tile
// index) pairs per row.  The global top k is contained in their union, so the
// exact global selection is the k largest composite keys
//   key = (float_key(score) << 32) | (0xffffffff - tile)
// i.e. score descending, then tile index ascending — the same rule the
// one-GPU selection uses.  One CTA per row; each thread ranks its candidates
// by counting larger keys (at most a few thousand candidates per row), so the
// kernel needs no sort and no scratch.  It also writes the slice of the
// selection this rank owns as local tile indices (-1 elsewhere), which the
// partial attention consumes directly.
#include "kvr_common.cuh"
#include "kvr_topk.cuh"

namespace kvr {

constexpr int kMergeThreads = 256;
constexpr int kMergeMaxCand = 4096;

__global__ void __launch_bounds__(kMergeThreads) merge_candidates_kernel(
    const float *__restrict__ scores, const int32_t *__restrict__ idx, int n_ranks, int rows, int k_local, int k_sel,
    int64_t tile_base, int64_t n_local, int32_t *__restrict__ gsel, int32_t *__restrict__ lsel) {
  __shared__ unsigned long long keys[kMergeMaxCand];
  __shared__ int n_valid;
  const int row = blockIdx.x;
  const int n = n_ranks * k_local;
  if (threadIdx.x == 0) n_valid = 0;
  __syncthreads();
  // candidate c = (rank r, slot j): scores[(r * rows + row) * k_local + j]
  for (int c = threadIdx.x; c < n; c += kMergeThreads) {
    const int r = c / k_local, j = c - r * k_local;
    const int64_t o = ((int64_t)r * rows + row) * k_local + j;
    const float s = scores[o];
    const int32_t t = idx[o];
    const bool ok = t >= 0 && s > -INFINITY;  // NaN and -inf compare false: not a candidate
    keys[c] = ok ? make_key(s, t) : 0ull;
    if (ok) atomicAdd(&n_valid, 1);
  }
  __syncthreads();
  const int nv = n_valid;
  for (int j = threadIdx.x; j < k_sel; j += kMergeThreads) {
    if (j >= nv) {
      if (gsel) gsel[(int64_t)row * k_sel + j] = -1;
      lsel[(int64_t)row * k_sel + j] = -1;
    }
  }
  for (int c = threadIdx.x; c < n; c += kMergeThreads) {
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

}  // namespace kvr

using namespace kvr;

extern "C" int kvr_merge_candidates(const float *scores, const int32_t *idx, int n_ranks, int rows, int k_local,
                                    int k_sel, int64_t tile_base, int64_t n_local, int32_t *global_sel,
                                    int32_t *local_sel, kvr_stream_t stream) {
  clear_error();
  KVR_REQUIRE(scores && idx && local_sel, "kvr_merge_candidates: null pointer");
  KVR_REQUIRE(n_ranks > 0 && rows >= 0 && k_local > 0 && k_sel > 0, "kvr_merge_candidates: bad sizes");
  KVR_REQUIRE((int64_t)n_ranks * k_local <= kMergeMaxCand, "kvr_merge_candidates: more than %d candidates per row",
              kMergeMaxCand);
  KVR_REQUIRE(tile_base >= 0 && n_local >= 0 && tile_base + n_local < 0xffffffffll, "kvr_merge_candidates: bad tile range");
  if (rows == 0) return KVR_OK;
  merge_candidates_kernel<<<rows, kMergeThreads, 0, as_cuda(stream)>>>(scores, idx, n_ranks, rows, k_local, k_sel,
                                                                       tile_base, n_local, global_sel, local_sel);
  return check_launch("kvr_merge_candidates");
}
