// tree.cu — speculative verification over a draft tree: KV compaction of the accepted path and
// seeded temperature sampling of the verified rows.
//
// The reference verifies a chain of drafts greedily (crates/llama-stage-backend/src/lib.rs:
// 2143-2185: accept while the argmax equals the draft, bonus at the first mismatch).  For a tree
// the same rule walks from the root: the token drawn at a node (argmax, or a temperature sample)
// is accepted if a child carries it.  The tree rows are written to the cache at positions
// prefix .. prefix+n-1; once the path is known its rows move to prefix .. prefix+len(path)-1.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace sfc {

// grid (layer, K|V, kv head); threads copy whole rows (head_dim elements) in 16-byte pieces
__global__ void kv_compact_kernel(uint8_t *__restrict__ arena, int max_sessions, int64_t slot_stride, int slot,
                                  int64_t max_ctx, int head_dim, int elt_bytes, int pos0,
                                  const int32_t *__restrict__ path, int m) {
  pdl_wait();
  pdl_launch_dependents();
  const int layer = blockIdx.x, kvsel = blockIdx.y, head = blockIdx.z;
  const int64_t row_bytes = int64_t(head_dim) * elt_bytes;
  uint8_t *base = arena + ((int64_t(layer) * max_sessions + slot) * slot_stride +
                           int64_t(kvsel) * (slot_stride / 2) + int64_t(head) * max_ctx * head_dim) *
                              elt_bytes;
  const int pieces = int(row_bytes / 16);
  for (int i = 1; i < m; ++i) {  // path[0] is the root: already in place
    const int src = path[i];
    if (src == i) continue;
    const uint4 *s = reinterpret_cast<const uint4 *>(base + int64_t(pos0 + src) * row_bytes);
    uint4 *d = reinterpret_cast<uint4 *>(base + int64_t(pos0 + i) * row_bytes);
    for (int k = threadIdx.x; k < pieces; k += blockDim.x) d[k] = s[k];
  }
}

cudaError_t kv_compact(void *kv_arena, int n_layers, int max_sessions, int64_t slot_stride, int slot, int n_kv,
                       int64_t max_ctx, int head_dim, int elt_bytes, int pos0, const int32_t *path, int m,
                       cudaStream_t st) {
  if (m <= 1 || n_layers <= 0) return cudaSuccess;
  if ((int64_t(head_dim) * elt_bytes) % 16) return cudaErrorInvalidValue;
  return launch_pdl(kv_compact_kernel, dim3(unsigned(n_layers), 2u, unsigned(n_kv)), dim3(128), 0, st,
                    static_cast<uint8_t *>(kv_arena), max_sessions, slot_stride, slot, max_ctx, head_dim, elt_bytes,
                    pos0, path, m);
}

constexpr int SAMPLE_THREADS = 1024;

// One CTA per row.  Thread j owns the contiguous vocabulary segment [j*seg, (j+1)*seg); weights
// are exp((s - max) / T) summed in index order per segment, segment prefixes are summed in order
// by one thread, and the owner of the drawn mass walks its segment.
__global__ void __launch_bounds__(SAMPLE_THREADS) sample_temperature_kernel(const float *__restrict__ scores,
                                                                           int64_t vocab, float temperature,
                                                                           uint64_t seed, int64_t *__restrict__ out) {
  __shared__ float s_max[SAMPLE_THREADS / 32];
  __shared__ float s_seg[SAMPLE_THREADS];
  __shared__ float s_pre[SAMPLE_THREADS];
  __shared__ float s_target;
  __shared__ int64_t s_pick;
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x, tid = threadIdx.x;
  const float *sc = scores + int64_t(row) * vocab;
  const int64_t seg = (vocab + SAMPLE_THREADS - 1) / SAMPLE_THREADS;
  const int64_t lo = int64_t(tid) * seg, hi = lo + seg < vocab ? lo + seg : vocab;
  float m = -INFINITY;
  for (int64_t i = lo; i < hi; ++i) m = fmaxf(m, sc[i]);
  m = warp_max(m);
  if ((tid & 31) == 0) s_max[tid >> 5] = m;
  __syncthreads();
  float mx = -INFINITY;
  for (int w = 0; w < SAMPLE_THREADS / 32; ++w) mx = fmaxf(mx, s_max[w]);
  const float inv_t = 1.0f / temperature;
  float acc = 0.f;
  for (int64_t i = lo; i < hi; ++i) acc += expf((sc[i] - mx) * inv_t);
  s_seg[tid] = acc;
  if (tid == 0) s_pick = -1;
  __syncthreads();
  if (tid == 0) {
    float run = 0.f;
    for (int j = 0; j < SAMPLE_THREADS; ++j) {
      s_pre[j] = run;
      run += s_seg[j];
    }
    const float u = float(mix64(seed, uint64_t(row)) >> 40) * (1.0f / 16777216.0f);  // [0, 1), 24 bits
    s_target = u * run;
  }
  __syncthreads();
  const float target = s_target;
  if (lo < hi && target >= s_pre[tid] && target < s_pre[tid] + s_seg[tid]) {
    float run = s_pre[tid];
    int64_t pick = hi - 1;
    for (int64_t i = lo; i < hi; ++i) {
      run += expf((sc[i] - mx) * inv_t);
      if (run > target) {
        pick = i;
        break;
      }
    }
    s_pick = pick;
  }
  __syncthreads();
  if (tid == 0) {
    int64_t pick = s_pick;
    if (pick < 0) {  // the drawn mass fell past the rounded total: take the last index with weight
      pick = vocab - 1;
      while (pick > 0 && !(sc[pick] > -INFINITY)) --pick;
    }
    out[row] = pick;
  }
}

cudaError_t sample_rows_temperature(const float *scores, int64_t n, int64_t vocab, float temperature, uint64_t seed,
                                    int64_t *out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (vocab <= 0 || !(temperature > 0.f)) return cudaErrorInvalidValue;
  return launch_pdl(sample_temperature_kernel, dim3(unsigned(n)), dim3(SAMPLE_THREADS), 0, st, scores, vocab,
                    temperature, seed, out);
}

}  // namespace sfc
