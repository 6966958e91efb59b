// noalloc.cu — logits + softcap + argmax for callers that cannot allocate device memory.
//
// sfc_logits_argmax keeps its per-CTA partial results in a scratch buffer that it allocates
// with cudaMalloc the first time it needs one.  Some callers cannot let a library do that:
// serving processes whose device memory is reserved up front by their own allocator or budget,
// where a stray cudaMalloc either fails or fragments the reservation (and synchronizes the
// device), and hosts that hand the library only the buffers they own.  sfc_logits_argmax_noalloc
// computes the same result with its scratch in a fixed array that belongs to this library and is
// sized at load time.
#include <cuda_runtime.h>

#include <mutex>

#include "capi_common.h"
#include "common.cuh"
#include "kernels.h"

namespace sfc {

// Scratch for the per-CTA (score, index) partials of the no-alloc logits path.  64 KiB covers
// 2 CTAs per SM x 4 tokens per pass (or 4 CTAs per SM x 1 token) x 16 bytes on GPUs with up to
// 512 SMs.  Every GPU that loads
// the library holds this array until the process exits.
constexpr size_t NOALLOC_SCRATCH_BYTES = 64 * 1024;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch, looked up once per device with that device current.
// (In host code the symbol itself is only a host-side stand-in, not a device address.)  The
// cached address stays valid while the device's context does; after a cudaDeviceReset by the
// host process the module is loaded again and the address may differ, so the entry point's
// contract excludes calls on a device after it has been reset.
static std::mutex g_noalloc_mu;
static void *g_noalloc_ptr[64] = {};

static int noalloc_scratch(void **out) {
  int dev = 0;
  SFC_CUDA(cudaGetDevice(&dev));
  SFC_REQUIRE(dev >= 0 && dev < 64, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SFC_OK;
}

}  // namespace sfc

using namespace sfc;

extern "C" int sfc_logits_argmax_noalloc(int ggml_type, const void *w_dev, int64_t vocab, int64_t dim,
                                         const float *h_dev, int64_t n_tok, float cap, float *all_scores_dev,
                                         int64_t *argmax_dev, float *score_dev, void *stream) {
  clear_error();
  SFC_REQUIRE(ggml_type == T_F16 || ggml_type == T_F32 || ggml_type == T_BF16,
              "logits support F16/F32/BF16 tables, got %d", ggml_type);
  SFC_REQUIRE(vocab > 0 && dim > 0 && n_tok >= 0, "bad shape");
  SFC_REQUIRE(w_dev && h_dev && argmax_dev && score_dev, "null pointer");
  const size_t need = logits_scratch_bytes(n_tok);
  if (need > NOALLOC_SCRATCH_BYTES) {
    set_error("sfc_logits_argmax_noalloc needs %zu scratch bytes on this GPU but its fixed array holds %zu", need,
              NOALLOC_SCRATCH_BYTES);
    return SFC_E_NOMEM;
  }
  void *scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  SFC_CUDA(logits_argmax(ggml_type, w_dev, vocab, int(dim), h_dev, n_tok, cap, all_scores_dev, argmax_dev, score_dev,
                         scratch, NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream)));
  return SFC_OK;
}
