// ref_mmvq.cu — the reference's own GPU GEMV (vendor/llama.cpp/ggml/src/ggml-cuda/mmvq.cu, with the
// activation quantizer of quantize.cu), built for sm_100a from the reference tree as a comparator
// for the stage GEMV: same GGUF Q4_K / Q6_K rows, same activations, timed on the same B200.
//
// Test infrastructure, like the rest of oracle/: only tests/ call it, never the product path.
// oracle/Makefile compiles this file with -I pointing into the reference checkout; the two
// reference .cu files are included from there (nothing of theirs is copied into this repository).
// What is defined here is the small host surface those files link against on this call path:
// the device table (filled as ggml-cuda.cu does for NVIDIA devices: cc = 100*major + 10*minor),
// device get/set, and error reporting; the ggml-tensor helpers used only by the ggml-tensor entry
// point (ggml_cuda_mul_mat_vec_q, not called here) abort if reached.
#include "ggml-cuda/mmvq.cu"
#include "ggml-cuda/quantize.cu"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>

// ---------------------------------------------------------------- host surface
const ggml_cuda_device_info &ggml_cuda_info() {
  static ggml_cuda_device_info info = {};
  static std::once_flag once;
  std::call_once(once, [] {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
    info.device_count = n < GGML_CUDA_MAX_DEVICES ? n : GGML_CUDA_MAX_DEVICES;
    for (int id = 0; id < info.device_count; ++id) {
      cudaDeviceProp prop;
      if (cudaGetDeviceProperties(&prop, id) != cudaSuccess) continue;
      info.devices[id].cc = 100 * prop.major + 10 * prop.minor;
      info.devices[id].nsm = prop.multiProcessorCount;
      info.devices[id].smpb = prop.sharedMemPerBlock;
      info.devices[id].smpbo = prop.sharedMemPerBlockOptin;
      info.devices[id].warp_size = prop.warpSize;
      info.devices[id].total_vram = prop.totalGlobalMem;
    }
  });
  return info;
}

int ggml_cuda_get_device() {
  int id = 0;
  cudaGetDevice(&id);
  return id;
}

void ggml_cuda_set_device(int device) { cudaSetDevice(device); }

[[noreturn]] void ggml_cuda_error(const char *stmt, const char *func, const char *file, int line, const char *msg) {
  fprintf(stderr, "comparator: CUDA error %s in %s (%s:%d): %s\n", msg, func, file, line, stmt);
  abort();
}

extern "C" [[noreturn]] void ggml_abort(const char *file, int line, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  fprintf(stderr, "comparator: abort at %s:%d: ", file, line);
  vfprintf(stderr, fmt, ap);
  va_end(ap);
  fprintf(stderr, "\n");
  abort();
}

[[noreturn]] static void off_path(const char *what) {
  fprintf(stderr, "comparator: %s is not on the comparator's call path\n", what);
  abort();
}

std::unique_ptr<ggml_cuda_pool> ggml_backend_cuda_context::new_pool_for_device(int, int) { off_path("pool"); }
extern "C" {
// block geometry of the types this comparator passes (GGUF format facts); others are off path
size_t ggml_type_size(enum ggml_type t) {
  switch (t) {
    case GGML_TYPE_F32: return 4;
    case GGML_TYPE_Q4_K: return sizeof(block_q4_K);
    case GGML_TYPE_Q6_K: return sizeof(block_q6_K);
    case GGML_TYPE_Q8_1: return sizeof(block_q8_1);
    default: off_path("ggml_type_size");
  }
}
int64_t ggml_blck_size(enum ggml_type t) {
  switch (t) {
    case GGML_TYPE_F32: return 1;
    case GGML_TYPE_Q4_K:
    case GGML_TYPE_Q6_K: return QK_K;
    case GGML_TYPE_Q8_1: return QK8_1;
    default: off_path("ggml_blck_size");
  }
}
size_t ggml_nbytes(const struct ggml_tensor *) { off_path("ggml_nbytes"); }
bool ggml_are_same_stride(const struct ggml_tensor *, const struct ggml_tensor *) { off_path("ggml_are_same_stride"); }
bool ggml_is_contiguously_allocated(const struct ggml_tensor *) { off_path("ggml_is_contiguously_allocated"); }
size_t ggml_backend_buffer_get_alloc_size(ggml_backend_buffer_t, const struct ggml_tensor *) {
  off_path("ggml_backend_buffer_get_alloc_size");
}
enum ggml_backend_buffer_usage ggml_backend_buffer_get_usage(ggml_backend_buffer_t) {
  off_path("ggml_backend_buffer_get_usage");
}
}

// ---------------------------------------------------------------- C entry points
extern "C" {

// Bytes of the q8_1 activation buffer for K-element rows of n_tok tokens.
size_t ref_mmvq_q8_bytes(int64_t K, int64_t n_tok) {
  const int64_t padded = (K + MATRIX_ROW_PADDING - 1) / MATRIX_ROW_PADDING * MATRIX_ROW_PADDING;
  return size_t(n_tok * padded / QK8_1) * sizeof(block_q8_1);
}

// y[t][r] = W[r] . x[t] for GGUF rows W (Q4_K = 12, Q6_K = 14; rows x K, row-major blocks), f32 x
// [n_tok][K], y [n_tok][rows], n_tok <= 8: the activation quantization to q8_1 and the MMVQ kernel,
// as ggml_cuda_mul_mat_vec_q launches them for one matrix.  Returns a cudaError_t value.
int ref_mmvq(int type, const void *w, int64_t rows, int64_t K, const float *x, int64_t n_tok, float *y, void *q8,
             void *stream) {
  if ((type != GGML_TYPE_Q4_K && type != GGML_TYPE_Q6_K) || K % QK_K || n_tok < 1 || n_tok > 8 || rows < 1)
    return int(cudaErrorInvalidValue);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t padded = (K + MATRIX_ROW_PADDING - 1) / MATRIX_ROW_PADDING * MATRIX_ROW_PADDING;
  quantize_row_q8_1_cuda(x, nullptr, q8, ggml_type(type), K, K, K * n_tok, K * n_tok, padded, n_tok, 1, 1, st);
  const int64_t s01 = K / QK_K;           // blocks per weight row
  const int64_t s11 = padded / QK8_1;     // q8_1 blocks per activation row
  ggml_cuda_mm_fusion_args_device fusion{};
  mul_mat_vec_q_switch_type(w, ggml_type(type), q8, nullptr, fusion, y, int(K), int(rows), int(n_tok), int(s01),
                            int(s11), int(rows), 1, 1, 1, int(s01 * rows), int(s11 * n_tok), int(rows * n_tok), 1, 1,
                            int(s01 * rows), int(s11 * n_tok), int(rows * n_tok), 0, st);
  return int(cudaGetLastError());
}

}  // extern "C"
