// capi_kernels.cpp — kernel-level C ABI (device pointers, caller's stream).
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "capi_common.h"
#include "common.cuh"
#include "kernels.h"

namespace sfc {

static thread_local std::string t_err;

void set_error(const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
}
void clear_error() { t_err.clear(); }

static bool type_supported(int t) { return t == T_F32 || t == T_F16 || t == T_BF16 || t == T_Q4_K || t == T_Q6_K; }

// Per-device scratch for the stand-alone logits entry point (the stage owns its own).
static std::mutex g_scratch_mu;
static std::unordered_map<int, std::pair<void *, size_t>> g_scratch;

static int device_scratch(size_t bytes, void **out) {
  int dev = 0;
  SFC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  auto &e = g_scratch[dev];
  if (e.second < bytes) {
    if (e.first) cudaFree(e.first);
    e.first = nullptr;
    e.second = 0;
    SFC_CUDA(cudaMalloc(&e.first, bytes));
    e.second = bytes;
  }
  *out = e.first;
  return SFC_OK;
}

}  // namespace sfc

using namespace sfc;

extern "C" {

int sfc_abi_version(void) { return SFC_ABI_VERSION; }

const char *sfc_last_error(void) { return t_err.c_str(); }

int sfc_device_error(unsigned *code) {
  SFC_REQUIRE(code, "code is null");
  unsigned *p = device_error_ptr();
  SFC_REQUIRE(p, "device error word unavailable");
  unsigned zero = 0;
  SFC_CUDA(cudaMemcpy(code, p, sizeof(unsigned), cudaMemcpyDeviceToHost));
  SFC_CUDA(cudaMemcpy(p, &zero, sizeof(unsigned), cudaMemcpyHostToDevice));
  return SFC_OK;
}

int64_t sfc_kernel_launches(void) { return g_kernel_launches; }

int sfc_selftest_bounded_wait(unsigned spin_limit, int complete, void *stream) {
  clear_error();
  SFC_REQUIRE(spin_limit > 0, "spin_limit must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SFC_CUDA(wait_selftest(spin_limit, complete ? 1 : 0, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  return SFC_OK;
}

int64_t sfc_weight_device_bytes(int ggml_type, int64_t rows, int64_t in_dim) {
  if (!type_supported(ggml_type) || rows < 0) {
    set_error("unsupported ggml type %d", ggml_type);
    return SFC_E_INVALID;
  }
  const int64_t bytes = device_tensor_bytes(ggml_type, rows, in_dim);
  if (bytes < 0) {
    set_error("in_dim %lld invalid for type %d", (long long)in_dim, ggml_type);
    return SFC_E_INVALID;
  }
  return bytes;
}

int sfc_prepare_weights(int ggml_type, const void *gguf_dev, int64_t rows, int64_t in_dim, void *dst_dev,
                        void *stream) {
  SFC_REQUIRE(type_supported(ggml_type), "unsupported ggml type %d", ggml_type);
  SFC_REQUIRE(device_row_bytes(ggml_type, in_dim) > 0 && rows >= 0, "bad shape rows=%lld in_dim=%lld",
              (long long)rows, (long long)in_dim);
  SFC_REQUIRE(gguf_dev && dst_dev, "null pointer");
  SFC_CUDA(prepare_weights(ggml_type, gguf_dev, rows, in_dim, dst_dev, static_cast<cudaStream_t>(stream)));
  return SFC_OK;
}

int sfc_dequantize_rows(int ggml_type, const void *gguf_dev, int64_t rows, int64_t in_dim, float *out_dev,
                        void *stream) {
  SFC_REQUIRE(ggml_type == T_Q4_K || ggml_type == T_Q6_K, "dequantize supports Q4_K and Q6_K, got %d", ggml_type);
  SFC_REQUIRE(in_dim > 0 && in_dim % 256 == 0 && rows >= 0, "in_dim %lld must be a positive multiple of 256",
              (long long)in_dim);
  SFC_REQUIRE(gguf_dev && out_dev, "null pointer");
  SFC_CUDA(dequantize(ggml_type, gguf_dev, rows, in_dim, out_dev, static_cast<cudaStream_t>(stream)));
  return SFC_OK;
}

static int matmul_common(int ggml_type, const void *w0, const void *w1, int64_t out_dim, int64_t in_dim,
                         const float *x, int64_t n_tok, float *y, void *stream) {
  SFC_REQUIRE(type_supported(ggml_type), "unsupported ggml type %d", ggml_type);
  SFC_REQUIRE(device_row_bytes(ggml_type, in_dim) > 0, "in_dim %lld invalid for type %d", (long long)in_dim,
              ggml_type);
  SFC_REQUIRE(out_dim >= 0 && n_tok >= 0, "negative shape");
  SFC_REQUIRE((ggml_type != T_Q4_K && ggml_type != T_Q6_K) || in_dim <= 10240,
              "K-quant in_dim %lld exceeds the GEMV limit 10240", (long long)in_dim);
  SFC_REQUIRE(w0 && x && y, "null pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_tok >= QGEMM_MIN_TOKENS && qgemm_supported(ggml_type, in_dim)) {
    // tensor-core GEMM; a gate/up pair writes both products to scratch and applies GeGLU after
    const size_t gbytes = qgemm_scratch_bytes(n_tok, in_dim);
    const size_t pair_bytes = w1 ? size_t(2) * n_tok * out_dim * 4 : 0;
    void *scratch = nullptr;
    int rc = device_scratch(gbytes + pair_bytes + 256, &scratch);
    if (rc) return rc;
    float *tmp = reinterpret_cast<float *>(static_cast<char *>(scratch) + (gbytes + 255) / 256 * 256);
    QGemmOut outs[2] = {{ggml_type, w0, out_dim, w1 ? tmp : y, out_dim},
                        {ggml_type, w1, out_dim, tmp + n_tok * out_dim, out_dim}};
    GemmPrologue pro = {};
    pro.mode = 0;
    pro.x = x;
    SFC_CUDA(qgemm(outs, w1 ? 2 : 1, in_dim, pro, n_tok, scratch, gbytes, st));
    if (w1) SFC_CUDA(geglu(tmp, tmp + n_tok * out_dim, y, n_tok * out_dim, st));
    return SFC_OK;
  }
  SFC_CUDA(gemv(ggml_type, w0, w1, out_dim, in_dim, x, n_tok, y, out_dim, st));
  return SFC_OK;
}

int sfc_matmul(int ggml_type, const void *w_dev, int64_t out_dim, int64_t in_dim, const float *x_dev, int64_t n_tok,
               float *y_dev, void *stream) {
  return matmul_common(ggml_type, w_dev, nullptr, out_dim, in_dim, x_dev, n_tok, y_dev, stream);
}

int sfc_matmul_pair_geglu(int ggml_type, const void *w_gate_dev, const void *w_up_dev, int64_t out_dim,
                          int64_t in_dim, const float *x_dev, int64_t n_tok, float *act_dev, void *stream) {
  SFC_REQUIRE(w_up_dev, "null up matrix");
  return matmul_common(ggml_type, w_gate_dev, w_up_dev, out_dim, in_dim, x_dev, n_tok, act_dev, stream);
}

int sfc_rms_norm(const float *x_dev, const float *w_dev, int64_t n_tok, int64_t dim, float eps, float *out_dev,
                 void *stream) {
  SFC_REQUIRE(x_dev && w_dev && out_dev, "null pointer");
  SFC_REQUIRE(dim > 0 && dim < (1 << 24) && n_tok >= 0, "bad shape");
  SFC_CUDA(rms_norm(x_dev, w_dev, n_tok, int(dim), eps, out_dev, static_cast<cudaStream_t>(stream)));
  return SFC_OK;
}

int sfc_logits_argmax(int ggml_type, const void *w_dev, int64_t vocab, int64_t dim, const float *h_dev, int64_t n_tok,
                      float cap, float *all_scores_dev, int64_t *argmax_dev, float *score_dev, void *stream) {
  SFC_REQUIRE(ggml_type == T_F16 || ggml_type == T_F32 || ggml_type == T_BF16,
              "logits support F16/F32/BF16 tables, got %d", ggml_type);
  SFC_REQUIRE(vocab > 0 && dim > 0 && n_tok >= 0, "bad shape");
  SFC_REQUIRE(w_dev && h_dev && argmax_dev && score_dev, "null pointer");
  void *scratch = nullptr;
  const size_t sb = logits_scratch_bytes(n_tok);
  int rc = device_scratch(sb, &scratch);
  if (rc) return rc;
  SFC_CUDA(logits_argmax(ggml_type, w_dev, vocab, int(dim), h_dev, n_tok, cap, all_scores_dev, argmax_dev, score_dev,
                         scratch, sb, static_cast<cudaStream_t>(stream)));
  return SFC_OK;
}

int sfc_sample_temperature(const float *scores_dev, int64_t n, int64_t vocab, float temperature, uint64_t seed,
                           int64_t *tokens_dev, void *stream) {
  clear_error();
  SFC_REQUIRE(scores_dev && tokens_dev, "null pointer");
  SFC_REQUIRE(n >= 0 && vocab > 0, "bad shape");
  SFC_REQUIRE(temperature > 0.f, "temperature must be positive (use the argmax for greedy)");
  SFC_CUDA(sample_rows_temperature(scores_dev, n, vocab, temperature, seed, tokens_dev,
                                   static_cast<cudaStream_t>(stream)));
  return SFC_OK;
}

int sfc_synth_tensor(int ggml_type, uint64_t seed, const char *name, int64_t rows, int64_t in_dim, float sigma,
                     float mean, void *out_dev, void *stream) {
  SFC_REQUIRE(name && out_dev, "null pointer");
  SFC_REQUIRE(type_supported(ggml_type), "unsupported ggml type %d", ggml_type);
  SFC_REQUIRE(gguf_row_bytes(ggml_type, in_dim) > 0 && rows >= 0, "bad shape");
  SFC_CUDA(synth_tensor(ggml_type, tensor_key(seed, name), rows, in_dim, sigma, mean, out_dev,
                        static_cast<cudaStream_t>(stream)));
  return SFC_OK;
}

}  // extern "C"
