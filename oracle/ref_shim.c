/*
 * ref_shim.c — link stubs for building the reference's ggml-quants.c alone.
 *
 * TEST INFRASTRUCTURE ONLY. ggml-quants.c (vendor/llama.cpp/ggml/src) references
 * four ggml core symbols from its quantizer validation helpers. The dequantizers
 * the oracle cross-checks (dequantize_row_q4_K / _q6_K) never reach them, so the
 * stubs only abort or report zero.
 */
#include <stdarg.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

void ggml_abort(const char *file, int line, const char *fmt, ...) {
  fprintf(stderr, "ggml_abort from reference quants at %s:%d\n", file, line);
  abort();
}
size_t ggml_row_size(int type, int64_t ne) { (void)type; (void)ne; return 0; }
const char *ggml_type_name(int type) { (void)type; return "?"; }
size_t ggml_type_size(int type) { (void)type; return 0; }
