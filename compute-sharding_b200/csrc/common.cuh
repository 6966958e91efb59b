// common.cuh — shared device helpers for the sm_100a stage-forward kernels.
//
// GGUF K-quant block layouts follow crates/stage-forward-lab/src/quants.rs:10-21:
//   Q4_K: 144 B / 256 elements = d f16 | dmin f16 | 12 B packed 6-bit (sc, m) x 8 | 128 B nibbles
//   Q6_K: 210 B / 256 elements = ql 128 B | qh 64 B | 16 x int8 scales | d f16
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sfc {

constexpr int QK_K = 256;
constexpr int BLOCK_Q4_K = 144;
constexpr int BLOCK_Q6_K = 210;

enum GgmlType : int { T_F32 = 0, T_F16 = 1, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30 };

// Device layout of K-quant weights (written by prepare_weights): rows in tiles of 16 (the last tile
// zero-padded), one record per (tile, 256-element block), records tile-major (record index
// tile * nb + block), so any tile's run of blocks is one contiguous byte range:
//   Q4_K record, 2304 B:  hdr[16][16] (d, dmin, 12 packed scale bytes per row) | qs[16][128]
//   Q6_K record, 3360 B:  ql[16][128] | qh[16][64] | sc[16][16] | d[16] (fp16)
// Inside qs and ql the 16-byte chunk j of row r is stored at chunk j ^ (r & 7), inside qh at
// j ^ ((r >> 1) & 3): the 8 rows that one warp reads at a time then hit distinct shared-memory banks.
constexpr int KQ_TILE = 16;
constexpr int REC_Q4_K = 2304;
constexpr int REC_Q6_K = 3360;
__host__ __device__ constexpr int kquant_rec_bytes(int type) {
  return type == T_Q4_K ? REC_Q4_K : type == T_Q6_K ? REC_Q6_K : 0;
}

// Device-side error word: kernels whose bounded waits expire record a code here
// instead of spinning forever; the host reads it after synchronising.
enum DeviceError : unsigned { DEV_OK = 0, DEV_WAIT_TIMEOUT = 1, DEV_BAD_ARG = 2 };

// Bounded-wait budget for mbarrier polls (each try_wait suspends for up to the
// hardware time hint, so this is seconds, far above any legitimate latency).
constexpr unsigned MBAR_SPIN_LIMIT = 1u << 24;

// SplitMix64 finaliser of key + (ctr + 1) * golden ratio: the counter-based hash behind the
// synthetic weights and the seeded sampling uniforms (identical on host and device).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t key, uint64_t ctr) {
  uint64_t z = key + (ctr + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---- mbarrier + bulk async copy (TMA engine, non-tensor form) ----------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Returns true once the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls (MBAR_SPIN_LIMIT by default) and records
// DEV_WAIT_TIMEOUT in *err.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, unsigned *err,
                                                  unsigned limit = MBAR_SPIN_LIMIT) {
  for (unsigned i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicExch(err, DEV_WAIT_TIMEOUT);
  return false;
}

// One bulk global->shared copy completing on `bar` (16 B aligned src/dst, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: wait for the producing grid's memory, and let the
// next grid start its independent prologue (weight prefetch) early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

__device__ __forceinline__ int dp4a_us(uint32_t a_u8x4, uint32_t b_s8x4, int c) {
  int r;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a_u8x4), "r"(b_s8x4), "r"(c));
  return r;
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

// ---------------------------------------------------------------- residual-stream RMSNorm order
// Every RMSNorm of the residual stream sums its squares in one order, whichever kernel computes
// it (a GEMV or GEMM prologue, the residual add that closes a stage, the output norm): the row is
// cut into 256-element blocks, lane l of a warp holds elements 8l..8l+7 of a block (zero past the
// row's end) and sums their squares by fused multiply-add from zero in element order, the block
// sum is the xor butterfly of warp_sum over the lanes, and the row total adds the block sums from
// zero in block order.  The scale 1/sqrt(total/dim + eps) and everything computed from it are
// then the same bits in every kernel, so a layer range split over several stages reproduces the
// single-stage hidden states exactly.
__device__ __forceinline__ float block_sumsq(const float (&v)[8]) {
  float q = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) q = __fmaf_rn(v[e], v[e], q);
  return warp_sum(q);
}

// The row total of that order computed by the NW warps of a block: warp w takes blocks w, w+NW, ..
// and load8(b, v) fills the calling lane's 8 values of block b.  `red` holds 64 shared floats.
// Every thread of the block must call it; all of them return the total.
template <int NW, class Load8>
__device__ __forceinline__ float row_sumsq(int nb, float *red, Load8 load8) {
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
  float tot = 0.f;
  for (int c0 = 0; c0 < nb; c0 += 64) {
    const int c1 = nb < c0 + 64 ? nb : c0 + 64;
    for (int b = c0 + warp; b < c1; b += NW) {
      float v[8];
      load8(b, v);
      const float s = block_sumsq(v);
      if (lane == 0) red[b - c0] = s;
    }
    __syncthreads();
    for (int b = c0; b < c1; ++b) tot = __fadd_rn(tot, red[b - c0]);
    __syncthreads();
  }
  return tot;
}

// The residual add of a post-norm block: (a * s) * w + resid (w null: a + resid), then times the
// layer scale when there is one, each operation rounded on its own (no contraction), in the order
// of real_math.rs:30-47 followed by the residual add.
__device__ __forceinline__ float resid_add(float a, float s, const float *w, float wv, float resid, const float *ls,
                                           float lsv) {
  float r = __fadd_rn(w ? __fmul_rn(__fmul_rn(a, s), wv) : a, resid);
  if (ls) r = __fmul_rn(r, lsv);
  return r;
}

}  // namespace sfc
