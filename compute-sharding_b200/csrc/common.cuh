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

}  // namespace sfc
