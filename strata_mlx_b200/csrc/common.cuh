// Shared device code of the quantized-expert library: block types, activation types, the codebook tables,
// byte readers, and the PTX wrappers for mbarriers and bulk (TMA) copies.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/strata_cuda.h"

#define SC_TABLE static __device__ const
#include "iq_tables.h"
#undef SC_TABLE

namespace sc {

// ---- block types (strata_mlx/blocks.py:35-38, strata_mlx/gguf.py:27 for Q8_0)

struct BlockInfo { int per_block, block_bytes; };

__host__ __device__ constexpr BlockInfo block_info(int kind) {
  return kind == SC_Q2_0 ? BlockInfo{64, 18} : kind == SC_IQ4_NL ? BlockInfo{32, 18}
       : kind == SC_IQ4_XS ? BlockInfo{256, 136} : kind == SC_IQ3_S ? BlockInfo{256, 110}
       : kind == SC_IQ3_XXS ? BlockInfo{256, 98} : kind == SC_IQ2_S ? BlockInfo{256, 82}
       : kind == SC_IQ2_XS ? BlockInfo{256, 74} : kind == SC_IQ2_XXS ? BlockInfo{256, 66}
       : kind == SC_IQ1_M ? BlockInfo{256, 56} : kind == SC_Q3_K ? BlockInfo{256, 110}
       : kind == SC_Q8_0 ? BlockInfo{32, 34} : BlockInfo{0, 0};
}

// bytes of a row of `cols` weights, or -1 when the row does not end on a block
__host__ __device__ inline int64_t row_bytes(int kind, int64_t cols) {
  BlockInfo b = block_info(kind);
  if (b.per_block == 0 || cols % b.per_block) return -1;
  return cols / b.per_block * b.block_bytes;
}

// ---- activation types

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// round a float32 to T and back: the value an array of type T would hold
template <typename T> __device__ __forceinline__ float round_to(float v) { return to_f32<T>(from_f32<T>(v)); }

// ---- little-endian readers (strata_mlx/blocks.py:40-47); byte-wise, as fields sit at odd offsets

__device__ __forceinline__ uint32_t u16_at(const uint8_t* b) { return uint32_t(b[0]) | (uint32_t(b[1]) << 8); }
__device__ __forceinline__ uint32_t u32_at(const uint8_t* b) {
  return uint32_t(b[0]) | (uint32_t(b[1]) << 8) | (uint32_t(b[2]) << 16) | (uint32_t(b[3]) << 24);
}
__device__ __forceinline__ float half_bits(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)v)); }
__device__ __forceinline__ float half_at(const uint8_t* b) { return half_bits(u16_at(b)); }

// ---- the codebooks a kernel reads; copied into shared memory at a block's start

struct Tabs {
  const uint32_t* iq3s;   // 512
  const uint32_t* iq3xxs; // 256
  const uint64_t* iq2s;   // 1024
  const uint64_t* iq2xs;  // 512
  const uint64_t* iq2xxs; // 256
  const uint64_t* iq1;    // 2048, values + 1
  const uint8_t* ksigns;  // 128
  const int8_t* kvalues;  // 16
};

// shared-memory bytes the tables of `kind` take
__host__ __device__ constexpr int table_bytes(int kind) {
  return kind == SC_IQ3_S ? 512 * 4 : kind == SC_IQ3_XXS ? 256 * 4 + 128
       : kind == SC_IQ2_S ? 1024 * 8 : kind == SC_IQ2_XS ? 512 * 8 + 128
       : kind == SC_IQ2_XXS ? 256 * 8 + 128 : kind == SC_IQ1_M ? 2048 * 8
       : (kind == SC_IQ4_NL || kind == SC_IQ4_XS) ? 16 : 0;
}

// Copies the tables `KIND` needs to `smem` (8-byte aligned, table_bytes(KIND) long) with every thread of the
// block; the caller synchronizes before use.
template <int KIND>
__device__ __forceinline__ Tabs load_tabs(uint8_t* smem) {
  Tabs t{};
  const int tid = threadIdx.x + blockDim.x * (threadIdx.y + blockDim.y * threadIdx.z);
  const int nt = blockDim.x * blockDim.y * blockDim.z;
  auto copy64 = [&](const uint64_t* src, int n, uint8_t* dst) {
    uint64_t* d = reinterpret_cast<uint64_t*>(dst);
    for (int i = tid; i < n; i += nt) d[i] = src[i];
    return reinterpret_cast<const uint64_t*>(dst);
  };
  auto copy32 = [&](const uint32_t* src, int n, uint8_t* dst) {
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    for (int i = tid; i < n; i += nt) d[i] = src[i];
    return reinterpret_cast<const uint32_t*>(dst);
  };
  auto copy8 = [&](const uint8_t* src, int n, uint8_t* dst) {
    for (int i = tid; i < n; i += nt) dst[i] = src[i];
    return reinterpret_cast<const uint8_t*>(dst);
  };
  if (KIND == SC_IQ3_S) t.iq3s = copy32(IQ3S_GRID, 512, smem);
  if (KIND == SC_IQ3_XXS) { t.iq3xxs = copy32(IQ3XXS_GRID, 256, smem); t.ksigns = copy8(KSIGNS, 128, smem + 1024); }
  if (KIND == SC_IQ2_S) t.iq2s = copy64(IQ2S_GRID, 1024, smem);
  if (KIND == SC_IQ2_XS) { t.iq2xs = copy64(IQ2XS_GRID, 512, smem); t.ksigns = copy8(KSIGNS, 128, smem + 4096); }
  if (KIND == SC_IQ2_XXS) { t.iq2xxs = copy64(IQ2XXS_GRID, 256, smem); t.ksigns = copy8(KSIGNS, 128, smem + 2048); }
  if (KIND == SC_IQ1_M) t.iq1 = copy64(IQ1_GRID, 2048, smem);
  if (KIND == SC_IQ4_NL || KIND == SC_IQ4_XS)
    t.kvalues = reinterpret_cast<const int8_t*>(copy8(reinterpret_cast<const uint8_t*>(KVALUES), 16, smem));
  return t;
}

// ---- error word: kernels record what went wrong here instead of trapping

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---- mbarriers and bulk copies (PTX)

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete, for at most about `limit` clock cycles (a second at the
// B200's clocks by default). Returns false, having recorded SC_ERR_TIMEOUT, when the wait gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          long long limit = 2000000000LL) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > limit) {
      record_error(err, SC_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// mbar_wait for warps that share their SM with others doing the work: each try_wait may suspend the thread for
// up to `hint_ns` (it wakes when the phase completes), so a waiting warp takes no issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* err,
                                                long long limit = 2000000000LL, uint32_t hint_ns = 1000000) {
  if (mbar_try_wait_sleep(bar, parity, hint_ns)) return true;
  const long long start = clock64();
  while (!mbar_try_wait_sleep(bar, parity, hint_ns)) {
    if (clock64() - start > limit) {
      record_error(err, SC_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// One-dimensional bulk copy global -> this block's shared memory, completing `bytes` on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue, and wait for the
// previous kernel's results. Both are no-ops when the launch did not ask for it.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// A failed CUDA call in host code: SC_ERR_CUDA, and with SC_VERBOSE=1 in the environment the call site and CUDA's
// error name on stderr (the C ABI returns codes only; this is for finding which call failed).
int cuda_failed(cudaError_t e, const char* where);

// Raises kernel `kern`'s dynamic shared-memory limit on the current device to at least `bytes`, remembering per
// (device, kernel) what it was set to, so that the driver is called only when a launch needs more than before.
// The record is per kernel: several host paths that launch one kernel with different sizes share it.
int raise_smem(const void* kern, int bytes, const char* where);

__host__ __device__ constexpr int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ constexpr int align16(int v) { return (v + 15) & ~15; }

}  // namespace sc
