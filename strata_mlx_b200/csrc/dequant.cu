// sc_dequant: every weight of a stack of block matrices as float32/float16/bfloat16
// (strata_mlx/blocks.py:261-270 _DEQUANT, :397-404 dequantize). One thread decodes one run of 32 weights with
// the exact decoders of decode.cuh and writes them as four 16-byte (or 8-byte) stores.
#include "decode.cuh"

namespace sc {

template <int KIND, typename OutT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ blocks, int64_t total_runs,
                                                      int runs, int64_t rbytes, OutT* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem[];
  const Tabs t = load_tabs<KIND>(smem);
  __syncthreads();
  for (int64_t g = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; g < total_runs; g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = g / runs;
    const int n = int(g - r * runs);
    float w[32];
    unpack32<KIND>(blocks + r * rbytes, n, w, t);
    OutT* o = out + g * 32;  // row r, run n: (r * runs + n) * 32
    if constexpr (sizeof(OutT) == 4) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(w[j], w[j + 1], w[j + 2], w[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 v;
        OutT h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = from_f32<OutT>(w[j + i]);
        memcpy(&v, h, 16);
        *reinterpret_cast<uint4*>(o + j) = v;
      }
    }
  }
}

}  // namespace sc

using namespace sc;

extern "C" int sc_dequant(int kind, const void* blocks, int64_t mats, int rows, int cols, int out_dtype, void* out,
                          void* stream) {
  if (!blocks || !out || mats < 0 || rows < 0 || cols < 0) return SC_ERR_ARG;
  if (block_info(kind).per_block == 0) return SC_ERR_KIND;
  const int64_t rb = row_bytes(kind, cols);
  if (rb < 0) return SC_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) return SC_ERR_ALIGN;
  const int64_t total_runs = mats * rows * int64_t(cols / 32);
  if (total_runs == 0) return SC_OK;
  const int threads = 256;
  const int64_t want = ceil_div(total_runs, threads);
  const int grid = int(want < 148 * 16 ? want : 148 * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool ok_dtype = true;
  dispatch_kind(kind, [&]<int KIND>() {
    ok_dtype = dispatch_dtype(out_dtype, [&]<typename OutT>() {
      dequant_kernel<KIND, OutT><<<grid, threads, table_bytes(KIND) + 16, s>>>(
          static_cast<const uint8_t*>(blocks), total_runs, cols / 32, rb, static_cast<OutT*>(out));
    });
  });
  if (!ok_dtype) return SC_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}
