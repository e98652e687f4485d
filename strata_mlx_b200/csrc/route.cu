// The MoE block's supporting kernels (strata_mlx/fused.py):
//   sc_router        WindowLinear.__call__ (fused.py:334-390): float16 weights x activations, float32 sums
//   sc_top_k         top_k (fused.py:400-436): the k largest logits, largest first, ties to the lower index
//   sc_top_k_softmax top_k, then the softmax over the chosen logits (fused.py:490-491)
//   sc_moe_combine   moe_combine (fused.py:439-481): the routed sum in MLX's col_reduce order + sigmoid-gated shared
//   sc_swiglu        mlx-lm's swiglu (strata_mlx/blocks.py:230-238)
#include <algorithm>

#include "matvec.cuh"
#include "route.cuh"

namespace sc {

// ---- router: one warp per weight row, 16-byte loads of eight float16 weights, every token of the window per load

template <typename InT>
__global__ void __launch_bounds__(256) router_kernel(const __half* __restrict__ w, int rows, int cols,
                                                     const InT* __restrict__ x, int tokens, float* __restrict__ out) {
  extern __shared__ __align__(16) float xs[];  // (tokens, cols) float32
  for (int i = threadIdx.x; i < tokens * cols; i += blockDim.x) xs[i] = to_f32(x[i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + warp; r < rows; r += gridDim.x * 8) {
    router_row<ROUTER_MAX_TOKENS>(w + int64_t(r) * cols, cols, xs, tokens, lane, out + r, rows);
  }
}

// ---- router for a chunk of a prompt (more than ROUTER_MAX_TOKENS tokens): logits (tokens, rows) = x . W^T as a
// tiled product on the CUDA cores, 64 tokens x 64 rows a block, 4 x 4 a thread, float32 sums of the float16 weights
// and the activations (the reference multiplies floats here, fused.py:386-388 through the layer's own product)

constexpr int RTB = 64, RKB = 32;

template <typename InT>
__global__ void __launch_bounds__(256) router_tile_kernel(const __half* __restrict__ w, int rows, int cols,
                                                          const InT* __restrict__ x, int tokens,
                                                          float* __restrict__ out) {
  __shared__ float xs[RKB][RTB + 4], ws[RKB][RTB + 4];
  const int t0 = blockIdx.y * RTB, r0 = blockIdx.x * RTB;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // outputs: tokens t0 + 4 ty .., rows r0 + 4 tx ..
  float acc[4][4] = {};
  for (int k0 = 0; k0 < cols; k0 += RKB) {
    for (int i = threadIdx.x; i < RTB * RKB; i += 256) {
      const int a = i / RKB, k = i % RKB;
      xs[k][a] = (t0 + a < tokens && k0 + k < cols) ? to_f32(x[int64_t(t0 + a) * cols + k0 + k]) : 0.f;
      ws[k][a] = (r0 + a < rows && k0 + k < cols) ? __half2float(w[int64_t(r0 + a) * cols + k0 + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < RKB; ++k) {
      float xa[4], wb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xa[j] = xs[k][4 * ty + j];
        wb[j] = ws[k][4 * tx + j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wb[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = t0 + 4 * ty + i, r = r0 + 4 * tx + j;
      if (t < tokens && r < rows) out[int64_t(t) * rows + r] = acc[i][j];
    }
}

// ---- top-k (+ softmax): one warp per row of logits

__global__ void topk_kernel(const float* __restrict__ logits, int rows, int n, int k, uint32_t* __restrict__ idx,
                            float* __restrict__ wts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  warp_topk(logits + int64_t(warp) * n, n, k, lane, idx + int64_t(warp) * k, wts ? wts + int64_t(warp) * k : nullptr);
}

// ---- combine

template <typename T>
__global__ void combine_kernel(const T* __restrict__ y, const float* __restrict__ w, const T* __restrict__ g,
                               const T* __restrict__ s, int rows, int k, int d, T* __restrict__ out) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= int64_t(rows) * d) return;
  const int t = int(i / d), c = int(i % d);
  float yk[16];
  for (int q = 0; q < k; ++q) yk[q] = to_f32(y[(int64_t(t) * k + q) * d + c]);
  out[i] = from_f32<T>(combine_one<T>(yk, w + int64_t(t) * k, k, to_f32(g[t]), to_f32(s[i])));
}

template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t n, T* __restrict__ out) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = from_f32<T>(swiglu_mlx<T>(to_f32(g[i]), to_f32(u[i])));
}

// 16 bytes a thread (8 values of a 2-byte type; n8 = n / 8, every pointer 16-byte aligned)
template <typename T>
__global__ void swiglu16_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u, int64_t n8,
                                uint4* __restrict__ out) {
  static_assert(sizeof(T) == 2, "16-byte vectors of a 2-byte type");
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const uint4 gv = g[i], uv = u[i];
    const T* gs = reinterpret_cast<const T*>(&gv);
    const T* us = reinterpret_cast<const T*>(&uv);
    uint4 o;
    T* os = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) os[j] = from_f32<T>(swiglu_mlx<T>(to_f32(gs[j]), to_f32(us[j])));
    out[i] = o;
  }
}

}  // namespace sc

using namespace sc;

static int launch_rc() { return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA; }

extern "C" int sc_router(const void* w, int rows, int cols, const void* x, int dtype, int tokens, float* logits,
                         void* stream) {
  if (!w || !x || !logits || rows < 0 || cols < 0 || tokens < 0) return SC_ERR_ARG;
  if (cols % 8 || (reinterpret_cast<uintptr_t>(w) & 15)) return SC_ERR_ALIGN;
  if (rows == 0 || tokens == 0) return SC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (tokens > ROUTER_MAX_TOKENS) {  // a chunk of a prompt: the tiled product, the weights read once a 64 tokens
    const dim3 grid(unsigned(ceil_div(rows, RTB)), unsigned(ceil_div(tokens, RTB)));
    bool ok = dispatch_dtype(dtype, [&]<typename InT>() {
      router_tile_kernel<InT><<<grid, 256, 0, s>>>(static_cast<const __half*>(w), rows, cols,
                                                    static_cast<const InT*>(x), tokens, logits);
    });
    if (!ok) return SC_ERR_DTYPE;
    return launch_rc();
  }
  // windows of up to ROUTER_MAX_TOKENS tokens whose float32 activations fit shared memory
  const int per = std::max(1, std::min(ROUTER_MAX_TOKENS, int((96 * 1024) / (int64_t(cols) * 4))));
  const int grid = int(std::min<int64_t>(ceil_div(rows, 8), 148 * 4));
  for (int t0 = 0; t0 < tokens; t0 += per) {
    const int nt = std::min(per, tokens - t0);
    const size_t smem = size_t(nt) * cols * 4;
    bool ok = dispatch_dtype(dtype, [&]<typename InT>() {
      auto kern = router_kernel<InT>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      kern<<<grid, 256, smem, s>>>(static_cast<const __half*>(w), rows, cols, static_cast<const InT*>(x) + int64_t(t0) * cols,
                                   nt, logits + int64_t(t0) * rows);
    });
    if (!ok) return SC_ERR_DTYPE;
    if (int rc = launch_rc()) return rc;
  }
  return SC_OK;
}

static int topk_common(const float* logits, int rows, int n, int k, uint32_t* idx, float* wts, void* stream) {
  if (!logits || !idx || rows < 0 || n < 1 || k < 1) return SC_ERR_ARG;
  if (k > TOPK_MAX_K || k > n || n > TOPK_MAX_N) return SC_ERR_SHAPE;
  if (rows == 0) return SC_OK;
  const int threads = 128;
  const int grid = int(ceil_div(int64_t(rows) * 32, threads));
  topk_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(logits, rows, n, k, idx, wts);
  return launch_rc();
}

extern "C" int sc_top_k(const float* logits, int rows, int n, int k, uint32_t* idx, void* stream) {
  return topk_common(logits, rows, n, k, idx, nullptr, stream);
}

extern "C" int sc_top_k_softmax(const float* logits, int rows, int n, int k, uint32_t* idx, float* weights,
                                void* stream) {
  if (!weights) return SC_ERR_ARG;
  return topk_common(logits, rows, n, k, idx, weights, stream);
}

extern "C" int sc_moe_combine(const void* y, const float* w, const void* g, const void* s, int rows, int k, int d,
                              int dtype, void* out, void* stream) {
  if (!y || !w || !g || !s || !out || rows < 0 || k < 1 || d < 1) return SC_ERR_ARG;
  if (k > 16) return SC_ERR_SHAPE;
  if (rows == 0) return SC_OK;
  const int64_t n = int64_t(rows) * d;
  const int threads = 256;
  bool ok = dispatch_dtype(dtype, [&]<typename T>() {
    combine_kernel<T><<<int(ceil_div(n, threads)), threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const T*>(y), w, static_cast<const T*>(g), static_cast<const T*>(s), rows, k, d, static_cast<T*>(out));
  });
  if (!ok) return SC_ERR_DTYPE;
  return launch_rc();
}

extern "C" int sc_swiglu(const void* gate, const void* up, int64_t n, int dtype, void* out, void* stream) {
  if (!gate || !up || !out || n < 0) return SC_ERR_ARG;
  if (n == 0) return SC_OK;
  const int threads = 256;
  const int grid = int(std::min<int64_t>(ceil_div(n, threads), 148 * 8));
  const bool vec = dtype != SC_F32 && n % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) |
                     reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  bool ok = dispatch_dtype(dtype, [&]<typename T>() {
    if constexpr (sizeof(T) == 2) {
      if (vec) {
        const int g8 = int(std::min<int64_t>(ceil_div(n / 8, threads), 148 * 8));
        swiglu16_kernel<T><<<g8, threads, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint4*>(gate), static_cast<const uint4*>(up), n / 8, static_cast<uint4*>(out));
        return;
      }
    }
    swiglu_kernel<T><<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const T*>(gate),
                                                                               static_cast<const T*>(up), n,
                                                                               static_cast<T*>(out));
  });
  if (!ok) return SC_ERR_DTYPE;
  return launch_rc();
}
