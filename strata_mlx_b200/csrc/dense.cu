// Dense layers held as Q6_K's three parts (strata_mlx/dense.py:109-167 ScaledLinear): a weight is code * scale * d,
// the code a signed byte (the block's six bits less 32), a signed byte scale to every 16 weights of a row, a
// float16 d to every d_step (256, or fewer where the inputs were reordered). 8.56 bits a weight.
//
//   scaled_matvec_kernel  out[t] = W . x[t] for a window of up to 8 tokens: a warp a row, 16 weights a lane at a
//                         time (one 16-byte load of codes, one scale), float32 sums reduced across the warp
//   scaled_floats_kernel  every weight as a float of the output type, worked out in float32 as the reference does
//                         (float(d) * float(scale), times float(code)) and rounded once (dense.py:73-82)
#include "decode.cuh"

namespace sc {

constexpr int SC_DENSE_MAX_TOKENS = 8;  // dense.py:33 MAX_TOKENS: more is a chunk of a prompt, multiplied as floats
constexpr int SCL_WARPS = 8;

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&v)[16]);
template <>
__device__ __forceinline__ void load16<float>(const float* p, float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(p) + j);
    v[4 * j] = f.x, v[4 * j + 1] = f.y, v[4 * j + 2] = f.z, v[4 * j + 3] = f.w;
  }
}
template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&v)[16]) {  // the 16-bit types: two 16-byte loads
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + j);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[8 * j + i] = to_f32(h[i]);
  }
}

template <typename T>
__global__ void __launch_bounds__(SCL_WARPS * 32) scaled_matvec_kernel(const int8_t* __restrict__ codes,
                                                                      const int8_t* __restrict__ scales,
                                                                      const __half* __restrict__ d, int rows, int cols,
                                                                      int d_step, const T* __restrict__ x, int tokens,
                                                                      T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * SCL_WARPS + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int8_t* cr = codes + int64_t(r) * cols;
  const int8_t* sr = scales + int64_t(r) * (cols / 16);
  const __half* dr = d + int64_t(r) * (cols / d_step);
  float acc[SC_DENSE_MAX_TOKENS];
#pragma unroll
  for (int t = 0; t < SC_DENSE_MAX_TOKENS; ++t) acc[t] = 0.f;
  for (int c = 16 * lane; c < cols; c += 16 * 32) {
    const int4 q = __ldg(reinterpret_cast<const int4*>(cr + c));
    const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
    float w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = float(qb[i]);
    const float s = __half2float(dr[c / d_step]) * float(sr[c / 16]);
#pragma unroll
    for (int t = 0; t < SC_DENSE_MAX_TOKENS; ++t) {
      if (t < tokens) {
        float xv[16];
        load16<T>(x + int64_t(t) * cols + c, xv);
        float p = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) p = fmaf(w[i], xv[i], p);
        acc[t] = fmaf(s, p, acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < SC_DENSE_MAX_TOKENS; ++t) {
    if (t < tokens) {
      float v = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) out[int64_t(t) * rows + r] = from_f32<T>(v);
    }
  }
}

template <typename T>
__global__ void scaled_floats_kernel(const int8_t* __restrict__ codes, const int8_t* __restrict__ scales,
                                     const __half* __restrict__ d, int rows, int cols, int d_step,
                                     T* __restrict__ out) {
  const int groups = cols / 16;
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;  // one scale's 16 weights
  if (i >= int64_t(rows) * groups) return;
  const int r = int(i / groups), g = int(i % groups);
  const float s = __half2float(d[int64_t(r) * (cols / d_step) + 16 * g / d_step]) * float(scales[i]);
  const int4 q = __ldg(reinterpret_cast<const int4*>(codes + int64_t(r) * cols + 16 * g));
  const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
  T* o = out + int64_t(r) * cols + 16 * g;
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j] = from_f32<T>(s * float(qb[j]));
}

}  // namespace sc

using namespace sc;

static int scaled_check(const void* codes, const void* scales, const void* d, int rows, int cols, int d_step) {
  if (!codes || !scales || !d || rows < 0 || cols < 0) return SC_ERR_ARG;
  if (cols % 256 || rows % 4 || d_step < 16 || d_step % 16 || cols % d_step) return SC_ERR_SHAPE;  // dense.py:97-99
  if ((reinterpret_cast<uintptr_t>(codes) & 15)) return SC_ERR_ALIGN;
  return SC_OK;
}

extern "C" int sc_scaled_matvec(const void* codes, const void* scales, const void* d, int rows, int cols, int d_step,
                                const void* x, int dtype, int tokens, void* out, void* stream) {
  if (int rc = scaled_check(codes, scales, d, rows, cols, d_step)) return rc;
  if (!x || !out || tokens < 0) return SC_ERR_ARG;
  if (tokens > SC_DENSE_MAX_TOKENS) return SC_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) & 15)) return SC_ERR_ALIGN;
  if (rows == 0 || tokens == 0) return SC_OK;
  const int grid = int(ceil_div(rows, SCL_WARPS));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool ok = dispatch_dtype(dtype, [&]<typename T>() {
    scaled_matvec_kernel<T><<<grid, SCL_WARPS * 32, 0, s>>>(
        static_cast<const int8_t*>(codes), static_cast<const int8_t*>(scales), static_cast<const __half*>(d), rows,
        cols, d_step, static_cast<const T*>(x), tokens, static_cast<T*>(out));
  });
  if (!ok) return SC_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

extern "C" int sc_scaled_floats(const void* codes, const void* scales, const void* d, int rows, int cols, int d_step,
                                int out_dtype, void* out, void* stream) {
  if (int rc = scaled_check(codes, scales, d, rows, cols, d_step)) return rc;
  if (!out) return SC_ERR_ARG;
  if (rows == 0) return SC_OK;
  const int64_t n = int64_t(rows) * (cols / 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool ok = dispatch_dtype(out_dtype, [&]<typename T>() {
    scaled_floats_kernel<T><<<int(ceil_div(n, 256)), 256, 0, s>>>(static_cast<const int8_t*>(codes),
                                                                  static_cast<const int8_t*>(scales),
                                                                  static_cast<const __half*>(d), rows, cols, d_step,
                                                                  static_cast<T*>(out));
  });
  if (!ok) return SC_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}
