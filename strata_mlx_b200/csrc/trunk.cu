// The synthetic decoder's trunk around the MoE blocks (configurations 4 and 5): RMSNorm with the residual add, and
// RoPE with the paged cache's write, each one kernel where torch's operations took several. Not the hot path; they
// keep a decode step's launches few.
//
//   sc_add_rmsnorm  x = T(x + delta) (when delta is given), out = T(x * rsqrt(mean(x^2) + eps) * w), float32 math
//   sc_rope_cache   RoPE (rotate-half, angles from cos / sin tables at the positions pos .. pos + t - 1 read on the
//                   device) on q in place and on k, and k, v written into the cache's slots of those positions
#include "common.cuh"

namespace sc {
namespace tr {

// a block per row, 256 threads, eight values a thread (cols a multiple of 8, at most 8192)
template <typename T>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(T* __restrict__ x, const T* __restrict__ delta,
                                                          const T* __restrict__ w, int cols, float eps,
                                                          T* __restrict__ out) {
  const int row = blockIdx.x;
  T* xr = x + int64_t(row) * cols;
  float v[4][8];
  float ss = 0.f;
  const int n8 = cols / 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = threadIdx.x + j * 256;
    if (c < n8) {
      uint4 a = reinterpret_cast<const uint4*>(xr)[c];
      const T* av = reinterpret_cast<const T*>(&a);
      if (delta) {
        const uint4 b = reinterpret_cast<const uint4*>(delta + int64_t(row) * cols)[c];
        const T* bv = reinterpret_cast<const T*>(&b);
        T* aw = reinterpret_cast<T*>(&a);
#pragma unroll
        for (int e = 0; e < 8; ++e) aw[e] = from_f32<T>(to_f32(av[e]) + to_f32(bv[e]));
        reinterpret_cast<uint4*>(xr)[c] = a;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[j][e] = to_f32(av[e]);
        ss = fmaf(v[j][e], v[j][e], ss);
      }
    }
  }
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / float(cols) + eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = threadIdx.x + j * 256;
    if (c < n8) {
      const uint4 wv = reinterpret_cast<const uint4*>(w)[c];
      const T* ww = reinterpret_cast<const T*>(&wv);
      uint4 o;
      T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) ov[e] = from_f32<T>(v[j][e] * r * to_f32(ww[e]));
      reinterpret_cast<uint4*>(out + int64_t(row) * cols)[c] = o;
    }
  }
}

// grid (t, q_heads + kv_heads): a block per (token, head), HALF threads (half the head dimension)
template <typename T>
__global__ void rope_cache_kernel(T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, int hq, int hkv,
                                  int half, const float* __restrict__ cos, const float* __restrict__ sin,
                                  const int32_t* __restrict__ pos, const int32_t* __restrict__ table, int page,
                                  T* __restrict__ kc, T* __restrict__ vc) {
  const int i = blockIdx.x, h = blockIdx.y, d = threadIdx.x, dim = 2 * half;
  const int p = *pos + i;
  const float c = cos[int64_t(p) * half + d], s = sin[int64_t(p) * half + d];
  if (h < hq) {
    T* r = q + (int64_t(i) * hq + h) * dim;
    const float a = to_f32(r[d]), b = to_f32(r[d + half]);
    r[d] = from_f32<T>(a * c - b * s);
    r[d + half] = from_f32<T>(b * c + a * s);
    return;
  }
  const int hk = h - hq;
  const int64_t slot = int64_t(table[p / page]) * page + p % page;
  const T* kr = k + (int64_t(i) * hkv + hk) * dim;
  const T* vr = v + (int64_t(i) * hkv + hk) * dim;
  T* kd = kc + (slot * hkv + hk) * dim;
  T* vd = vc + (slot * hkv + hk) * dim;
  const float a = to_f32(kr[d]), b = to_f32(kr[d + half]);
  kd[d] = from_f32<T>(a * c - b * s);
  kd[d + half] = from_f32<T>(b * c + a * s);
  vd[d] = vr[d];
  vd[d + half] = vr[d + half];
}

}  // namespace tr
}  // namespace sc

using namespace sc;

extern "C" int sc_add_rmsnorm(void* x, const void* delta, const void* w, int rows, int cols, float eps, int dtype,
                              void* out, void* stream) {
  if (!x || !w || !out || rows < 0) return SC_ERR_ARG;
  if (cols % 8 || cols > 8192 || cols < 8) return SC_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return SC_ERR_ALIGN;
  if (rows == 0) return SC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SC_BF16)
    tr::add_rmsnorm_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>(static_cast<__nv_bfloat16*>(x),
                                                               static_cast<const __nv_bfloat16*>(delta),
                                                               static_cast<const __nv_bfloat16*>(w), cols, eps,
                                                               static_cast<__nv_bfloat16*>(out));
  else if (dtype == SC_F16)
    tr::add_rmsnorm_kernel<__half><<<rows, 256, 0, s>>>(static_cast<__half*>(x), static_cast<const __half*>(delta),
                                                        static_cast<const __half*>(w), cols, eps,
                                                        static_cast<__half*>(out));
  else
    return SC_ERR_DTYPE;
  if (cudaError_t e = cudaGetLastError()) return cuda_failed(e, "add_rmsnorm launch");
  return SC_OK;
}

extern "C" int sc_rope_cache(void* q, const void* k, const void* v, int tokens, int q_heads, int kv_heads, int head_dim,
                             const float* cos, const float* sin, const int32_t* pos, const int32_t* table, int page,
                             void* k_cache, void* v_cache, int dtype, void* stream) {
  if (!q || !k || !v || !cos || !sin || !pos || !table || !k_cache || !v_cache) return SC_ERR_ARG;
  if (tokens < 1 || head_dim % 2 || head_dim > 2048 || page < 1) return SC_ERR_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(tokens, q_heads + kv_heads);
  if (dtype == SC_BF16)
    tr::rope_cache_kernel<__nv_bfloat16><<<grid, head_dim / 2, 0, s>>>(
        static_cast<__nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
        q_heads, kv_heads, head_dim / 2, cos, sin, pos, table, page, static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache));
  else
    return SC_ERR_DTYPE;
  if (cudaError_t e = cudaGetLastError()) return cuda_failed(e, "rope_cache launch");
  return SC_OK;
}
