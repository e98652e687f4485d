// Dense layers held as Q6_K's three parts (strata_mlx/dense.py:109-167 ScaledLinear): a weight is code * scale * d,
// the code a signed byte (the block's six bits less 32), a signed byte scale to every 16 weights of a row, a
// float16 d to every d_step (256, or fewer where the inputs were reordered). 8.56 bits a weight.
//
//   scaled_matvec_kernel  out[t] = W . x[t] for a window of up to 8 tokens: warps over rows, a lane's row chunks of 16
//                         codes requested together, the activations staged in shared memory, float32 sums
//                         reduced across the warp
//   scaled_mma_kernel     the same for float16 / bfloat16 activations on mma.sync: codes made exact small integers
//                         of the activations' type, a 16-weight scale group per m16n8k16 step
//   scaled_floats_kernel  every weight as a float of the output type, worked out in float32 as the reference does
//                         (float(d) * float(scale), times float(code)) and rounded once (dense.py:73-82)
#include <algorithm>

#include "decode.cuh"
#include "mma_decode.cuh"

namespace sc {

constexpr int SC_DENSE_MAX_TOKENS = 8;  // dense.py:33 MAX_TOKENS: more is a chunk of a prompt, multiplied as floats
constexpr int SCL_WARPS = 8;
constexpr int SCL_AHEAD = 8;              // 16-byte chunks of codes a lane has in flight: a 4096-wide row
constexpr int SCL_STAGE_MAX = 96 * 1024;  // activations staged in shared memory up to this many bytes

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

// int8 code -> float exactly without a conversion instruction (those run at a quarter of the FMA rate): the byte,
// its sign bit flipped (code + 128), as the low mantissa byte of 2^23, less 2^23 + 128
__device__ __forceinline__ float code_f(uint32_t flipped_word, int i) {
  return __uint_as_float(__byte_perm(flipped_word, 0x4B000000u, uint32_t(i) | 0x7540u)) - 8388736.0f;
}

// xs: the window's activations as float32 (tokens, cols) in shared memory when `staged`, else read from x directly.
// Warps go over rows (persistent: the grid is two blocks an SM); a lane asks for SCL_AHEAD chunks of 16 codes (and
// their scale bytes and d) before it uses any, so that a whole 4096-wide row is on its way at once. TT: the tokens
// the registers are laid out for (1, 2, 4 or 8; tokens <= TT).
template <typename T, int TT>
__global__ void __launch_bounds__(SCL_WARPS * 32, 2) scaled_matvec_kernel(const int8_t* __restrict__ codes,
                                                                         const int8_t* __restrict__ scales,
                                                                         const __half* __restrict__ d, int rows,
                                                                         int cols, int d_step, const T* __restrict__ x,
                                                                         int tokens, int staged, T* __restrict__ out) {
  extern __shared__ float xs[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (staged) {  // 16-byte pieces, four a thread in flight at once
    constexpr int E = 16 / int(sizeof(T));
    const int n16 = tokens * cols / E;
    for (int i0 = threadIdx.x; i0 < n16; i0 += 4 * blockDim.x) {
      uint4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (i0 + j * int(blockDim.x) < n16) v[j] = __ldg(reinterpret_cast<const uint4*>(x) + i0 + j * blockDim.x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j * int(blockDim.x);
        if (i < n16) {
          const T* h = reinterpret_cast<const T*>(&v[j]);
#pragma unroll
          for (int k = 0; k < E; ++k) xs[i * E + k] = to_f32(h[k]);
        }
      }
    }
    __syncthreads();
  }
  for (int r = blockIdx.x * SCL_WARPS + warp; r < rows; r += gridDim.x * SCL_WARPS) {
    const int8_t* cr = codes + int64_t(r) * cols;
    const int8_t* sr = scales + int64_t(r) * (cols / 16);
    const __half* dr = d + int64_t(r) * (cols / d_step);
    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[t] = 0.f;
    for (int c0 = 16 * lane; c0 < cols; c0 += 16 * 32 * SCL_AHEAD) {
      int4 q[SCL_AHEAD];
      int8_t sb[SCL_AHEAD];
      __half db[SCL_AHEAD];
#pragma unroll
      for (int u = 0; u < SCL_AHEAD; ++u) {
        const int c = c0 + 16 * 32 * u;
        if (c < cols) {
          q[u] = __ldcs(reinterpret_cast<const int4*>(cr + c));  // read once: streaming
          sb[u] = sr[c / 16];
          db[u] = dr[c / d_step];
        }
      }
#pragma unroll
      for (int u = 0; u < SCL_AHEAD; ++u) {
        const int c = c0 + 16 * 32 * u;
        if (c >= cols) break;
        const float sc = __half2float(db[u]) * float(sb[u]);
        const uint32_t qw[4] = {uint32_t(q[u].x) ^ 0x80808080u, uint32_t(q[u].y) ^ 0x80808080u,
                                uint32_t(q[u].z) ^ 0x80808080u, uint32_t(q[u].w) ^ 0x80808080u};
        float w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = code_f(qw[i >> 2], i & 3);
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          if (t < tokens) {
            float xv[16];
            if (staged) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float4 f = *reinterpret_cast<const float4*>(xs + t * cols + c + 4 * j);
                xv[4 * j] = f.x, xv[4 * j + 1] = f.y, xv[4 * j + 2] = f.z, xv[4 * j + 3] = f.w;
              }
            } else {
              load16<T>(x + int64_t(t) * cols + c, xv);
            }
            float p = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) p = fmaf(w[i], xv[i], p);
            acc[t] = fmaf(sc, p, acc[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (t < tokens) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) out[int64_t(t) * rows + r] = from_f32<T>(v);
      }
    }
  }
}

// ---- the window on the tensor cores, for float16 / bfloat16 activations (whose values the MMA takes exactly)
//
// A block takes 16 rows: their codes (one bulk copy a row, into rows padded by 16 bytes so that the fragment loads
// fall on distinct banks) and scales by bulk copies, d and the activations by loads. Eight warps split the row's
// 16-weight groups; a group is one m16n8k16 step: lane (g, t) holds weights 4t .. 4t + 3 of the group for rows g and
// g + 8 (one 4-byte load each), the activations' columns 4t .. 4t + 3 for token g (one 8-byte load), the codes made
// exact small integers of the activations' type (code + 32, the block's six bits, in the mantissa next to a
// power-of-two bias that is then taken off), float32 sums; the group's scale * d multiplies the step's partial sums.
// The warps' sums are added in order through shared memory.
constexpr int SMMA_ROWS = 16, SMMA_WARPS = 8;

struct SmmaSmem {
  int bar, codes, cstride, scales, d, sfl, xs, red, total;
};

__host__ __device__ inline SmmaSmem smma_smem(int cols, int d_step, int tokens) {
  SmmaSmem s;
  int o = 0;
  s.bar = o; o += 16 * (SMMA_WARPS + 1);
  s.cstride = cols + 16;
  s.codes = o; o += SMMA_ROWS * s.cstride;
  s.scales = o; o += align16(SMMA_ROWS * (cols / 16));
  s.d = o; o += align16(SMMA_ROWS * (cols / d_step) * 2);
  // scale * d of every row's groups, float32, rows sfl_stride() apart: a stride of 4 words more than the groups, so
  // that the eight rows a warp's lanes read at once fall on different banks (256 groups: all on one otherwise)
  s.sfl = o; o += SMMA_ROWS * (cols / 16 + 4) * 4;
  s.xs = o; o += align16(tokens * cols * 2);
  s.red = o; o += SMMA_WARPS * 32 * 4 * 4;
  s.total = o;
  return s;
}

template <typename T>
__global__ void __launch_bounds__(SMMA_WARPS * 32) scaled_mma_kernel(const int8_t* __restrict__ codes,
                                                                    const int8_t* __restrict__ scales,
                                                                    const __half* __restrict__ d, int rows, int cols,
                                                                    int d_step, const T* __restrict__ x, int tokens,
                                                                    T* __restrict__ out, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const SmmaSmem S = smma_smem(cols, d_step, tokens);
  // bars[0]: the block's rows of codes, one bulk copy a row (into rows padded by 16 bytes: the eight rows a warp's
  // lanes read at once fall on different banks); bars[1]: their scales. One copy a row, not one a warp's column
  // slice of a row: the copy engine's cost per copy, not the bytes, had set the kernel's pace.
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.bar);
  const int r0 = blockIdx.x * SMMA_ROWS, nrow = min(SMMA_ROWS, rows - r0);
  const int groups = cols / 16, dper = cols / d_step, gper = d_step / 16;
  const int j0 = warp * groups / SMMA_WARPS, j1 = (warp + 1) * groups / SMMA_WARPS;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars[1], uint32_t(nrow * groups));
      bulk_load(smem + S.scales, scales + int64_t(r0) * groups, uint32_t(nrow * groups), &bars[1]);
      mbar_arrive_expect_tx(&bars[0], uint32_t(nrow) * uint32_t(cols));
    }
    __syncwarp();
    if (lane < nrow)
      bulk_load(smem + S.codes + lane * S.cstride, codes + int64_t(r0 + lane) * cols, uint32_t(cols), &bars[0]);
  }
  // the next kernel of the stream (the next layer, launched the same way) may fetch its weights from now on; it
  // reads this one's output only after its own wait below
  pdl_launch_dependents();
  __half* dsm = reinterpret_cast<__half*>(smem + S.d);
  for (int i = tid; i < nrow * dper; i += blockDim.x) dsm[i] = d[int64_t(r0) * dper + i];
  __syncthreads();
  bool ok = mbar_wait_sleep(&bars[1], 0, err);
  float* sfl = reinterpret_cast<float*>(smem + S.sfl);
  const int8_t* ssm = reinterpret_cast<const int8_t*>(smem + S.scales);
  const int gshift = __ffs(gper) - 1;  // d_step / 16, a power of two
  const int fstride = groups + 4;
  for (int rr = 0; rr < nrow; ++rr)
    for (int j = tid; j < groups; j += blockDim.x)
      sfl[rr * fstride + j] = __half2float(dsm[rr * dper + (j >> gshift)]) * float(ssm[rr * groups + j]);
  pdl_wait();  // the activations: the previous kernel's output
  T* xs = reinterpret_cast<T*>(smem + S.xs);
  for (int i = tid; i < tokens * cols / 8; i += blockDim.x)
    reinterpret_cast<uint4*>(xs)[i] = __ldcg(reinterpret_cast<const uint4*>(x) + i);
  __syncthreads();
  ok = ok && mbar_wait_sleep(&bars[0], 0, err);

  const int g = lane >> 2, t = lane & 3;
  const uint8_t* ca = smem + S.codes + g * S.cstride + 4 * t;
  const uint8_t* cb = ca + 8 * S.cstride;
  const float* sa = sfl + g * fstride;
  const float* sb = sa + 8 * fstride;  // rows past nrow: stale values, in rows never written out
  const bool mine = g < tokens;
  const T* xg = xs + g * cols + 4 * t;
  constexpr uint32_t HI = Bias<T>::hi * 0x01010101u, SUB = Bias<T>::pair + 0x00200020u;  // bias + 32: code + 32 - it
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (ok) {
#pragma unroll 4
    for (int j = j0; j < j1; ++j) {
      const uint32_t ua = (*reinterpret_cast<const uint32_t*>(ca + 16 * j) & 0x3F3F3F3Fu) ^ 0x20202020u;  // code + 32
      const uint32_t ub = (*reinterpret_cast<const uint32_t*>(cb + 16 * j) & 0x3F3F3F3Fu) ^ 0x20202020u;
      const uint32_t a[4] = {sub2<T>(__byte_perm(ua, HI, 0x5140), SUB), sub2<T>(__byte_perm(ub, HI, 0x5140), SUB),
                             sub2<T>(__byte_perm(ua, HI, 0x7362), SUB), sub2<T>(__byte_perm(ub, HI, 0x7362), SUB)};
      uint2 xv = make_uint2(0, 0);
      if (mine) xv = *reinterpret_cast<const uint2*>(xg + 16 * j);
      float dd[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816<T>(dd, a, xv.x, xv.y);
      const float s0 = sa[j], s1 = sb[j];
      acc[0] = fmaf(s0, dd[0], acc[0]);
      acc[1] = fmaf(s0, dd[1], acc[1]);
      acc[2] = fmaf(s1, dd[2], acc[2]);
      acc[3] = fmaf(s1, dd[3], acc[3]);
    }
  }
  float* red = reinterpret_cast<float*>(smem + S.red);  // [value][warp][lane]
#pragma unroll
  for (int q = 0; q < 4; ++q) red[(q * SMMA_WARPS + warp) * 32 + lane] = acc[q];
  __syncthreads();
  if (tid < 128) {
    const int q = tid >> 5, L = tid & 31;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < SMMA_WARPS; ++w) v += red[(q * SMMA_WARPS + w) * 32 + L];
    const int m = (q < 2 ? 0 : 8) + (L >> 2), tok = 2 * (L & 3) + (q & 1);  // C fragment: rows g, g + 8; tokens 2t, 2t + 1
    if (m < nrow && tok < tokens) out[int64_t(tok) * rows + r0 + m] = from_f32<T>(v);
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
                                const void* x, int dtype, int tokens, void* out, int* err, void* stream) {
  if (int rc = scaled_check(codes, scales, d, rows, cols, d_step)) return rc;
  if (!x || !out || tokens < 0) return SC_ERR_ARG;
  if (tokens > SC_DENSE_MAX_TOKENS) return SC_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) & 15)) return SC_ERR_ALIGN;
  if (rows == 0 || tokens == 0) return SC_OK;
  if (dtype == SC_F16 || dtype == SC_BF16) {  // the tensor cores, where the block's rows fit shared memory
    const int smem = smma_smem(cols, d_step, tokens).total;
    if (smem <= 200 * 1024 && (reinterpret_cast<uintptr_t>(scales) & 15) == 0 && (d_step & (d_step - 1)) == 0) {
      cudaError_t e = cudaSuccess;
      dispatch_dtype(dtype, [&]<typename T>() {
        if constexpr (sizeof(T) == 2) {
          auto kern = scaled_mma_kernel<T>;
          e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
          if (e == cudaSuccess) {
            // programmatic dependent launch: the weights' copies go out while the kernel before finishes
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(unsigned(ceil_div(rows, SMMA_ROWS)));
            cfg.blockDim = dim3(SMMA_WARPS * 32);
            cfg.dynamicSmemBytes = size_t(smem);
            cfg.stream = static_cast<cudaStream_t>(stream);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaLaunchKernelEx(&cfg, kern, static_cast<const int8_t*>(codes), static_cast<const int8_t*>(scales),
                                   static_cast<const __half*>(d), rows, cols, d_step, static_cast<const T*>(x),
                                   tokens, static_cast<T*>(out), err);
          }
        }
      });
      if (e != cudaSuccess) return SC_ERR_CUDA;
      return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
    }
  }
  const int grid = int(std::min<int64_t>(ceil_div(rows, SCL_WARPS), 2 * 148));
  const int64_t xbytes = int64_t(tokens) * cols * 4;
  const int staged = xbytes <= SCL_STAGE_MAX ? 1 : 0;
  const int smem = staged ? int(xbytes) : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  const bool ok = dispatch_dtype(dtype, [&]<typename T>() {
    auto kern = tokens == 1   ? scaled_matvec_kernel<T, 1>
                : tokens == 2 ? scaled_matvec_kernel<T, 2>
                : tokens <= 4 ? scaled_matvec_kernel<T, 4>
                              : scaled_matvec_kernel<T, SC_DENSE_MAX_TOKENS>;
    if (smem > 48 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SCL_STAGE_MAX);
    if (e == cudaSuccess)
      kern<<<grid, SCL_WARPS * 32, smem, s>>>(static_cast<const int8_t*>(codes), static_cast<const int8_t*>(scales),
                                            static_cast<const __half*>(d), rows, cols, d_step,
                                            static_cast<const T*>(x), tokens, staged, static_cast<T*>(out));
  });
  if (e != cudaSuccess) return SC_ERR_CUDA;
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
