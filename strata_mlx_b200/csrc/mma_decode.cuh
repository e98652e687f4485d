// Block decode straight into tensor-core fragments (mma.sync m16n8k16, bf16 or f16 operands, f32 accumulate).
//
// A warp multiplies 16 weight rows by up to 8 token vectors, one run of 32 weights (two k-steps of 16) at a
// time. Lane (g = lane / 4, t = lane % 4) owns weights 8t .. 8t+7 of the run for rows g and g + 8. Those eight
// weights are decoded as exact small integers -- a code or a grid value with its sign, e.g. Q2_0's c - 1 or
// IQ3_S's +-g -- written into the mantissa of a 16-bit float next to a power-of-two bias (128 for bf16, 1024 for
// f16, where one unit of the mantissa is 1), and the bias subtracted exactly; the per-run scale (d, or d times the
// run's scale) is applied to the run's f32 partial sums. Products and sums are then those of a float32
// accumulation of the reference's weights, to the tensor core's f32 rounding.
//
// The k order inside a lane's eight weights is (0,4) (1,5) (2,6) (3,7): register pair q holds weights q and q+4,
// which makes the byte-to-pair moves one PRMT each. Activations are staged in shared memory in that same order
// (stage_x_permuted), so that a 16-byte load gives a lane both k-steps' B fragments.
#pragma once

#include "common.cuh"

namespace sc {

template <typename T> struct Bias;
template <> struct Bias<__nv_bfloat16> {
  static constexpr uint32_t pair = 0x43004300u;  // bf16 128.0 in both halves: the mantissa's unit is 1
  static constexpr uint32_t hi = 0x43u;
  __device__ static __nv_bfloat162 minus(float v) { return __floats2bfloat162_rn(v, v); }
};
template <> struct Bias<__half> {
  static constexpr uint32_t pair = 0x64006400u;  // f16 1024.0
  static constexpr uint32_t hi = 0x64u;
  __device__ static __half2 minus(float v) { return __floats2half2_rn(v, v); }
};

template <typename T> __device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b);
template <> __device__ __forceinline__ uint32_t sub2<__nv_bfloat16>(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
template <> __device__ __forceinline__ uint32_t sub2<__half>(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&r);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 r = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&r);
}

// d += A . B on the tensor cores, A 16x16 (four registers), B 16x8 (two), D 16x8 f32 (four)
template <typename T> __device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <> __device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <> __device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// sign bits q and q+4 of a lane's sign byte -> bits 15 and 31 (the signs of register pair q)
__device__ __forceinline__ uint32_t flip_signs(uint32_t v, uint32_t sbyte, int q) {
  const uint32_t m = sbyte * ((1u << (15 - q)) | (1u << (27 - q)));
  return v ^ (m & 0x80008000u);
}

// bytes q of grid entries a and b -> the pair (bias + a_q, bias + b_q) as two 16-bit floats
template <typename T>
__device__ __forceinline__ uint32_t grid_pair(uint32_t a, uint32_t b, int q) {
  const uint32_t v = __byte_perm(a, b, uint32_t(q) | (uint32_t(4 + q) << 4));  // bytes 0, 1 = a_q, b_q
  return __byte_perm(v, Bias<T>::hi * 0x01010101u, 0x5140);                   // [a_q, hi, b_q, hi]
}

// Types with a fragment decoder. dec8 fills p[q] = weight pair (q, q+4) of the lane's eight weights of run n of a
// row, as 16-bit floats without their scale, and returns the run's scale (the weight is scale * value).
template <int KIND> struct HasMma { static constexpr bool value = KIND == SC_Q2_0 || KIND == SC_IQ3_S || KIND == SC_IQ3_XXS; };

template <int KIND, typename T>
__device__ __forceinline__ float dec8(const uint8_t* row, int n, int t, const uint32_t* grid, uint32_t (&p)[4]) {
  if constexpr (KIND == SC_Q2_0) {  // strata_mlx/blocks.py:58-67: w = d * (code - 1), a block of 64 = two runs
    const uint8_t* b = row + (n >> 1) * 18;
    const float d = half_bits(ld_u16(b));
    const uint32_t v = ld_u16(b + 2 + 8 * (n & 1) + 2 * t);  // codes of weights 8t .. 8t+7, two bits each
    const uint32_t u = __byte_perm(v, 0, 0x4140);              // [byte0, 0, byte1, 0]: pair q = (code q, code q+4)
    const uint32_t bias_plus_one = Bias<T>::pair + 0x00010001u;  // 129 (bf16) or 1025 (f16): code - 1
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = sub2<T>(((u >> (2 * q)) & 0x00030003u) | Bias<T>::pair, bias_plus_one);
    return d;
  } else if constexpr (KIND == SC_IQ3_S) {  // blocks.py:89-101
    const uint8_t* b = row + (n >> 3) * 110;
    const int ib = n & 7;
    const float d = half_bits(ld_u16(b)) * float(1 + 2 * ((uint32_t(b[106 + (ib >> 1)]) >> (4 * (ib & 1))) & 15));
    const uint32_t qs = ld_u16(b + 2 + 8 * ib + 2 * t);        // grid indices of entries 2t, 2t+1 (low 8 bits)
    const uint32_t qh = uint32_t(b[66 + ib]) >> (2 * t);       // their ninth bits
    const uint32_t s8 = b[74 + 4 * ib + t];                    // signs of weights 8t .. 8t+7
    const uint32_t ga = grid[(qs & 0xffu) | ((qh & 1u) << 8)];
    const uint32_t gb = grid[(qs >> 8) | ((qh & 2u) << 7)];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = flip_signs(sub2<T>(grid_pair<T>(ga, gb, q), Bias<T>::pair), s8, q);
    return d;
  } else if constexpr (KIND == SC_IQ3_XXS) {  // blocks.py:103-115
    const uint8_t* b = row + (n >> 3) * 98;
    const int ib = n & 7;
    const uint32_t aux = ld_u16(b + 66 + 4 * ib) | (ld_u16(b + 68 + 4 * ib) << 16);
    const float d = half_bits(ld_u16(b)) * (0.5f + float(aux >> 28)) * 0.5f;
    const uint32_t qs = ld_u16(b + 2 + 8 * ib + 2 * t);
    const uint32_t k7 = (aux >> (7 * t)) & 127u;               // ksigns[k7] = k7 with its parity as bit 7
    const uint32_t s8 = k7 | ((__popc(k7) & 1u) << 7);
    const uint32_t ga = grid[qs & 0xffu];
    const uint32_t gb = grid[qs >> 8];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = flip_signs(sub2<T>(grid_pair<T>(ga, gb, q), Bias<T>::pair), s8, q);
    return d;
  } else {
    return 0.f;
  }
}

// Activations (tokens, cols) of T into shared memory, each group of eight reordered (0,4,1,5,2,6,3,7) so that
// lane t's 16-byte load at column 32n + 8t yields the B fragments of run n's two k-steps; rows `stride`
// elements apart. Called by `nthreads` threads of the block starting at `tid`.
template <typename T>
__device__ __forceinline__ void stage_x_permuted(const T* __restrict__ x, int tokens, int cols, T* xs, int stride, int tid,
                                                 int nthreads) {
  const int groups = cols / 8;
  for (int i = tid; i < tokens * groups; i += nthreads) {
    const int tok = i / groups, gidx = i % groups;
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(x + int64_t(tok) * cols + 8 * gidx));  // another kernel's output
    uint4 o;
    o.x = __byte_perm(v.x, v.z, 0x5410);  // (0, 4)
    o.y = __byte_perm(v.x, v.z, 0x7632);  // (1, 5)
    o.z = __byte_perm(v.y, v.w, 0x5410);  // (2, 6)
    o.w = __byte_perm(v.y, v.w, 0x7632);  // (3, 7)
    *reinterpret_cast<uint4*>(xs + tok * stride + 8 * gidx) = o;
  }
}

}  // namespace sc
