// The block decoders: run n (32 weights) of a row of GGUF blocks -> 32 float32 weights, each computed with
// the float32 operations, in the order, of strata-mlx's unpack32 bodies (strata_mlx/blocks.py:57-193) --
// explicit __fmul_rn/__fadd_rn so that nothing is contracted -- hence bit for bit the reference's weights.
#pragma once

#include "common.cuh"

namespace sc {

__device__ __forceinline__ float neg_if(float v, uint32_t bit) { return bit ? -v : v; }

// the k-th of a Q3_K block's sixteen 6-bit scales, less 32 (strata_mlx/blocks.py:48-53)
__device__ __forceinline__ float q3k_scale(const uint8_t* s, uint32_t k) {
  uint32_t p = k % 4, word = k / 4;
  uint32_t low = word < 2 ? (uint32_t(s[4 * word + p]) & 15) : (uint32_t(s[4 * (word - 2) + p]) >> 4);
  return float(int(low | (((uint32_t(s[8 + p]) >> (2 * word)) & 3) << 4)) - 32);
}

template <int KIND>
__device__ __forceinline__ void unpack32(const uint8_t* row, int n, float* w, const Tabs& t) {
  if constexpr (KIND == SC_Q2_0) {  // blocks.py:58-67
    const uint8_t* b = row + (n / 2) * 18;
    const uint8_t* q = b + 2 + 8 * (n % 2);
    const float d = half_at(b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t c = q[i];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[4 * i + j] = __fmul_rn(d, float((c >> (2 * j)) & 3) - 1.0f);
    }
  } else if constexpr (KIND == SC_IQ4_NL) {  // blocks.py:69-77
    const uint8_t* b = row + n * 18;
    const float d = half_at(b);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t q = b[2 + i];
      w[i] = __fmul_rn(d, float(t.kvalues[q & 15]));
      w[16 + i] = __fmul_rn(d, float(t.kvalues[q >> 4]));
    }
  } else if constexpr (KIND == SC_IQ4_XS) {  // blocks.py:78-88
    const uint8_t* b = row + (n / 8) * 136;
    const uint32_t ib = n % 8;
    const uint32_t ls = ((uint32_t(b[4 + ib / 2]) >> (4 * (ib % 2))) & 15) | (((u16_at(b + 2) >> (2 * ib)) & 3) << 4);
    const float d = __fmul_rn(half_at(b), float(ls) - 32.0f);
    const uint8_t* q = b + 8 + 16 * ib;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t v = q[i];
      w[i] = __fmul_rn(d, float(t.kvalues[v & 15]));
      w[16 + i] = __fmul_rn(d, float(t.kvalues[v >> 4]));
    }
  } else if constexpr (KIND == SC_IQ3_S) {  // blocks.py:89-101
    const uint8_t* b = row + (n / 8) * 110;
    const uint32_t ib = n % 8;
    const float d = __fmul_rn(half_at(b), float(1 + 2 * ((uint32_t(b[106 + ib / 2]) >> (4 * (ib % 2))) & 15)));
    const uint32_t high = b[66 + ib];
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const uint32_t g = t.iq3s[uint32_t(b[2 + 8 * ib + l]) | (((high >> l) & 1) << 8)];
      const uint32_t sign = uint32_t(b[74 + 4 * ib + l / 2]) >> (4 * (l % 2));
#pragma unroll
      for (int j = 0; j < 4; ++j) w[4 * l + j] = neg_if(__fmul_rn(d, float((g >> (8 * j)) & 255)), (sign >> j) & 1);
    }
  } else if constexpr (KIND == SC_IQ3_XXS) {  // blocks.py:103-115
    const uint8_t* b = row + (n / 8) * 98;
    const uint32_t ib = n % 8;
    const uint32_t aux = u32_at(b + 66 + 4 * ib);
    const float d = __fmul_rn(__fmul_rn(half_at(b), __fadd_rn(0.5f, float(aux >> 28))), 0.5f);
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const uint32_t g = t.iq3xxs[b[2 + 8 * ib + l]];
      const uint32_t sign = uint32_t(t.ksigns[(aux >> (7 * (l / 2))) & 127]) >> (4 * (l % 2));
#pragma unroll
      for (int j = 0; j < 4; ++j) w[4 * l + j] = neg_if(__fmul_rn(d, float((g >> (8 * j)) & 255)), (sign >> j) & 1);
    }
  } else if constexpr (KIND == SC_IQ2_S) {  // blocks.py:117-131
    const uint8_t* b = row + (n / 8) * 82;
    const uint32_t ib = n % 8;
    const float d = __fmul_rn(half_at(b), 0.25f);
    const uint32_t high = b[66 + ib], scales = b[74 + ib];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const uint64_t g = t.iq2s[uint32_t(b[2 + 4 * ib + l]) | (((high >> (2 * l)) & 3) << 8)];
      const uint32_t sign = b[34 + 4 * ib + l];
      const float dl = __fmul_rn(d, __fadd_rn(0.5f, float(l < 2 ? scales & 15 : scales >> 4)));
#pragma unroll
      for (int j = 0; j < 8; ++j) w[8 * l + j] = neg_if(__fmul_rn(dl, float((g >> (8 * j)) & 255)), (sign >> j) & 1);
    }
  } else if constexpr (KIND == SC_IQ2_XS) {  // blocks.py:132-147
    const uint8_t* b = row + (n / 8) * 74;
    const uint32_t ib = n % 8;
    const float d = __fmul_rn(half_at(b), 0.25f);
    const uint32_t scales = b[66 + ib];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const uint32_t q = u16_at(b + 2 + 2 * (4 * ib + l));
      const uint64_t g = t.iq2xs[q & 511];
      const uint32_t sign = t.ksigns[q >> 9];
      const float dl = __fmul_rn(d, __fadd_rn(0.5f, float(l < 2 ? scales & 15 : scales >> 4)));
#pragma unroll
      for (int j = 0; j < 8; ++j) w[8 * l + j] = neg_if(__fmul_rn(dl, float((g >> (8 * j)) & 255)), (sign >> j) & 1);
    }
  } else if constexpr (KIND == SC_IQ2_XXS) {  // blocks.py:148-161
    const uint8_t* b = row + (n / 8) * 66;
    const uint8_t* q = b + 2 + 8 * (n % 8);
    const uint32_t aux = u32_at(q + 4);
    const float d = __fmul_rn(__fmul_rn(half_at(b), __fadd_rn(0.5f, float(aux >> 28))), 0.25f);
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const uint64_t g = t.iq2xxs[q[l]];
      const uint32_t sign = t.ksigns[(aux >> (7 * l)) & 127];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[8 * l + j] = neg_if(__fmul_rn(d, float((g >> (8 * j)) & 255)), (sign >> j) & 1);
    }
  } else if constexpr (KIND == SC_Q3_K) {  // blocks.py:164-175
    const uint8_t* b = row + (n / 8) * 110;
    const uint32_t r = n % 8;
    const uint8_t* q = b + 32 + 32 * (r / 4);
    const uint32_t shift = 2 * (r % 4);
    const float d = half_at(b + 108);
    const float s0 = __fmul_rn(d, q3k_scale(b + 96, 2 * r)), s1 = __fmul_rn(d, q3k_scale(b + 96, 2 * r + 1));
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int v = int((uint32_t(q[i]) >> shift) & 3) - (((uint32_t(b[i]) >> r) & 1) ? 0 : 4);
      w[i] = __fmul_rn(i < 16 ? s0 : s1, float(v));
    }
  } else if constexpr (KIND == SC_IQ1_M) {  // blocks.py:176-193
    const uint8_t* b = row + (n / 8) * 56;
    const uint32_t ib = n % 8;
    const uint32_t packed = (u16_at(b + 48) >> 12) | ((u16_at(b + 50) >> 8) & 0x00f0) | ((u16_at(b + 52) >> 4) & 0x0f00) |
                            (u16_at(b + 54) & 0xf000);
    const float d = half_bits(packed);
    const uint32_t scales = u16_at(b + 48 + 2 * (ib / 2)) >> (6 * (ib % 2));
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const uint32_t high = (uint32_t(b[32 + 2 * ib + l / 2]) >> (4 * (l % 2))) & 15;
      const uint64_t g = t.iq1[uint32_t(b[4 * ib + l]) | ((high & 7) << 8)];
      const float dl = __fmul_rn(d, float(2 * ((scales >> (3 * (l / 2))) & 7) + 1));
      const float delta = (high & 8) ? -1.125f : -0.875f;
#pragma unroll
      for (int j = 0; j < 8; ++j) w[8 * l + j] = __fmul_rn(dl, __fadd_rn(float((g >> (8 * j)) & 255), delta));
    }
  } else if constexpr (KIND == SC_Q8_0) {  // strata_mlx/gguf.py:203-206: d * int8 code
    const uint8_t* b = row + n * 34;
    const float d = half_at(b);
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = __fmul_rn(d, float(int8_t(b[2 + i])));
  }
}

// Calls f.template operator()<KIND>() for the runtime block type `kind`; returns false for an unknown one.
template <typename F>
__host__ bool dispatch_kind(int kind, F&& f) {
  switch (kind) {
    case SC_Q2_0: f.template operator()<SC_Q2_0>(); return true;
    case SC_IQ4_NL: f.template operator()<SC_IQ4_NL>(); return true;
    case SC_IQ4_XS: f.template operator()<SC_IQ4_XS>(); return true;
    case SC_IQ3_S: f.template operator()<SC_IQ3_S>(); return true;
    case SC_IQ3_XXS: f.template operator()<SC_IQ3_XXS>(); return true;
    case SC_IQ2_S: f.template operator()<SC_IQ2_S>(); return true;
    case SC_IQ2_XS: f.template operator()<SC_IQ2_XS>(); return true;
    case SC_IQ2_XXS: f.template operator()<SC_IQ2_XXS>(); return true;
    case SC_IQ1_M: f.template operator()<SC_IQ1_M>(); return true;
    case SC_Q3_K: f.template operator()<SC_Q3_K>(); return true;
    case SC_Q8_0: f.template operator()<SC_Q8_0>(); return true;
    default: return false;
  }
}

template <typename F>
__host__ bool dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case SC_F32: f.template operator()<float>(); return true;
    case SC_F16: f.template operator()<__half>(); return true;
    case SC_BF16: f.template operator()<__nv_bfloat16>(); return true;
    default: return false;
  }
}

}  // namespace sc
