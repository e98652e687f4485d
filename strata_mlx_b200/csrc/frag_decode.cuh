// Block decode straight into mma.sync fragments (m16n8k16, bf16 or f16 operands, f32 accumulate), as the decode
// block's kernels use it: a warp's 16 weight rows (g and g + 8 for lane g = lane / 4, t = lane % 4) times up to 8
// tokens over a range of runs of 32 weights, four runs an iteration.
//
// Every weight enters the tensor core as an exact small integer of the activations' type, its block's scale applied
// to the run's float32 sums afterwards, so that products and sums are those of a float32 accumulation of the
// reference's weights (strata_mlx/blocks.py:57-115), to the tensor core's rounding:
//   Q2_0     (blocks.py:58-67) w = d (c - 1): the 2-bit code c is masked into the mantissa next to a power-of-two
//            bias B (one LOP3 a register of two weights, the code at bits 2q where B's mantissa unit is 1), and
//            B + 1 taken off in one exact 16-bit add: c - 1. A lane's register q holds weights q and q + 4 of its
//            eight (both codes sit at bits 2q of the two code bytes); activations are staged in that order
//            (x_pairs). A block's d scales the float32 sums of its two runs at once.
//   IQ3_S    (blocks.py:89-101) and IQ3_XXS (:103-115): the grid entry's four values are read as four 16-bit
//            floats from an expanded codebook in shared memory (one 8-byte load an entry), the signs XORed into
//            bits 15 and 31 (an IMAD and a LOP3 a register); registers hold weights (0,1) (2,3) (4,5) (6,7) of the
//            lane's eight, activations staged in their natural order. The run's scale d (1 + 2 s) or d (0.5 + s) / 2
//            is worked out once by lane t for run n + t and taken by the others with a shuffle.
#pragma once

#include "mma_decode.cuh"

namespace sc {

// the order a kind's decoder wants the activations in: pairs (0,4,1,5,2,6,3,7 in each group of eight) or natural
__host__ __device__ constexpr bool x_pairs(int kind) { return kind == SC_Q2_0; }

// Activations (tokens, cols) of T into shared memory in the order `pairs` asks, rows `stride` elements apart. Called
// by `nthreads` threads from `tid`.
template <typename T>
__device__ __forceinline__ void stage_x(const T* __restrict__ x, int tokens, int cols, T* xs, int stride, int tid,
                                        int nthreads, bool pairs) {
  if (pairs) {
    stage_x_permuted<T>(x, tokens, cols, xs, stride, tid, nthreads);
    return;
  }
  const int groups = cols / 8;
  for (int i = tid; i < tokens * groups; i += nthreads) {
    const int tok = i / groups, gidx = i % groups;
    *reinterpret_cast<uint4*>(xs + tok * stride + 8 * gidx) =
        __ldcg(reinterpret_cast<const uint4*>(x + int64_t(tok) * cols + 8 * gidx));
  }
}

// where value r of a row (0 <= r < cols) sits in the order `pairs` asks
__device__ __forceinline__ int x_col(int r, bool pairs) {
  if (!pairs) return r;
  const int j = r & 7;
  return (r & ~7) + (j < 4 ? 2 * j : 2 * (j - 4) + 1);
}

// The expanded codebooks in shared memory: IQ3_S's 512 entries, then IQ3_XXS's 256, each four values of T (8 bytes).
constexpr int GRID_TAB_BYTES = (512 + 256) * 8;

template <typename T>
__device__ __forceinline__ void build_grid_tabs(uint2* tab, int tid, int nthreads) {
  for (int i = tid; i < 512 + 256; i += nthreads) {
    const uint32_t g = i < 512 ? IQ3S_GRID[i] : IQ3XXS_GRID[i - 512];
    const T v0 = from_f32<T>(float(g & 255)), v1 = from_f32<T>(float((g >> 8) & 255));
    const T v2 = from_f32<T>(float((g >> 16) & 255)), v3 = from_f32<T>(float(g >> 24));
    uint2 e;
    e.x = uint32_t(*reinterpret_cast<const uint16_t*>(&v0)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&v1)) << 16);
    e.y = uint32_t(*reinterpret_cast<const uint16_t*>(&v2)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&v3)) << 16);
    tab[i] = e;
  }
}
template <int KIND>
__device__ __forceinline__ const uint2* grid_tab(const uint2* tabs) {
  return KIND == SC_IQ3_XXS ? tabs + 512 : tabs;
}

// One kind's codebook in REP copies, entry i of copy c at i * REP + c: a lane that reads copy lane % REP from
// rep_tab(tab, lane) finds its entry in its own pair of banks (REP = 16: a warp's eight-byte loads take the two
// passes they must, whatever the entries). REP * entries * 8 bytes.
template <int KIND> constexpr int grid_entries() { return KIND == SC_IQ3_XXS ? 256 : 512; }

template <typename T, int KIND, int REP>
__device__ __forceinline__ void build_grid_tab_rep(uint2* tab, int tid, int nthreads) {
  for (int i = tid; i < grid_entries<KIND>() * REP; i += nthreads) {
    const int e = i / REP;
    const uint32_t g = KIND == SC_IQ3_XXS ? IQ3XXS_GRID[e] : IQ3S_GRID[e];
    const T v0 = from_f32<T>(float(g & 255)), v1 = from_f32<T>(float((g >> 8) & 255));
    const T v2 = from_f32<T>(float((g >> 16) & 255)), v3 = from_f32<T>(float(g >> 24));
    uint2 w;
    w.x = uint32_t(*reinterpret_cast<const uint16_t*>(&v0)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&v1)) << 16);
    w.y = uint32_t(*reinterpret_cast<const uint16_t*>(&v2)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&v3)) << 16);
    tab[i] = w;
  }
}
template <int REP>
__device__ __forceinline__ const uint2* rep_tab(const uint2* tab, int lane) {
  return tab + (lane % REP);
}

// One IQ3 kind's codebook replicated REP times (rep_tab's layout), built by `nthreads` threads from `tid`: each
// thread expands an entry once and stores it into two adjacent copies with one 16-byte store.
template <typename T, int KIND, int REP>
__device__ __forceinline__ void build_grid_tab_rep2(uint2* tab, int tid, int nthreads) {
  static_assert(REP % 2 == 0, "copies are stored in pairs");
  for (int i = tid; i < grid_entries<KIND>() * (REP / 2); i += nthreads) {
    const int e = i / (REP / 2), c = 2 * (i % (REP / 2));
    const uint32_t g = KIND == SC_IQ3_XXS ? IQ3XXS_GRID[e] : IQ3S_GRID[e];
    const T v0 = from_f32<T>(float(g & 255)), v1 = from_f32<T>(float((g >> 8) & 255));
    const T v2 = from_f32<T>(float((g >> 16) & 255)), v3 = from_f32<T>(float(g >> 24));
    uint4 w;
    w.x = uint32_t(*reinterpret_cast<const uint16_t*>(&v0)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&v1)) << 16);
    w.y = uint32_t(*reinterpret_cast<const uint16_t*>(&v2)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&v3)) << 16);
    w.z = w.x;
    w.w = w.y;
    *reinterpret_cast<uint4*>(tab + e * REP + c) = w;
  }
}

// Q2_0's biases: pair q's codes at bits 2q of each half (pair 3 shifted down 4 bits first), the exponent making one
// unit of the mantissa there 1; -(B + 1) as a pair of T, exact.
template <typename T> struct Q2;
template <> struct Q2<__nv_bfloat16> {  // B = 128, 32, 8, 32
  __device__ static uint32_t mask(int q) { return q == 0 ? 0x00030003u : q == 2 ? 0x00300030u : 0x000C000Cu; }
  __device__ static uint32_t expo(int q) { return q == 0 ? 0x43004300u : q == 2 ? 0x41004100u : 0x42004200u; }
  __device__ static uint32_t neg(int q) { return q == 0 ? 0xC301C301u : q == 2 ? 0xC110C110u : 0xC204C204u; }
  static constexpr bool shift3 = true;
};
template <> struct Q2<__half> {  // B = 1024, 256, 64, 16: every pair fits the 10-bit mantissa unshifted
  __device__ static uint32_t mask(int q) { return 0x00030003u << (2 * q); }
  __device__ static uint32_t expo(int q) {
    return q == 0 ? 0x64006400u : q == 1 ? 0x5C005C00u : q == 2 ? 0x54005400u : 0x4C004C00u;
  }
  __device__ static uint32_t neg(int q) {
    return q == 0 ? 0xE401E401u : q == 1 ? 0xDC04DC04u : q == 2 ? 0xD410D410u : 0xCC40CC40u;
  }
  static constexpr bool shift3 = false;
};

template <typename T> __device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b);
template <> __device__ __forceinline__ uint32_t add2<__nv_bfloat16>(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hadd2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
template <> __device__ __forceinline__ uint32_t add2<__half>(uint32_t a, uint32_t b) {
  __half2 r = __hadd2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// sign bits j and j + 1 of a lane's sign byte into bits 15 and 31 of its register r (j = 2r)
__device__ __forceinline__ uint32_t signs_of(uint32_t s8, int r) {
  const uint32_t m = r == 0 ? 0x40008000u : r == 1 ? 0x10002000u : r == 2 ? 0x04000800u : 0x01000200u;
  return (s8 * m) & 0x80008000u;
}

// acc (the C fragment: rows g, g + 8; tokens 2t, 2t + 1) += the product of rows ra (row g) and rb (row g + 8) over
// runs [n0, n1) (n0, n1 multiples of 4) with the activations at xg (the lane's token row g of the staged window, in
// the kind's order, in shared or global memory; nullptr when row g is not a token of this tile, which then
// multiplies zeros). With REP > 1, tab is the lane's copy of a codebook in REP copies (rep_tab).
template <int KIND, typename T, int REP = 1>
__device__ __forceinline__ void frag_runs(const uint8_t* ra, const uint8_t* rb, const T* xg, int n0, int n1, int lane,
                                          const uint2* tab, float (&acc)[4]) {
  const int t = lane & 3;
  const int src = lane & ~3;
  for (int n = n0; n < n1; n += 4) {
    uint4 xv[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
      xv[r] = xg ? *reinterpret_cast<const uint4*>(xg + 32 * (n + r) + 8 * t) : make_uint4(0, 0, 0, 0);
    if constexpr (KIND == SC_Q2_0) {
#pragma unroll
      for (int bk = 0; bk < 2; ++bk) {  // a block of 64 weights: runs n + 2bk, n + 2bk + 1, one d
        const int blk = (n >> 1) + bk;
        const uint8_t* ba = ra + blk * 18;
        const uint8_t* bb = rb + blk * 18;
        const float da = half_bits(ld_u16(ba)), db = half_bits(ld_u16(bb));
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 xr = xv[2 * bk + h];
          const uint32_t ua = __byte_perm(ld_u16(ba + 2 + 8 * h + 2 * t), 0, 0x4140);  // [byte0, 0, byte1, 0]
          const uint32_t ub = __byte_perm(ld_u16(bb + 2 + 8 * h + 2 * t), 0, 0x4140);
          uint32_t pa[4], pb[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // B + c, less B + 1 in one exact subtraction: c - 1
            const uint32_t sa = (Q2<T>::shift3 && q == 3) ? ua >> 4 : ua;
            const uint32_t sb = (Q2<T>::shift3 && q == 3) ? ub >> 4 : ub;
            pa[q] = add2<T>((sa & Q2<T>::mask(q)) | Q2<T>::expo(q), Q2<T>::neg(q));
            pb[q] = add2<T>((sb & Q2<T>::mask(q)) | Q2<T>::expo(q), Q2<T>::neg(q));
          }
          const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]}, a1[4] = {pa[2], pb[2], pa[3], pb[3]};
          mma16816<T>(d, a0, xr.x, xr.y);
          mma16816<T>(d, a1, xr.z, xr.w);
        }
        acc[0] = fmaf(da, d[0], acc[0]); acc[1] = fmaf(da, d[1], acc[1]);
        acc[2] = fmaf(db, d[2], acc[2]); acc[3] = fmaf(db, d[3], acc[3]);
      }
    } else {
      // the scales of runs n .. n + 3: lane t works out run n + t's, the others shuffle it over
      float sa_t, sb_t;
      {
        const int m = n + t, ib = m & 7;
        if constexpr (KIND == SC_IQ3_S) {
          const uint8_t* ba = ra + (m >> 3) * 110;
          const uint8_t* bb = rb + (m >> 3) * 110;
          sa_t = half_bits(ld_u16(ba)) * float(1 + 2 * ((uint32_t(ba[106 + (ib >> 1)]) >> (4 * (ib & 1))) & 15));
          sb_t = half_bits(ld_u16(bb)) * float(1 + 2 * ((uint32_t(bb[106 + (ib >> 1)]) >> (4 * (ib & 1))) & 15));
        } else {
          const uint8_t* ba = ra + (m >> 3) * 98;
          const uint8_t* bb = rb + (m >> 3) * 98;
          sa_t = half_bits(ld_u16(ba)) * (0.5f + float(ld_u16(ba + 68 + 4 * ib) >> 12)) * 0.5f;
          sb_t = half_bits(ld_u16(bb)) * (0.5f + float(ld_u16(bb + 68 + 4 * ib) >> 12)) * 0.5f;
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int m = n + r, ib = m & 7;
        uint32_t pa[4], pb[4];
        auto decode = [&](const uint8_t* row, uint32_t (&p)[4]) {
          uint32_t ia, ib2, s8;
          if constexpr (KIND == SC_IQ3_S) {
            const uint8_t* b = row + (m >> 3) * 110;
            const uint32_t qs = ld_u16(b + 2 + 8 * ib + 2 * t);
            const uint32_t qh = uint32_t(b[66 + ib]) >> (2 * t);
            s8 = b[74 + 4 * ib + t];
            ia = (qs & 0xffu) | ((qh & 1u) << 8);
            ib2 = (qs >> 8) | ((qh & 2u) << 7);
          } else {
            const uint8_t* b = row + (m >> 3) * 98;
            const uint32_t qs = ld_u16(b + 2 + 8 * ib + 2 * t);
            const uint32_t aux = ld_u16(b + 66 + 4 * ib) | (ld_u16(b + 68 + 4 * ib) << 16);
            const uint32_t k7 = (aux >> (7 * t)) & 127u;  // ksigns[k7] = k7 with its parity as bit 7
            s8 = k7 | ((__popc(k7) & 1u) << 7);
            ia = qs & 0xffu;
            ib2 = qs >> 8;
          }
          const uint2 ga = tab[ia * REP], gb = tab[ib2 * REP];
          p[0] = ga.x ^ signs_of(s8, 0);
          p[1] = ga.y ^ signs_of(s8, 1);
          p[2] = gb.x ^ signs_of(s8, 2);
          p[3] = gb.y ^ signs_of(s8, 3);
        };
        decode(ra, pa);
        decode(rb, pb);
        const float sa = __shfl_sync(0xffffffffu, sa_t, src | r), sb = __shfl_sync(0xffffffffu, sb_t, src | r);
        const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]}, a1[4] = {pa[2], pb[2], pa[3], pb[3]};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816<T>(d, a0, xv[r].x, xv[r].y);
        mma16816<T>(d, a1, xv[r].z, xv[r].w);
        acc[0] = fmaf(sa, d[0], acc[0]); acc[1] = fmaf(sa, d[1], acc[1]);
        acc[2] = fmaf(sb, d[2], acc[2]); acc[3] = fmaf(sb, d[3], acc[3]);
      }
    }
  }
}

// Two products against the same activations at once (a gate/up item's gate rows and up rows), each run's decodes of
// both interleaved: the same sums, in the same order, as two frag_runs calls.
template <int KIND, typename T, int REP = 1>
__device__ __forceinline__ void frag_runs2(const uint8_t* ga, const uint8_t* gb, const uint8_t* ua, const uint8_t* ub,
                                           const T* xg, int n0, int n1, int lane, const uint2* tab,
                                           float (&accg)[4], float (&accu)[4]) {
  for (int n = n0; n < n1; n += 4) {
    frag_runs<KIND, T, REP>(ga, gb, xg, n, n + 4, lane, tab, accg);
    frag_runs<KIND, T, REP>(ua, ub, xg, n, n + 4, lane, tab, accu);
  }
}

}  // namespace sc
