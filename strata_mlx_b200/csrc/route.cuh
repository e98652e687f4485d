// Device pieces of the MoE block's routing and combine, shared by the stand-alone kernels (route.cu) and the
// fused decode layer (moe.cu).
#pragma once

#include "common.cuh"

namespace sc {

constexpr int ROUTER_MAX_TOKENS = 8;
constexpr int TOPK_MAX_K = 16;
constexpr int TOPK_MAX_N = 2048;

// One router row for a window of tokens (strata_mlx/fused.py:334-354): out[t * stride] = w_row . xs[t], w_row
// float16 (16-byte aligned, cols a multiple of 8), xs float32 in shared memory. Called by a whole warp.
// A token's sum is taken in the same order whatever the window.
template <int MAXT>
__device__ __forceinline__ void router_row(const __half* __restrict__ w_row, int cols, const float* xs, int tokens,
                                           int lane, float* out, int stride) {
  float acc[MAXT];
#pragma unroll
  for (int t = 0; t < MAXT; ++t) acc[t] = 0.f;
  const uint4* w4 = reinterpret_cast<const uint4*>(w_row);
  for (int c = lane; c < cols / 8; c += 32) {
    const uint4 raw = __ldg(w4 + c);
    const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
    float wf[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h2[j]);
      wf[2 * j] = f.x;
      wf[2 * j + 1] = f.y;
    }
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
      if (t < tokens) {
        const float4 a = *reinterpret_cast<const float4*>(xs + t * cols + 8 * c);
        const float4 b = *reinterpret_cast<const float4*>(xs + t * cols + 8 * c + 4);
        float s = acc[t];
        s = fmaf(wf[0], a.x, s); s = fmaf(wf[1], a.y, s); s = fmaf(wf[2], a.z, s); s = fmaf(wf[3], a.w, s);
        s = fmaf(wf[4], b.x, s); s = fmaf(wf[5], b.y, s); s = fmaf(wf[6], b.z, s); s = fmaf(wf[7], b.w, s);
        acc[t] = s;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MAXT; ++t) {
    if (t < tokens) {
      float v = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) out[int64_t(t) * stride] = v;
    }
  }
}

// The k largest of n logits (n <= TOPK_MAX_N, k <= TOPK_MAX_K), largest first, ties to the lower index (the
// rule of strata_mlx/fused.py:400-418); optionally the softmax over them (fused.py:491). Called by a whole
// warp; lane 0 writes idx (and w).
__device__ __forceinline__ void warp_topk(const float* __restrict__ logits, int n, int k, int lane, uint32_t* idx,
                                          float* w) {
  constexpr int PER = TOPK_MAX_N / 32;
  const uint32_t NONE = 0xffffffffu;
  float v[PER];
  uint64_t taken = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) v[i] = (i * 32 + lane < n) ? __ldcg(logits + i * 32 + lane) : -INFINITY;
  float sel[TOPK_MAX_K];
  uint32_t who[TOPK_MAX_K];
  for (int r = 0; r < k; ++r) {
    float best = -INFINITY;
    uint32_t at = NONE;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = i * 32 + lane;
      if (j < uint32_t(n) && !((taken >> i) & 1) && (at == NONE || v[i] > best)) {
        best = v[i];
        at = j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const uint32_t oa = __shfl_xor_sync(0xffffffffu, at, o);
      if (oa != NONE && (at == NONE || ob > best || (ob == best && oa < at))) {
        best = ob;
        at = oa;
      }
    }
    sel[r] = best;
    who[r] = at;
    if (at != NONE && int(at % 32) == lane) {
      const int wi = int(at / 32);
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (i == wi) taken |= uint64_t(1) << i;
    }
  }
  if (lane == 0) {
    for (int r = 0; r < k; ++r) idx[r] = who[r];
    if (w) {
      const float m = sel[0];
      float e[TOPK_MAX_K], sum = 0.f;
      for (int r = 0; r < k; ++r) {
        e[r] = expf(sel[r] - m);
        sum += e[r];
      }
      for (int r = 0; r < k; ++r) w[r] = e[r] / sum;
    }
  }
}

// One output of moe_combine (strata_mlx/fused.py:448-462): the k products y_k * w_k, each rounded to float32
// before it is added (contraction off), summed as MLX's col_reduce sums them (8 partials, partial j taking
// k = j, j + 8, ...; then the partials in order), rounded to T; plus T(T(sigmoid(g)) * s). Returns the value
// before the final rounding to T. y_k is at y[k * YSTRIDE].
template <typename T, int YSTRIDE = 1>
__device__ __forceinline__ float combine_one(const float* y, const float* w, int k, float g, float s) {
  // unrolled to the largest k with the products guarded: the same adds in the same order, without the loops'
  // branches (a one-thread chain, on the decode block's critical path)
  float part[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) part[j] = 0.f;
#pragma unroll
  for (int q = 0; q < TOPK_MAX_K; ++q)
    if (q < k) part[q & 7] = __fadd_rn(__fmul_rn(y[q * YSTRIDE], w[q]), part[q & 7]);
  float acc = part[0];
#pragma unroll
  for (int j = 1; j < 8; ++j)
    if (j < k) acc = __fadd_rn(part[j], acc);
  const float routed = round_to<T>(acc);
  const float gate = round_to<T>(1.0f / (1.0f + expf(-g)));
  const float shared = round_to<T>(__fmul_rn(gate, s));
  return __fadd_rn(routed, shared);
}

}  // namespace sc
