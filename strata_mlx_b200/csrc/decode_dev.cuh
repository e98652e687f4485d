// Device pieces shared by the decode block's kernels: the three-kernel block (decode_layer.cu) and the persistent
// chain kernel (decode_chain.cu). Both must route and combine alike, bit for bit: the expert-parallel path runs the
// three kernels and is checked against the single-device block.
#pragma once

#include "decode_layer.cuh"
#include "route.cuh"

namespace sc {
namespace dl {

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// eight float16 router weights times eight activations of T, float32 products summed in order
template <typename T>
__device__ __forceinline__ float dot8_half(const uint4& w, const uint4& x) {
  const __half2* wh = reinterpret_cast<const __half2*>(&w);
  const T* xv = reinterpret_cast<const T*>(&x);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(wh[j]);
    s = fmaf(f.x, to_f32(xv[2 * j]), s);
    s = fmaf(f.y, to_f32(xv[2 * j + 1]), s);
  }
  return s;
}

// A float as an unsigned key in the same order (larger float, larger key)
__device__ __forceinline__ uint32_t fkey(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unkey(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }

// One round of a warp's selection: the largest key among the lanes' candidates, ties to the lower index; two
// warp reductions (redux.sync). Returns the winner's index (0xffffffff when no lane has a candidate).
__device__ __forceinline__ uint32_t warp_best(uint32_t key, uint32_t idx, uint32_t& best_key) {
  best_key = __reduce_max_sync(0xffffffffu, key);
  return __reduce_min_sync(0xffffffffu, key == best_key ? idx : 0xffffffffu);
}

__device__ __forceinline__ int atomic_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

constexpr int TAIL_WARPS = 16;  // the route tail runs on sixteen warps
constexpr int TAIL_CAP = 128;   // candidates a token's list holds before the slow path

// Shared memory of the route tail (the caller's: static in the route kernel, a carved region in the chain kernel).
struct TailSmem {
  uint32_t w_max[MAXT][TAIL_WARPS], s_theta[MAXT], s_cnt[MAXT];
  __align__(16) uint32_t m_k[MAXT][TAIL_CAP];
  __align__(16) uint32_t m_i[MAXT][TAIL_CAP];
  uint32_t s_key[MAXT * TOPK_MAX_K], s_idx[MAXT * TOPK_MAX_K];
  float s_w[MAXT * TOPK_MAX_K];
  uint32_t s_bits[32], s_pre[32], s_mask[MAXU], s_kpack[MAXU];
  int s_expert[MAXU];
};

// The route tail of a window: top-k of each token over logits (T, E) float32 in global memory (written by other
// blocks, read through L2), the softmax over the chosen logits (strata_mlx/fused.py:400-436, :491), and the plan
// of this rank's experts [e0, e1) as units (unit 0 the shared expert, then the distinct experts in ascending order,
// each with its tokens and their ranks). Run by TAIL_WARPS warps (tid < 512); `sync` synchronizes exactly those.
// Results in S: s_idx, s_w (T, K), s_expert / s_mask / s_kpack of units 1.., and the unit count is returned.
//
// Every step is a few dependent operations across all lanes: a long chain of dependent shuffles or selection rounds
// in one warp costs microseconds.
//   A. warp w takes the logits [seg w, seg w + seg) (seg 32 or 64, one or two a lane) and their maximum;
//   B. theta = the K-th largest of the warps' maxima (0 when fewer than K warps hold logits): K warps each hold a
//      logit >= theta, so every logit of the top K is >= theta;
//   C. the logits >= theta (usually a few more than K) are gathered into a short list;
//   D. warp t ranks token t's list by broadcast reads of it, keeps the K best in order (ties to the lower index, as
//      the reference's argpartition + sort) and takes their softmax. A list longer than TAIL_CAP (many ties) falls
//      back to K rounds of selection over all the logits.
template <int MT, typename Sync>
__device__ __forceinline__ int route_tail(const float* logits, int T_, int E, int K, int e0, int e1, TailSmem& S,
                                          int tid, Sync sync) {
  constexpr uint32_t NONE = 0xffffffffu;
  const int warp = tid >> 5, lane = tid & 31;
  const int seg = E > TAIL_WARPS * 32 ? 64 : 32;
  const int live = int(ceil_div(E, seg));  // warps with logits
  const int base = seg * warp;
  const bool ok0 = warp < live && base + lane < E, ok1 = warp < live && seg == 64 && base + 32 + lane < E;
  uint32_t k0[MT], k1[MT];  // keys of invalid slots are 0, below every non-NaN logit's key
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    k0[t] = ok0 && t < T_ ? fkey(__ldcg(logits + int64_t(t) * E + base + lane)) : 0u;
    k1[t] = ok1 && t < T_ ? fkey(__ldcg(logits + int64_t(t) * E + base + 32 + lane)) : 0u;
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const uint32_t mx = __reduce_max_sync(0xffffffffu, max(k0[t], k1[t]));
    if (lane == 0 && t < T_) S.w_max[t][warp] = mx;
  }
  if (tid < MAXT) S.s_cnt[tid] = 0;
  for (int i = tid; i < 32; i += TAIL_WARPS * 32) S.s_bits[i] = 0;
  for (int u = tid; u < MAXU; u += TAIL_WARPS * 32) {
    S.s_mask[u] = 0;
    S.s_kpack[u] = 0;
  }
  sync();
  if (warp < T_) {  // B, warp t for token t: lane l < live ranks warp l's maximum among the live warps' maxima
    const int t = warp;
    const uint32_t v = lane < live ? S.w_max[t][lane] : 0u;
    int r = 0;
#pragma unroll
    for (int j = 0; j < TAIL_WARPS; ++j) {
      const uint32_t a = j < live ? S.w_max[t][j] : 0u;
      r += int(a > v) | (int(a == v) & int(j < lane));
    }
    const uint32_t th = __reduce_max_sync(0xffffffffu, lane < live && r == K - 1 ? v : 0u);
    if (lane == 0) S.s_theta[t] = th;
  }
  sync();
#pragma unroll
  for (int t = 0; t < MT; ++t) {  // C
    if (t >= T_) break;
    const uint32_t th = S.s_theta[t];
    const bool in0 = ok0 && k0[t] >= th, in1 = ok1 && k1[t] >= th;
    const uint32_t b0 = __ballot_sync(0xffffffffu, in0), b1 = __ballot_sync(0xffffffffu, in1);
    if (b0 | b1) {
      int at = 0;
      if (lane == 0) at = atomicAdd(&S.s_cnt[t], __popc(b0) + __popc(b1));
      at = __shfl_sync(0xffffffffu, at, 0);
      const int p0 = at + __popc(b0 & ((1u << lane) - 1u)), p1 = at + __popc(b0) + __popc(b1 & ((1u << lane) - 1u));
      if (in0 && p0 < TAIL_CAP) {
        S.m_k[t][p0] = k0[t];
        S.m_i[t][p0] = uint32_t(base + lane);
      }
      if (in1 && p1 < TAIL_CAP) {
        S.m_k[t][p1] = k1[t];
        S.m_i[t][p1] = uint32_t(base + 32 + lane);
      }
    }
  }
  sync();
  for (int t = warp; t < T_; t += TAIL_WARPS) {  // D
    const int m = int(S.s_cnt[t]);
    if (m <= TAIL_CAP) {
      // lane l ranks entries l, l + 32, ... of the list; four partial counts keep the chains short
      const int nq = (m + 31) / 32;
#pragma unroll
      for (int q = 0; q < TAIL_CAP / 32; ++q) {
        if (q >= nq) break;
        const bool in = lane + 32 * q < m;
        const uint32_t kc = in ? S.m_k[t][lane + 32 * q] : 0u, ic = in ? S.m_i[t][lane + 32 * q] : NONE;
        int r4[4] = {0, 0, 0, 0};
        for (int j = 0; j < m; j += 4) {  // entries past m hold stale values: masked by j + e < m
          const uint4 a = *reinterpret_cast<const uint4*>(&S.m_k[t][j]);
          const uint4 ai = *reinterpret_cast<const uint4*>(&S.m_i[t][j]);
          const uint32_t av[4] = {a.x, a.y, a.z, a.w}, aiv[4] = {ai.x, ai.y, ai.z, ai.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)  // bitwise, not && / ||: no branches in the chain
            r4[e] += int(j + e < m) & (int(av[e] > kc) | (int(av[e] == kc) & int(aiv[e] < ic)));
        }
        const int r = r4[0] + r4[1] + r4[2] + r4[3];
        if (in && r < K) {
          S.s_key[t * K + r] = kc;
          S.s_idx[t * K + r] = ic;
        }
      }
    } else {
      // K rounds over all the logits, each taking the best that comes after the previous pick in the order
      uint32_t pk = 0, pi = NONE;
      for (int rr = 0; rr < K; ++rr) {
        uint32_t bk = 0, bi = NONE;
        for (int j = lane; j < E; j += 32) {
          const uint32_t kj = fkey(__ldcg(logits + int64_t(t) * E + j));
          const bool after = pi == NONE || kj < pk || (kj == pk && uint32_t(j) > pi);
          if (after && (bi == NONE || kj > bk)) {  // j ascends: an equal key keeps the lower index
            bk = kj;
            bi = uint32_t(j);
          }
        }
        const uint32_t who = warp_best(bi == NONE ? 0u : bk, bi, pk);
        pi = who;
        if (lane == 0) {
          S.s_key[t * K + rr] = pk;
          S.s_idx[t * K + rr] = who;
        }
      }
    }
    __syncwarp();
    // softmax over the chosen logits (fused.py:491), lane k taking choice k
    const float top = unkey(S.s_key[t * K]);
    const float e = lane < K ? expf(unkey(S.s_key[t * K + lane]) - top) : 0.f;
    float sum = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane < K) S.s_w[t * K + lane] = e / sum;
  }
  sync();
  const int P = T_ * K;
  for (int p = tid; p < P; p += TAIL_WARPS * 32) {  // this rank's distinct experts as bits of a bitmap (E <= 1024)
    const int le = int(S.s_idx[p]) - e0;  // the local expert
    if (le >= 0 && int(S.s_idx[p]) < e1) atomicOr(&S.s_bits[le >> 5], 1u << (le & 31));
  }
  sync();
  if (warp == 0) {  // exclusive prefix of the bitmap's popcounts
    const int c = __popc(S.s_bits[lane]);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    S.s_pre[lane] = uint32_t(incl - c);
  }
  sync();
  for (int p = tid; p < P; p += TAIL_WARPS * 32) {
    const int le = int(S.s_idx[p]) - e0;
    if (le < 0 || int(S.s_idx[p]) >= e1) continue;  // another rank's expert
    const uint32_t e = uint32_t(le);
    // unit 0 is the shared expert; the routed units follow in ascending expert order
    const int u = 1 + int(S.s_pre[e >> 5]) + __popc(S.s_bits[e >> 5] & ((1u << (e & 31)) - 1u));
    const int tok = p / K, k = p % K;
    S.s_expert[u] = int(e);
    atomicOr(&S.s_mask[u], 1u << tok);
    atomicOr(&S.s_kpack[u], uint32_t(k) << (4 * tok));
  }
  sync();
  return 1 + int(S.s_pre[31]) + __popc(S.s_bits[31]);
}

}  // namespace dl
}  // namespace sc
