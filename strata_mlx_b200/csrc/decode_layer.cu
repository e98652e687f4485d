// The decode MoE block in three kernels (strata_mlx/fused.py:487-497 for a window of 1..8 tokens), chained with
// programmatic dependent launch so that each kernel's independent prologue overlaps the kernel before it:
//
//   route   router product (float16 weights, fused.py:334-354) and the shared expert's gate, then -- in the
//           last block to finish, found with an atomic ticket -- top-k with the softmax over the chosen logits
//           (fused.py:400-436, :491) and the plan: the distinct experts of the window (units), each with the
//           tokens that chose it. Router weights are loaded into registers before waiting on the previous kernel.
//   gate_up every unit's gate and up rows [r0, r0 + 4) (unit 0 is the shared expert, its rows fetched before the
//           wait), streamed by 1-D bulk copies into a ring of shared-memory stages, decoded into tensor-core
//           fragments (mma_decode.cuh), multiplied by the window's activations on mma.sync (bf16/f16, f32 sums),
//           split over eight warps along the columns and reduced through shared memory; swiglu as mlx-lm rounds
//           it (blocks.py:230-238) -> h.
//   down    every unit's down rows [r0, r0 + 16) times its h, the same way; then moe_combine's epilogue
//           (fused.py:448-462) for those 16 outputs of every token, in MLX's order, with the shared expert's
//           sigmoid gate.
//
// Block types with fragment decoders: Q2_0, IQ3_S, IQ3_XXS (HasMma); other layers take moe.cu's chain.
#include <algorithm>

#include "matvec.cuh"
#include "mma_decode.cuh"
#include "route.cuh"
#include "decode_layer.cuh"

namespace sc {
namespace dl {

constexpr int WARPS = 8;
constexpr int THREADS = (WARPS + 1) * 32;
constexpr int MAX_STAGES = 8;

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

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

// ---------------------------------------------------------------------------------------------------- route

template <typename T>
__global__ void __launch_bounds__(128) route_kernel(LayerDev L) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int row = blockIdx.x * 4 + warp;  // router rows 0 .. E-1; row E is the shared expert's gate
  const int H = L.H, E = L.E, K = L.K, T_ = L.T;
  const __half* wrow = row < E ? L.router + int64_t(row) * H : (row == E && L.Is > 0 ? L.shared_gate : nullptr);
  const int chunks = H / 256;  // 16-byte chunks a lane reads
  uint4 w[MAX_ROUTER_CHUNKS];
  if (wrow) {
#pragma unroll
    for (int c = 0; c < MAX_ROUTER_CHUNKS; ++c)
      if (c < chunks) w[c] = __ldg(reinterpret_cast<const uint4*>(wrow) + lane + 32 * c);
  }
  pdl_launch_dependents();
  pdl_wait();  // the window's activations are the previous kernel's output
  if (wrow) {
    for (int t = 0; t < T_; ++t) {
      const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const T*>(L.x) + int64_t(t) * H);
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < MAX_ROUTER_CHUNKS; ++c)
        if (c < chunks) acc += dot8_half<T>(w[c], xr[lane + 32 * c]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        if (row < E) L.logits[int64_t(t) * E + row] = acc;
        else L.gsh[t] = acc;
      }
    }
  }
  __shared__ int s_last;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(L.ticket, 1) == int(gridDim.x) - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---- the last block: top-k + softmax per token, then the plan
  __shared__ uint32_t s_idx[MAXT * TOPK_MAX_K];
  __shared__ float s_w[MAXT * TOPK_MAX_K];
  __shared__ int s_first[MAXT * TOPK_MAX_K], s_unit[MAXT * TOPK_MAX_K];
  __shared__ uint32_t s_mask[MAXU], s_kpack[MAXU];
  __shared__ int s_expert[MAXU];
  for (int t = warp; t < T_; t += 4) warp_topk(L.logits + int64_t(t) * E, E, K, lane, s_idx + t * K, s_w + t * K);
  const int P = T_ * K;
  for (int u = tid; u < MAXU; u += blockDim.x) {
    s_mask[u] = 0;
    s_kpack[u] = 0;
  }
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    L.idx[p] = s_idx[p];
    L.wts[p] = s_w[p];
    int first = 1;
    for (int q = 0; q < p; ++q) first &= s_idx[q] != s_idx[p];
    s_first[p] = first;
  }
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    if (s_first[p]) {
      int u = 1;  // unit 0 is the shared expert; the routed units follow in ascending expert order
      for (int q = 0; q < P; ++q) u += s_first[q] && s_idx[q] < s_idx[p];
      s_unit[p] = u;
      s_expert[u] = int(s_idx[p]);
    }
  }
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    int q0 = 0;
    while (s_idx[q0] != s_idx[p]) ++q0;  // the pair that named this expert first
    const int u = s_unit[q0], tok = p / K, k = p % K;
    atomicOr(&s_mask[u], 1u << tok);
    atomicOr(&s_kpack[u], uint32_t(k) << (4 * tok));
  }
  __syncthreads();
  int units = 1;
  for (int p = 0; p < P; ++p) units += s_first[p];
  for (int u = tid; u < units; u += blockDim.x) {
    Unit v;
    v.expert = u == 0 ? -1 : s_expert[u];
    v.tokmask = u == 0 ? (L.Is > 0 ? (1u << T_) - 1u : 0u) : s_mask[u];
    v.kpack = u == 0 ? 0u : s_kpack[u];
    v.pad = 0;
    L.plan->unit[u] = v;
  }
  if (tid == 0) {
    L.plan->units = units;
    *L.ticket = 0;  // ready for the next call on this workspace
  }
}

// ---------------------------------------------------------------------------------------------------- gate_up

struct GuSmem {
  int bars, tabs, plan, xs, red, stages, total;
};

__host__ __device__ inline GuSmem gu_smem(int tokens, int H, int stage_bytes, int stages) {
  GuSmem s;
  int o = 0;
  s.bars = o; o += align16(2 * MAX_STAGES * 8);
  s.tabs = o; o += align16(2048 + 8);
  s.plan = o; o += align16(int(sizeof(Plan)));
  s.xs = o; o += align16(tokens * (H + 32) * 2);
  s.red = o; o += 2 * WARPS * 32 * 8 * 4;
  s.stages = align16(o); o = s.stages + stages * stage_bytes;
  s.total = o;
  return s;
}

template <int KIND, typename T>
__global__ void __launch_bounds__(THREADS) gate_up_kernel(LayerDev L) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T_ = L.T, H = L.H;
  const GuSmem S = gu_smem(T_, H, L.gu_stage, L.gu_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S.bars);
  uint64_t* empty = full + MAX_STAGES;
  Plan* plan = reinterpret_cast<Plan*>(smem + S.plan);
  T* xs = reinterpret_cast<T*>(smem + S.xs);
  float* red = reinterpret_cast<float*>(smem + S.red);
  uint8_t* stage0 = smem + S.stages;
  const int r0 = blockIdx.x * RB;
  const int stride = L.gu_stride, xstride = H + 32;
  const int slot_bytes = 2 * RB * stride;  // a unit's gate rows then up rows

  if (tid == 0) {
    for (int s = 0; s < L.gu_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], WARPS);
    }
    fence_mbar_init();
  }
  const uint32_t* grid = nullptr;
  if constexpr (KIND == SC_IQ3_S) grid = load_tabs<KIND>(smem + S.tabs).iq3s;
  if constexpr (KIND == SC_IQ3_XXS) grid = load_tabs<KIND>(smem + S.tabs).iq3xxs;
  __syncthreads();

  // copies of unit u's rows [r0, r0 + rows) of gate and up into slot j of stage s (one bulk copy per row when the
  // shared-memory rows are padded, else one per matrix)
  auto issue_unit = [&](int s, int j, const uint8_t* g, const uint8_t* u, int rows, int64_t rb) {
    uint8_t* dst = stage0 + s * L.gu_stage + j * slot_bytes;
    if (stride == rb) {
      bulk_load(dst, g + r0 * rb, uint32_t(rows * rb), &full[s]);
      bulk_load(dst + RB * stride, u + r0 * rb, uint32_t(rows * rb), &full[s]);
    } else {
      for (int r = 0; r < rows; ++r) {
        bulk_load(dst + r * stride, g + (r0 + r) * rb, uint32_t(rb), &full[s]);
        bulk_load(dst + (RB + r) * stride, u + (r0 + r) * rb, uint32_t(rb), &full[s]);
      }
    }
  };
  const int shared_rows = L.Is > r0 ? min(RB, L.Is - r0) : 0;
  if (warp == WARPS && lane == 0 && shared_rows > 0) {  // the shared expert does not wait for the routes
    mbar_expect_tx(&full[0], uint32_t(2 * shared_rows * L.rb_sgu));
    issue_unit(0, 0, L.sgate, L.sup, shared_rows, L.rb_sgu);
  }
  pdl_launch_dependents();
  pdl_wait();  // the routes (and the window's activations)

  for (int i = tid; i < int(sizeof(Plan) / 16); i += blockDim.x)
    reinterpret_cast<int4*>(plan)[i] = __ldcg(reinterpret_cast<const int4*>(L.plan) + i);
  stage_x_permuted<T>(static_cast<const T*>(L.x), T_, H, xs, xstride, tid, blockDim.x);
  __syncthreads();
  const int units = plan->units;
  const int tiles = (units + 3) / 4;
  const int routed_rows = L.I > r0 ? min(RB, L.I - r0) : 0;

  if (warp == WARPS) {  // ---- producer
    if (lane == 0) {
      for (int i = 0; i < tiles; ++i) {
        const int s = i % L.gu_stages;
        if (i >= L.gu_stages && !mbar_wait(&empty[s], ((i / L.gu_stages) - 1) & 1, L.err)) break;
        uint32_t bytes = 0;
        for (int j = 0; j < 4; ++j) {
          const int u = 4 * i + j;
          if (u == 0 || u >= units || routed_rows == 0) continue;
          bytes += uint32_t(2 * routed_rows * L.rb_gu);
        }
        mbar_arrive_expect_tx(&full[s], bytes);
        for (int j = 0; j < 4; ++j) {
          const int u = 4 * i + j;
          if (u == 0 || u >= units || routed_rows == 0) continue;
          const int64_t e = plan->unit[u].expert;
          issue_unit(s, j, L.gate + e * L.I * L.rb_gu, L.up + e * L.I * L.rb_gu, routed_rows, L.rb_gu);
        }
      }
    }
    return;
  }

  // ---- consumers: warp w takes runs [w * runs / 8, (w + 1) * runs / 8) of every row of the tile
  const int g = lane >> 2, t = lane & 3;
  const int runs = H / 32, n0 = warp * runs / WARPS, n1 = (warp + 1) * runs / WARPS;
  for (int i = 0; i < tiles; ++i) {
    const int s = i % L.gu_stages;
    if (!mbar_wait(&full[s], (i / L.gu_stages) & 1, L.err)) break;
    const uint8_t* st = stage0 + s * L.gu_stage;
    // lane rows: tile row g (slot g / 4, row g % 4) and tile row g + 8 (slot 2 + g / 4)
    const uint8_t* ga = st + (g >> 2) * slot_bytes + (g & 3) * stride;
    const uint8_t* gb = st + (2 + (g >> 2)) * slot_bytes + (g & 3) * stride;
    const uint8_t* ua = ga + RB * stride;
    const uint8_t* ub = gb + RB * stride;
    float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
    for (int n = n0; n < n1; ++n) {
      uint4 xv = make_uint4(0, 0, 0, 0);
      if (g < T_) xv = *reinterpret_cast<const uint4*>(xs + g * xstride + 32 * n + 8 * t);
      uint32_t pa[4], pb[4];
      {
        const float sa = dec8<KIND, T>(ga, n, t, grid, pa), sb = dec8<KIND, T>(gb, n, t, grid, pb);
        const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]}, a1[4] = {pa[2], pb[2], pa[3], pb[3]};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816<T>(d, a0, xv.x, xv.y);
        mma16816<T>(d, a1, xv.z, xv.w);
        accg[0] = fmaf(sa, d[0], accg[0]); accg[1] = fmaf(sa, d[1], accg[1]);
        accg[2] = fmaf(sb, d[2], accg[2]); accg[3] = fmaf(sb, d[3], accg[3]);
      }
      {
        const float sa = dec8<KIND, T>(ua, n, t, grid, pa), sb = dec8<KIND, T>(ub, n, t, grid, pb);
        const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]}, a1[4] = {pa[2], pb[2], pa[3], pb[3]};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816<T>(d, a0, xv.x, xv.y);
        mma16816<T>(d, a1, xv.z, xv.w);
        accu[0] = fmaf(sa, d[0], accu[0]); accu[1] = fmaf(sa, d[1], accu[1]);
        accu[2] = fmaf(sb, d[2], accu[2]); accu[3] = fmaf(sb, d[3], accu[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    float* rb = red + (i & 1) * (WARPS * 32 * 8) + (warp * 32 + lane) * 8;
    *reinterpret_cast<float4*>(rb) = make_float4(accg[0], accg[1], accg[2], accg[3]);
    *reinterpret_cast<float4*>(rb + 4) = make_float4(accu[0], accu[1], accu[2], accu[3]);
    named_sync(1, WARPS * 32);
    if (tid < 128) {  // thread (value q, lane L): the sum over warps of one (row, token) of gate and up
      const int Lq = tid & 31, q = tid >> 5;
      const float* base = red + (i & 1) * (WARPS * 32 * 8) + Lq * 8;
      float sg = 0.f, su = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        sg += base[w * 32 * 8 + q];
        su += base[w * 32 * 8 + 4 + q];
      }
      const int m = (q < 2 ? 0 : 8) + (Lq >> 2);   // tile row
      const int tok = 2 * (Lq & 3) + (q & 1);      // token
      const int u = 4 * i + (m >> 2), r = r0 + (m & 3);
      if (u < units && tok < T_ && ((plan->unit[u].tokmask >> tok) & 1u) && r < (u == 0 ? L.Is : L.I)) {
        // h is stored in the fragment order of its consumer (groups of eight as 0,4,1,5,2,6,3,7)
        const int j = r & 7, col = (r & ~7) + (j < 4 ? 2 * j : 2 * (j - 4) + 1);
        static_cast<T*>(L.h)[(int64_t(u) * T_ + tok) * L.hstride + col] = from_f32<T>(swiglu_mlx<T>(sg, su));
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------- down

struct DnSmem {
  int bars, tabs, plan, wts, ys, red, stages, total;
};

__host__ __device__ inline DnSmem dn_smem(int tokens, int K, int stage_bytes, int stages) {
  DnSmem s;
  int o = 0;
  s.bars = o; o += align16(2 * MAX_STAGES * 8);
  s.tabs = o; o += align16(2048 + 8);
  s.plan = o; o += align16(int(sizeof(Plan)));
  s.wts = o; o += align16(tokens * (K + 1) * 4);
  s.ys = o; o += align16(tokens * (K + 1) * RC * 4);
  s.red = o; o += 2 * WARPS * 32 * 4 * 4;
  s.stages = align16(o); o = s.stages + stages * stage_bytes;
  s.total = o;
  return s;
}

template <int KIND, typename T>
__global__ void __launch_bounds__(THREADS) down_kernel(LayerDev L) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T_ = L.T, K = L.K, H = L.H;
  const DnSmem S = dn_smem(T_, K, L.dn_stage, L.dn_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S.bars);
  uint64_t* empty = full + MAX_STAGES;
  Plan* plan = reinterpret_cast<Plan*>(smem + S.plan);
  float* wts = reinterpret_cast<float*>(smem + S.wts);  // (T, K) routes' weights, then (T) the shared gates
  float* ys = reinterpret_cast<float*>(smem + S.ys);    // (T, K + 1, 16): routed outputs, then the shared one
  float* red = reinterpret_cast<float*>(smem + S.red);
  uint8_t* stage0 = smem + S.stages;
  const int r0 = blockIdx.x * RC;
  const int hbytes = T_ * L.hstride * 2;  // a unit's h: its tokens' rows
  const int wbytes_max = RC * max(L.rb_d, L.rb_sd);

  if (tid == 0) {
    for (int s = 0; s < L.dn_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], WARPS);
    }
    fence_mbar_init();
  }
  const uint32_t* grid = nullptr;
  if constexpr (KIND == SC_IQ3_S) grid = load_tabs<KIND>(smem + S.tabs).iq3s;
  if constexpr (KIND == SC_IQ3_XXS) grid = load_tabs<KIND>(smem + S.tabs).iq3xxs;
  __syncthreads();
  if (warp == WARPS && lane == 0 && L.Is > 0) {  // the shared expert's 16 down rows do not wait for anything
    mbar_expect_tx(&full[0], uint32_t(RC * L.rb_sd));
    bulk_load(stage0, L.sdown + r0 * L.rb_sd, uint32_t(RC * L.rb_sd), &full[0]);
  }
  pdl_launch_dependents();
  pdl_wait();  // h and the routes

  for (int i = tid; i < int(sizeof(Plan) / 16); i += blockDim.x)
    reinterpret_cast<int4*>(plan)[i] = __ldcg(reinterpret_cast<const int4*>(L.plan) + i);
  for (int i = tid; i < T_ * K; i += blockDim.x) wts[i] = __ldcg(L.wts + i);
  for (int i = tid; i < T_; i += blockDim.x) wts[T_ * K + i] = L.Is > 0 ? __ldcg(L.gsh + i) : -INFINITY;
  __syncthreads();
  const int units = plan->units;

  if (warp == WARPS) {  // ---- producer: unit u = tile u
    if (lane == 0) {
      for (int u = 0; u < units; ++u) {
        const int s = u % L.dn_stages;
        if (u >= L.dn_stages && !mbar_wait(&empty[s], ((u / L.dn_stages) - 1) & 1, L.err)) break;
        uint8_t* dst = stage0 + s * L.dn_stage;
        const bool shared = u == 0;
        if (shared && L.Is == 0) {
          mbar_arrive(&full[s]);
          continue;
        }
        const uint32_t wbytes = shared ? 0u : uint32_t(RC * L.rb_d);
        mbar_arrive_expect_tx(&full[s], wbytes + uint32_t(hbytes));
        if (!shared) bulk_load(dst, L.down + (int64_t(plan->unit[u].expert) * H + r0) * L.rb_d, wbytes, &full[s]);
        bulk_load(dst + align16(wbytes_max), static_cast<const T*>(L.h) + int64_t(u) * T_ * L.hstride, uint32_t(hbytes),
                  &full[s]);
      }
    }
    return;
  }

  // ---- consumers
  const int g = lane >> 2, t = lane & 3;
  for (int u = 0; u < units; ++u) {
    const int s = u % L.dn_stages;
    if (!mbar_wait(&full[s], (u / L.dn_stages) & 1, L.err)) break;
    const bool shared = u == 0;
    const uint8_t* st = stage0 + s * L.dn_stage;
    const T* hs = reinterpret_cast<const T*>(st + align16(wbytes_max));
    const int cols = shared ? L.Is : L.I;
    const int64_t rb = shared ? L.rb_sd : L.rb_d;
    const int runs = cols / 32, n0 = warp * runs / WARPS, n1 = (warp + 1) * runs / WARPS;
    const uint32_t mask = plan->unit[u].tokmask;
    const bool mine = g < T_ && ((mask >> g) & 1u);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (!(shared && L.Is == 0)) {
      const uint8_t* ra = st + g * rb;
      const uint8_t* rbp = st + (g + 8) * rb;
      for (int n = n0; n < n1; ++n) {
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (mine) xv = *reinterpret_cast<const uint4*>(hs + g * L.hstride + 32 * n + 8 * t);
        uint32_t pa[4], pb[4];
        const float sa = dec8<KIND, T>(ra, n, t, grid, pa), sb = dec8<KIND, T>(rbp, n, t, grid, pb);
        const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]}, a1[4] = {pa[2], pb[2], pa[3], pb[3]};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816<T>(d, a0, xv.x, xv.y);
        mma16816<T>(d, a1, xv.z, xv.w);
        acc[0] = fmaf(sa, d[0], acc[0]); acc[1] = fmaf(sa, d[1], acc[1]);
        acc[2] = fmaf(sb, d[2], acc[2]); acc[3] = fmaf(sb, d[3], acc[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    float* rbuf = red + (u & 1) * (WARPS * 32 * 4) + (warp * 32 + lane) * 4;
    *reinterpret_cast<float4*>(rbuf) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    named_sync(1, WARPS * 32);
    if (tid < 128) {
      const int Lq = tid & 31, q = tid >> 5;
      const float* base = red + (u & 1) * (WARPS * 32 * 4) + Lq * 4 + q;
      float y = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) y += base[w * 32 * 4];
      const int m = (q < 2 ? 0 : 8) + (Lq >> 2), tok = 2 * (Lq & 3) + (q & 1);
      if (tok < T_ && ((mask >> tok) & 1u)) {
        const int k = shared ? K : int((plan->unit[u].kpack >> (4 * tok)) & 15u);
        ys[(tok * (K + 1) + k) * RC + m] = round_to<T>(y);
      }
    }
  }
  named_sync(1, WARPS * 32);
  // ---- moe_combine for rows [r0, r0 + 16) of every token
  for (int i = tid; i < T_ * RC; i += WARPS * 32) {
    const int tok = i / RC, m = i % RC;
    float yk[TOPK_MAX_K];
    for (int k = 0; k < K; ++k) yk[k] = ys[(tok * (K + 1) + k) * RC + m];
    const float sv = L.Is > 0 ? ys[(tok * (K + 1) + K) * RC + m] : 0.f;
    const float gv = L.Is > 0 ? round_to<T>(wts[T_ * K + tok]) : -INFINITY;
    static_cast<T*>(L.out)[int64_t(tok) * H + r0 + m] = from_f32<T>(combine_one<T>(yk, wts + tok * K, K, gv, sv));
  }
}

// ---------------------------------------------------------------------------------------------------- host

template <typename Kern>
static cudaError_t launch_pdl(Kern kern, int grid, int threads, int smem, cudaStream_t s, const LayerDev& L) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, L);
}

static int gu_stride(int64_t rb) {
  int s = align16(int(rb));
  if ((s / 4) % 8 != 4) s += 16;  // rows of the eight lane groups fall on eight different bank groups
  return s;
}

template <int KGU, int KD, typename T>
static int run(LayerDev L, cudaStream_t s) {
  // gate/up: a stage is a tile of four units. Enough stages to have every tile of the window in flight (within
  // ~100 KB), so that the gate/up and down kernels fit one SM together and each one's prologue overlaps the other.
  const int max_units = L.T * L.K + 1;
  L.gu_stride = gu_stride(L.rb_gu);
  L.gu_stage = align16(4 * 2 * RB * L.gu_stride);
  const int gu_fixed = gu_smem(L.T, L.H, 0, 0).total;
  L.gu_stages = std::max(2, std::min({MAX_STAGES, int(ceil_div(max_units, 4)), (100 * 1024) / L.gu_stage}));
  const int gu_total = gu_smem(L.T, L.H, L.gu_stage, L.gu_stages).total;
  // down: a stage is one unit's 16 rows and its h
  L.dn_stage = align16(RC * int(std::max(L.rb_d, L.rb_sd))) + align16(L.T * L.hstride * 2);
  L.dn_stages = std::max(2, std::min({MAX_STAGES, max_units, (64 * 1024) / L.dn_stage}));
  const int dn_total = dn_smem(L.T, L.K, L.dn_stage, L.dn_stages).total;
  (void)gu_fixed;
  if (gu_total > 227 * 1024 || dn_total > 227 * 1024) return SC_ERR_SHAPE;

  auto kr = route_kernel<T>;
  auto kg = gate_up_kernel<KGU, T>;
  auto kd = down_kernel<KD, T>;
  static bool attrs_set = false;  // per-process: the attribute is a property of the function
  if (!attrs_set) {
    cudaFuncSetAttribute(kg, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(kd, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attrs_set = true;
  }
  const int grid_r = int(ceil_div(L.E + 1, 4));
  const int grid_g = int(ceil_div(std::max(L.I, L.Is), RB));
  const int grid_d = L.H / RC;
  if (launch_pdl(kr, grid_r, 128, 0, s, L) != cudaSuccess) return SC_ERR_CUDA;
  if (launch_pdl(kg, grid_g, THREADS, gu_total, s, L) != cudaSuccess) return SC_ERR_CUDA;
  if (launch_pdl(kd, grid_d, THREADS, dn_total, s, L) != cudaSuccess) return SC_ERR_CUDA;
  return SC_OK;
}

}  // namespace dl

// Whether the three-kernel path takes the layer, and the scratch it needs beyond the common header.
bool v2_takes(const sc_moe_layer* L, int tokens) {
  auto mma_kind = [](int k) { return k == SC_Q2_0 || k == SC_IQ3_S || k == SC_IQ3_XXS; };
  if (L->dtype != SC_BF16 && L->dtype != SC_F16) return false;
  if (tokens < 1 || tokens > dl::MAXT || L->top_k > TOPK_MAX_K || tokens * L->top_k > dl::MAXU - 1) return false;
  if (L->experts > TOPK_MAX_N) return false;
  if (!mma_kind(L->kind_gate) || L->kind_up != L->kind_gate || !mma_kind(L->kind_down)) return false;
  if (L->shared_inter > 0 && (L->kind_sgate != L->kind_gate || L->kind_sup != L->kind_gate || L->kind_sdown != L->kind_down))
    return false;
  if (L->hidden % 256 || L->hidden / 256 > dl::MAX_ROUTER_CHUNKS || L->hidden % dl::RC) return false;
  if (L->inter % 32 || L->inter % dl::RB || L->shared_inter % 32 || L->shared_inter % dl::RB) return false;
  if (row_bytes(L->kind_gate, L->hidden) % 16) return false;
  return true;
}

int v2_run(const sc_moe_layer* L, const void* x, int tokens, void* out, uint8_t* ws, const V2Offsets& o,
           cudaStream_t s) {
  dl::LayerDev d{};
  d.gate = static_cast<const uint8_t*>(L->gate);
  d.up = static_cast<const uint8_t*>(L->up);
  d.down = static_cast<const uint8_t*>(L->down);
  d.sgate = static_cast<const uint8_t*>(L->sgate);
  d.sup = static_cast<const uint8_t*>(L->sup);
  d.sdown = static_cast<const uint8_t*>(L->sdown);
  d.router = static_cast<const __half*>(L->router);
  d.shared_gate = static_cast<const __half*>(L->shared_gate);
  d.x = x;
  d.out = out;
  d.err = reinterpret_cast<int*>(ws + o.err);
  d.ticket = reinterpret_cast<int*>(ws + o.ticket);
  d.logits = reinterpret_cast<float*>(ws + o.logits);
  d.gsh = reinterpret_cast<float*>(ws + o.gsh);
  d.idx = reinterpret_cast<uint32_t*>(ws + o.idx);
  d.wts = reinterpret_cast<float*>(ws + o.wts);
  d.plan = reinterpret_cast<dl::Plan*>(ws + o.plan);
  d.h = ws + o.h;
  d.T = tokens;
  d.H = L->hidden;
  d.I = L->inter;
  d.Is = L->shared_inter;
  d.E = L->experts;
  d.K = L->top_k;
  d.hstride = v2_hstride(L);
  d.rb_gu = row_bytes(L->kind_gate, L->hidden);
  d.rb_d = row_bytes(L->kind_down, L->inter);
  d.rb_sgu = L->shared_inter ? row_bytes(L->kind_sgate, L->hidden) : 0;
  d.rb_sd = L->shared_inter ? row_bytes(L->kind_sdown, L->shared_inter) : 0;
  int rc = SC_ERR_UNSUPPORTED;
  auto go = [&]<int KGU, int KD>() {
    if (L->dtype == SC_BF16) rc = dl::run<KGU, KD, __nv_bfloat16>(d, s);
    else rc = dl::run<KGU, KD, __half>(d, s);
  };
  auto with_down = [&]<int KGU>() {
    if (L->kind_down == SC_Q2_0) go.template operator()<KGU, SC_Q2_0>();
    else if (L->kind_down == SC_IQ3_S) go.template operator()<KGU, SC_IQ3_S>();
    else go.template operator()<KGU, SC_IQ3_XXS>();
  };
  if (L->kind_gate == SC_Q2_0) with_down.template operator()<SC_Q2_0>();
  else if (L->kind_gate == SC_IQ3_S) with_down.template operator()<SC_IQ3_S>();
  else with_down.template operator()<SC_IQ3_XXS>();
  return rc;
}

}  // namespace sc
