// The decode MoE block in three kernels (strata_mlx/fused.py:487-497 for a window of 1..8 tokens), chained with
// programmatic dependent launch so that each kernel's independent prologue overlaps the kernel before it:
//
//   route   router product (float16 weights, fused.py:334-354) and the shared expert's gate, then -- in the
//           last block to finish, found with an atomic ticket -- top-k with the softmax over the chosen logits
//           (fused.py:400-436, :491) and the plan: the distinct experts of the window (units), each with the
//           tokens that chose it. Router weights are loaded into registers before waiting on the previous kernel.
//   gate_up a block per (unit, 16 rows): the unit's gate and up rows (unit 0 is the shared expert, its rows fetched
//           before the wait) by 1-D bulk copies into shared memory, decoded into tensor-core fragments
//           (mma_decode.cuh), multiplied by the window's activations on mma.sync (bf16/f16, f32 sums), split over
//           eight warps along the columns and reduced once through shared memory; swiglu as mlx-lm rounds it
//           (blocks.py:230-238) -> h.
//   down    a block per 16 output rows: every unit's down rows and h through a ring of stages, each warp taking
//           whole units; then moe_combine's epilogue (fused.py:448-462) for those rows of every token, in MLX's
//           order, with the shared expert's sigmoid gate.
//
// Block types with fragment decoders: Q2_0, IQ3_S, IQ3_XXS (HasMma); other layers take moe.cu's chain.
#include <algorithm>
#include <mutex>
#include <vector>

#include "matvec.cuh"
#include "frag_decode.cuh"
#include "route.cuh"
#include "decode_layer.cuh"
#include "decode_dev.cuh"
#include "ep.cuh"

namespace sc {
namespace dl {

constexpr int WARPS = 8;                        // gate/up: eight warps along the columns (16 made a second wave of blocks)
constexpr int DN_WARPS = 16;                    // down: sixteen consumer warps, each taking whole units
constexpr int DN_THREADS = (DN_WARPS + 1) * 32;  // and a producer warp
constexpr int MAX_STAGES = 32;
constexpr int RT_WARPS = 16;                    // route: a router row per warp; the last block's top-k uses all 16
constexpr int RT_THREADS = RT_WARPS * 32;

// Phase stamps for a profiling build (-DSC_TRACE): %globaltimer per kernel, block and phase. Compiled out otherwise.
#ifdef SC_TRACE
__device__ unsigned long long g_trace[3][8192][8];
#define TRACE_POINT(k, p)                                                    \
  do {                                                                       \
    if (threadIdx.x == 0) {                                                  \
      unsigned long long t_;                                                 \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                  \
      if (blockIdx.x < 8192) g_trace[k][blockIdx.x][p] = t_;                 \
    }                                                                        \
  } while (0)
#define TRACE_SMID(k, p)                                                     \
  do {                                                                       \
    if (threadIdx.x == 0) {                                                  \
      unsigned int s_;                                                       \
      asm volatile("mov.u32 %0, %%smid;" : "=r"(s_));                         \
      if (blockIdx.x < 8192) g_trace[k][blockIdx.x][p] = s_ + 1;             \
    }                                                                        \
  } while (0)
#define TRACE_WARP(k, p)                                                     \
  do {                                                                       \
    if ((threadIdx.x & 31) == 0) {                                           \
      unsigned long long t_;                                                 \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                  \
      g_trace[k][4096 + (threadIdx.x >> 5)][p] = t_;                         \
    }                                                                        \
  } while (0)
#else
#define TRACE_POINT(k, p) \
  do {                    \
  } while (0)
#define TRACE_SMID(k, p) \
  do {                   \
  } while (0)
#define TRACE_WARP(k, p) \
  do {                   \
  } while (0)
#endif

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------------------------------- route

// MT: the tokens the last block's registers are laid out for (1, 2, 4 or MAXT, the window's tokens or more: a shorter
// tail for small windows, as expert parallel makes them: one token a rank)
template <typename T, int MT>
__global__ void __launch_bounds__(RT_THREADS) route_kernel(LayerDev L) {
  TRACE_POINT(0, 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  // block b: router rows of row block b % RB (warp w: row 16 (b % RB) + w; rows 0 .. E-1, row E the shared expert's
  // gate) for token group b / RB of the window (groups of tpg tokens)
  const int RB = int(gridDim.x) / L.rt_groups;
  const int row = (blockIdx.x % RB) * RT_WARPS + warp, tg = blockIdx.x / RB;
  const int H = L.H, E = L.E, K = L.K, T_ = L.T;
  const int tpg = (T_ + L.rt_groups - 1) / L.rt_groups, t0 = tg * tpg, t1 = min(T_, t0 + tpg);
  const __half* wrow = row < E ? L.router + int64_t(row) * H : (row == E && L.Is > 0 ? L.shared_gate : nullptr);
  const int chunks = H / 256;  // 16-byte chunks a lane reads
  // the first PRE chunks are fetched before the wait; more would spill at 128 registers a thread
  constexpr int PRE = 8;
  const uint4* wv = reinterpret_cast<const uint4*>(wrow) + lane;
  uint4 w[PRE];
  if (wrow) {
#pragma unroll
    for (int c = 0; c < PRE; ++c)
      if (c < chunks) w[c] = __ldg(wv + 32 * c);
  }
  pdl_wait();  // the window's activations are the previous kernel's output
  TRACE_POINT(0, 1);
  if (L.peers) {  // expert parallel over peer memory: every rank's tokens are in the window once it counts full
    if (tid == 0) {
      const uint64_t own = L.peers[L.rank];
      ep::wait_count(ep::at_u32(own, ep::xcount_off(L.par)), L.xtarget, L.err);
      TRACE_POINT(0, 7);
    }
    __syncthreads();
  }
  if (wrow) {
    for (int t = t0; t < t1; ++t) {
      const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const T*>(L.x) + int64_t(t) * H);
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < PRE; ++c)
        if (c < chunks) acc += dot8_half<T>(w[c], __ldcg(xr + lane + 32 * c));
      for (int c = PRE; c < chunks; ++c) acc += dot8_half<T>(__ldg(wv + 32 * c), __ldcg(xr + lane + 32 * c));
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
  TRACE_POINT(0, 2);
  if (tid == 0) s_last = atomic_add_acq_rel(L.ticket, 1) == int(gridDim.x) - 1;  // release this block's logits
  __syncthreads();
  if (!s_last) return;
  // only now may the gate/up kernel start (it reads the activations before it waits on this kernel), when the other
  // blocks of this kernel are leaving: launched while they held their SMs, its blocks went to the other SMs only
  // (these blocks' registers leave room for none), a quarter of the SMs without one
  pdl_launch_dependents();
  TRACE_POINT(0, 3);

  // ---- the last block: top-k of each token, the softmax and the plan (decode_dev.cuh)
  __shared__ TailSmem S;
  const int units = route_tail<MT>(L.logits, T_, E, K, L.e0, L.e1, S, tid, [] { __syncthreads(); });
  TRACE_POINT(0, 4);
  for (int p = tid; p < T_ * K; p += blockDim.x) {
    L.idx[p] = S.s_idx[p];
    L.wts[p] = S.s_w[p];
  }
  for (int u = tid; u < units; u += blockDim.x) {
    Unit v;
    v.expert = u == 0 ? -1 : S.s_expert[u];
    v.tokmask = u == 0 ? (L.Is > 0 ? (1u << T_) - 1u : 0u) : S.s_mask[u];
    v.kpack = u == 0 ? 0u : S.s_kpack[u];
    v.pad = 0;
    L.plan->unit[u] = v;
  }
  if (tid == 0) {
    L.plan->units = units;
    *L.ticket = 0;  // ready for the next call on this workspace
    if (L.peers) ++*L.step;  // this call's step number: the tag of its pair outputs (every rank counts alike)
    TRACE_POINT(0, 5);
  }
}

// ---------------------------------------------------------------------------------------------------- gate_up
//
// Items are (unit, block of 16 rows): the unit's gate and up rows [r0, r0 + 16) (one bulk copy each), eight warps
// each taking an eighth of the columns, one reduction through shared memory at the end. When every item of the
// largest window fits on the GPU at once (one or two tokens), a block takes one item; otherwise (LOOP) the grid is
// as many blocks as are resident and block b takes items b, b + grid, ... of the window's units, so that the units
// a window does not have cost nothing and the codebook is built once per block. (One kernel for both cost the
// one-item case registers and ~1.5 us a launch.)

struct GuSmem {
  int bar, tabs, xs, red, rows, total;
};

// The codebook copies a kernel keeps of its kind (rep_tab: every lane of a half-warp its own banks); the gate/up
// kernel holds eight (three blocks an SM still fit at one or two tokens), the down kernel sixteen
constexpr int GU_REP = 8;
constexpr int DN_REP = 16;
__host__ __device__ constexpr int tab_bytes_of(int kind, int rep) {
  return kind == SC_Q2_0 ? 0 : (kind == SC_IQ3_XXS ? 256 : 512) * rep * 8;
}

// rs: the shared-memory stride of the staged gate / up rows (their row bytes). With `alias` the warps' sums take
// the rows' space once the rows are decoded (the looping kernel), else a region of their own.
__host__ __device__ inline GuSmem gu_smem(int kind, int tokens, int H, int rs, bool alias) {
  GuSmem s;
  int o = 0;
  s.bar = o; o += 16;
  s.tabs = o; o += align16(tab_bytes_of(kind, GU_REP));
  s.xs = o; o += align16(tokens * (H + 32) * 2);
  const int rows_bytes = 2 * align16(RG * rs), red_bytes = WARPS * 32 * 8 * 4;
  if (alias) {
    s.red = s.rows = o; o += rows_bytes > red_bytes ? rows_bytes : red_bytes;
  } else {
    s.red = o; o += red_bytes;
    s.rows = o; o += rows_bytes;
  }
  s.total = o;
  return s;
}

// The warps' sums of an item (C fragments: rows g, g + 8; tokens 2t, 2t + 1) met through shared memory `red`, in
// warp order, and swiglu as mlx-lm rounds it -> h, in the order its consumer (the down product's decoder) wants.
template <int KD, typename T>
__device__ __forceinline__ void gu_store(const LayerDev& L, float* red, const float (&accg)[4], const float (&accu)[4],
                                         int u, int r0, int rows, uint32_t tokmask, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  // red[value][warp][lane]: the reducing thread (value q, lane L) reads eight consecutive words
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    red[(q * WARPS + warp) * 32 + lane] = accg[q];
    red[((4 + q) * WARPS + warp) * 32 + lane] = accu[q];
  }
  __syncthreads();
  if (tid < 128) {
    const int Lq = tid & 31, q = tid >> 5;
    float sg = 0.f, su = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      sg += red[(q * WARPS + w) * 32 + Lq];
      su += red[((4 + q) * WARPS + w) * 32 + Lq];
    }
    const int m = (q < 2 ? 0 : 8) + (Lq >> 2), tok = 2 * (Lq & 3) + (q & 1);
    if (m < rows && tok < L.T && ((tokmask >> tok) & 1u))
      static_cast<T*>(L.h)[(int64_t(u) * L.T + tok) * L.hstride + x_col(r0 + m, x_pairs(KD))] =
          from_f32<T>(swiglu_mlx<T>(sg, su));
  }
}

template <int KIND, int KD, typename T, bool LOOP>
__global__ void __launch_bounds__(WARPS * 32) gate_up_kernel(LayerDev L) {
  TRACE_POINT(1, 0);
  TRACE_SMID(1, 2);
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T_ = L.T, H = L.H;
  const int nrb = int(ceil_div(max(L.I, L.Is), RG));
  // the rows stay unpadded in shared memory: Q2_0's 576-byte rows meet four-way bank conflicts on their code loads,
  // but padding them (a bulk copy per row, or the block's own loads) made this latency-bound kernel slower
  const int rs = int(max(L.rb_gu, L.rb_sgu));
  const GuSmem S = gu_smem(KIND, T_, H, rs, LOOP);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S.bar);
  T* xs = reinterpret_cast<T*>(smem + S.xs);
  float* red = reinterpret_cast<float*>(smem + S.red);
  uint8_t* wg = smem + S.rows;
  uint8_t* wu = wg + align16(RG * rs);
  auto rows_of = [&](int j, int& u, int& r0) {
    u = j / nrb;
    r0 = (j % nrb) * RG;
    return u == 0 ? min(RG, L.Is - r0) : min(RG, L.I - r0);
  };
  // the block's first item; if it is the shared expert's (unit 0 is in every window), its rows come before the wait
  int u0, r00;
  const int rows0 = rows_of(blockIdx.x, u0, r00);
  if constexpr (!LOOP) {
    if (rows0 <= 0) {  // this block's rows lie beyond the unit's (the shared expert may be narrower)
      pdl_launch_dependents();
      return;
    }
  }
  const bool prefetched = u0 == 0 && rows0 > 0;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    if (prefetched) {
      mbar_arrive_expect_tx(bar, uint32_t(2 * rows0 * L.rb_sgu));
      bulk_load(wg, L.sgate + r00 * L.rb_sgu, uint32_t(rows0 * L.rb_sgu), bar);
      bulk_load(wu, L.sup + r00 * L.rb_sgu, uint32_t(rows0 * L.rb_sgu), bar);
    }
  }
  uint2* tabs = reinterpret_cast<uint2*>(smem + S.tabs);
  if constexpr (KIND != SC_Q2_0) build_grid_tab_rep2<T, KIND, GU_REP>(tabs, tid, blockDim.x);
  const uint2* tab = rep_tab<GU_REP>(tabs, lane);
  // the window's activations are complete once the route kernel let this kernel start (it waits before it does);
  // over peer memory, the window's count is read here too (already full), for the peers' writes' visibility
  if (L.peers) {
    if (tid == 0) ep::wait_count(ep::at_u32(L.peers[L.rank], ep::xcount_off(L.par)), L.xtarget, L.err);
    __syncthreads();
  }
  stage_x<T>(static_cast<const T*>(L.x), T_, H, xs, H + 32, tid, blockDim.x, x_pairs(KIND));
  pdl_wait();  // the routes
  TRACE_POINT(1, 1);
  // only now may the down kernel start: it reads the routes and the plan before it waits on this kernel
  pdl_launch_dependents();
  __shared__ Unit s_unit;
  __shared__ int s_units;
  const int g = lane >> 2;
  const int q4 = H / 128, n0 = 4 * (warp * q4 / WARPS), n1 = 4 * ((warp + 1) * q4 / WARPS);  // runs, by fours
  const T* xg = g < T_ ? xs + g * (H + 32) : nullptr;
  // tid 0: unit u's plan entry into s_unit, and the copies of its rows [r0, r0 + rows) unless already issued
  auto fetch = [&](int u, int r0, int rows, bool issued) {
    const int4 v = __ldcg(reinterpret_cast<const int4*>(&L.plan->unit[u]));
    s_unit = Unit{v.x, uint32_t(v.y), uint32_t(v.z), 0};
    if (!issued) {
      const int64_t rb = u == 0 ? L.rb_sgu : L.rb_gu;
      const uint8_t* g0 = u == 0 ? L.sgate + r0 * rb : L.gate + (int64_t(v.x) * L.I + r0) * rb;
      const uint8_t* u1 = u == 0 ? L.sup + r0 * rb : L.up + (int64_t(v.x) * L.I + r0) * rb;
      mbar_arrive_expect_tx(bar, uint32_t(2 * rows * rb));
      bulk_load(wg, g0, uint32_t(rows * rb), bar);
      bulk_load(wu, u1, uint32_t(rows * rb), bar);
    }
  };
  if constexpr (!LOOP) {
    if (tid == 0) {
      s_units = __ldcg(&L.plan->units);
      if (u0 < s_units) fetch(u0, r00, rows0, prefetched);
    }
    __syncthreads();
    if (u0 >= s_units) return;  // no such unit in this window (the grid is sized for the largest window)
    const int64_t rb = u0 == 0 ? L.rb_sgu : L.rb_gu;
    float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
    if (!mbar_wait(bar, 0, L.err)) return;
    TRACE_POINT(1, 3);
    frag_runs2<KIND, T, GU_REP>(wg + g * rb, wg + (g + 8) * rb, wu + g * rb, wu + (g + 8) * rb, xg, n0, n1, lane,
                                tab, accg, accu);
    TRACE_POINT(1, 4);
    gu_store<KD, T>(L, red, accg, accu, u0, r00, rows0, s_unit.tokmask, tid);
  } else {
    int it = 0;  // items this block took: the barrier's phase
    if (tid == 0) s_units = __ldcg(&L.plan->units);
    for (int j = blockIdx.x;; j += gridDim.x) {
      int u, r0;
      const int rows = rows_of(j, u, r0);
      if (tid == 0 && u < s_units && rows > 0) fetch(u, r0, rows, it == 0 && prefetched);
      __syncthreads();
      if (u >= s_units) break;  // past the window's units (the grid is sized for the largest window)
      if (rows <= 0) continue;  // rows beyond the unit's (the shared expert may be narrower)
      const int64_t rb = u == 0 ? L.rb_sgu : L.rb_gu;
      float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
      if (!mbar_wait(bar, uint32_t(it & 1), L.err)) break;
      frag_runs2<KIND, T, GU_REP>(wg + g * rb, wg + (g + 8) * rb, wu + g * rb, wu + (g + 8) * rb, xg, n0, n1, lane,
                                  tab, accg, accu);
      __syncthreads();  // every warp is done with the rows: their space takes the sums
      gu_store<KD, T>(L, red, accg, accu, u, r0, rows, s_unit.tokmask, tid);
      __syncthreads();  // the sums are read: the next item's rows may land in their space
      ++it;
    }
  }
}

// ---------------------------------------------------------------------------------------------------- down
//
// One block per 16 rows of the output; a ring of stages, one per unit (its 16 down rows and its h); each warp takes
// whole units (all columns), so that a unit's outputs need no reduction; then moe_combine for those rows.

struct DnSmem {
  int bars, tabs, plan, wts, ys, stages, total;
};

__host__ __device__ inline DnSmem dn_smem(int kind, int tokens, int K, int stage_bytes, int stages) {
  DnSmem s;
  int o = 0;
  s.bars = o; o += align16(2 * MAX_STAGES * 8);
  s.tabs = o; o += align16(tab_bytes_of(kind, DN_REP));
  s.plan = o; o += align16(int(sizeof(Plan)));
  s.wts = o; o += align16(tokens * (K + 1) * 4);
  s.ys = o; o += align16(tokens * (K + 1) * RC * 4);
  s.stages = align16(o); o = s.stages + stages * stage_bytes;
  s.total = o;
  return s;
}

// Runs [n0, n1) of a unit's 16 down rows (in the stage `st`) times its h: the h columns of those runs first, from L2
// into the stage (every load in flight at once; a bulk copy issued after the wait took ~1.3 us to land, these ~0.6),
// then the products. acc: the C fragment (rows g, g + 8; tokens 2t, 2t + 1).
template <int KIND, typename T>
__device__ __forceinline__ void down_piece(const LayerDev& L, uint8_t* st, int hoff, int u, int n0, int n1, bool shared,
                                           uint32_t mask, const uint2* tab, int lane, float (&acc)[4]) {
  const int T_ = L.T, g = lane >> 2;
  T* hs = reinterpret_cast<T*>(st + hoff);
  {
    const T* hu = static_cast<const T*>(L.h) + int64_t(u) * T_ * L.hstride;
    const int per = 4 * (n1 - n0), n16 = T_ * per;  // 16-byte pieces a token, in all
    constexpr int PER = 2;  // a one-token unit's h is 64 pieces: two a lane (more only cost registers)
    for (int i0 = 0; i0 < n16; i0 += 32 * PER) {
      uint4 v[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int i = i0 + 32 * j + lane;
        if (i < n16) v[j] = __ldcg(reinterpret_cast<const uint4*>(hu + (i / per) * L.hstride + 32 * n0 + 8 * (i % per)));
      }
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int i = i0 + 32 * j + lane;
        if (i < n16) *reinterpret_cast<uint4*>(hs + (i / per) * L.hstride + 32 * n0 + 8 * (i % per)) = v[j];
      }
    }
    __syncwarp();
  }
  const int64_t rb = shared ? L.rb_sd : L.rb_d;
  const bool mine = g < T_ && ((mask >> g) & 1u);
  acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  frag_runs<KIND, T, DN_REP>(st + g * rb, st + (g + 8) * rb, mine ? hs + g * L.hstride : nullptr, n0, n1, lane, tab,
                             acc);
}

template <int KIND, typename T>
__global__ void __launch_bounds__(DN_THREADS) down_kernel(LayerDev L) {
  TRACE_POINT(2, 0);
  TRACE_SMID(2, 6);  // (slots 6 and 7 stamp the peer-memory epilogue; a single-device trace uses 6 for the SM)
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T_ = L.T, K = L.K, H = L.H;
  const DnSmem S = dn_smem(KIND, T_, K, L.dn_stage, L.dn_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S.bars);
  uint64_t* empty = full + MAX_STAGES;
  Plan* plan = reinterpret_cast<Plan*>(smem + S.plan);
  float* wts = reinterpret_cast<float*>(smem + S.wts);  // (T, K) routes' weights, then (T) the shared gates
  float* ys = reinterpret_cast<float*>(smem + S.ys);    // (T, K + 1, 16): routed outputs, then the shared one
  uint8_t* stage0 = smem + S.stages;
  const int r0 = blockIdx.x * RC;
  pdl_launch_dependents();  // the next layer's router may load its weights now

  if (tid == 0) {
    for (int s = 0; s < L.dn_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // a stage is one unit's, consumed by one warp
    }
    fence_mbar_init();
  }
  uint2* tabs = reinterpret_cast<uint2*>(smem + S.tabs);
  if constexpr (KIND != SC_Q2_0) build_grid_tab_rep2<T, KIND, DN_REP>(tabs, tid, blockDim.x);
  const uint2* tab = rep_tab<DN_REP>(tabs, lane);
  // the routes and the plan are complete once the gate/up kernel let this kernel start (it waits before it does)
  for (int i = tid; i < int(sizeof(Plan) / 16); i += blockDim.x)
    reinterpret_cast<int4*>(plan)[i] = __ldcg(reinterpret_cast<const int4*>(L.plan) + i);
  for (int i = tid; i < T_ * K; i += blockDim.x) wts[i] = __ldcg(L.wts + i);
  for (int i = tid; i < T_; i += blockDim.x) wts[T_ * K + i] = L.Is > 0 ? __ldcg(L.gsh + i) : -INFINITY;
  __syncthreads();
  TRACE_POINT(2, 1);
  const int units = plan->units;
  // the down rows of the first units do not wait for the gate/up kernel; their h does, and the consumer warp copies
  // it into the stage itself (a bulk copy issued by the producer after the wait took ~1.3 us to land, the warp's
  // loads ~0.6; loads of h inside the product's loop serialised it)
  const int hoff = align16(RC * int(max(L.rb_d, L.rb_sd)));
  auto weights = [&](int u, int s) {
    uint8_t* dst = stage0 + s * L.dn_stage;
    if (u == 0) {
      if (L.Is > 0) bulk_load(dst, L.sdown + r0 * L.rb_sd, uint32_t(RC * L.rb_sd), &full[s]);
    } else {
      bulk_load(dst, L.down + (int64_t(plan->unit[u].expert) * H + r0) * L.rb_d, uint32_t(RC * L.rb_d), &full[s]);
    }
  };
  auto weight_bytes = [&](int u) -> uint32_t { return u == 0 ? uint32_t(L.Is > 0 ? RC * L.rb_sd : 0) : uint32_t(RC * L.rb_d); };
  if (warp == DN_WARPS && lane == 0) {
    for (int u = 0; u < min(units, L.dn_stages); ++u) {
      if (weight_bytes(u) == 0) {  // no shared expert: nothing to load for unit 0
        mbar_arrive(&full[u]);
        continue;
      }
      mbar_arrive_expect_tx(&full[u], weight_bytes(u));
      weights(u, u);
    }
  }
  pdl_wait();  // h
  TRACE_POINT(2, 2);

  if (warp == DN_WARPS) {  // ---- producer: the ring's later units (unit 0, the shared expert, is never one)
    if (lane == 0) {
      for (int u = L.dn_stages; u < units; ++u) {
        const int s = u % L.dn_stages;
        if (!mbar_wait(&empty[s], ((u / L.dn_stages) - 1) & 1, L.err)) break;
        mbar_arrive_expect_tx(&full[s], weight_bytes(u));
        weights(u, s);
      }
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3;
  {
    // ---- consumers, a ring: every use of a stage goes to the same warp, in order (unit u to warp (u % stages) %
    // DN_WARPS), so that a warp waits on a stage's n-th phase only after it consumed the (n-1)-th: a wait on parity 1
    // while the barrier is still in its first phase would return at once. The warp's units are walked directly (a
    // scan of every unit took a runtime modulo per unit: ~1 us before the last warps reached their first unit).
    // Stage count S <= DN_WARPS or a multiple of it; the warp owns stages w, w + DN_WARPS, ... < S; after unit u in
    // stage s comes u + DN_WARPS while s + DN_WARPS < S, else stage w of the next round.
    const int S_ = L.dn_stages;
    for (int u = warp < S_ ? warp : units, s = warp; u < units;
         u = s + DN_WARPS < S_ ? u + DN_WARPS : u - s + S_ + warp, s = u % S_) {
      if (!mbar_wait(&full[s], (u / S_) & 1, L.err)) break;
      const bool shared = u == 0;
      if (shared && L.Is == 0) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        continue;
      }
      const uint32_t mask = plan->unit[u].tokmask, kpack = plan->unit[u].kpack;
      float acc[4];
      down_piece<KIND, T>(L, stage0 + s * L.dn_stage, hoff, u, 0, (shared ? L.Is : L.I) / 32, shared, mask, tab,
                          lane, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // C fragment: rows g, g + 8; tokens 2t, 2t + 1
        const int m = (q < 2 ? 0 : 8) + g, tok = 2 * t + (q & 1);
        if (tok < T_ && ((mask >> tok) & 1u)) {
          const int k = shared ? K : int((kpack >> (4 * tok)) & 15u);
          ys[(tok * (K + 1) + k) * RC + m] = round_to<T>(acc[q]);
        }
      }
    }
  }
  TRACE_POINT(2, 3);
  named_sync(1, DN_WARPS * 32);
  TRACE_POINT(2, 4);
  if (L.peers) {  // expert parallel over peer memory: each pair's output to its token's rank, as tagged words
    // a thread a pair (tok, k) of this rank's experts: its 16 rows [r0, r0 + 16) are eight words of the owner's Y,
    // each tagged with this call's step; then a thread a token for the shared expert's rows (local)
    const size_t yo = ep::yoff(L.par, T_, L.tl, K, H);
    const uint32_t step = __ldcg(L.step);
    auto pack16 = [&](const float* y, uint4 (&v)[2]) {  // 16 floats -> 16 values of T
      uint32_t w[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const T a = from_f32<T>(y[2 * q]), b = from_f32<T>(y[2 * q + 1]);
        w[q] = uint32_t(*reinterpret_cast<const uint16_t*>(&a)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&b)) << 16);
      }
      v[0] = make_uint4(w[0], w[1], w[2], w[3]);
      v[1] = make_uint4(w[4], w[5], w[6], w[7]);
    };
    for (int i = tid; i < T_ * K; i += DN_WARPS * 32) {
      const int tok = i / K, k = i % K;
      const int e = int(__ldcg(L.idx + i));
      if (e < L.e0 || e >= L.e1) continue;
      uint4 v[2];
      pack16(ys + (tok * (K + 1) + k) * RC, v);
      uint64_t* dst = reinterpret_cast<uint64_t*>(L.peers[tok / L.tl] + yo) + (int64_t(tok % L.tl) * K + k) * (H / 2) +
                      r0 / 2;
      const uint32_t w[8] = {v[0].x, v[0].y, v[0].z, v[0].w, v[1].x, v[1].y, v[1].z, v[1].w};
#pragma unroll
      for (int q = 0; q < 8; ++q) ep::store_tagged(dst + q, w[q], step);
    }
    for (int tok = tid; tok < T_; tok += DN_WARPS * 32) {
      uint4 v[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      if (L.Is > 0) pack16(ys + (tok * (K + 1) + K) * RC, v);
      uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(L.sout) + int64_t(tok) * H + r0);
      dst[0] = v[0];
      dst[1] = v[1];
    }
    // the shared expert's outputs are local: this rank's combine reads them once every block counted here
    named_sync(1, DN_WARPS * 32);
    if (tid == 0) {
      __threadfence();
      atomicAdd(L.done, 1u);
    }
    TRACE_POINT(2, 6);
    return;
  }
  if (L.ypairs) {  // expert parallel: the pairs' outputs (zero for other ranks' experts) and the shared expert's
    for (int i = tid; i < T_ * RC; i += DN_WARPS * 32) {
      const int tok = i / RC, m = i % RC;
      const float* yk = ys + tok * (K + 1) * RC + m;
      for (int k = 0; k < K; ++k) {
        const int e = int(__ldcg(L.idx + tok * K + k));
        const float v = e >= L.e0 && e < L.e1 ? yk[k * RC] : 0.f;
        static_cast<T*>(L.ypairs)[(int64_t(tok) * K + k) * H + r0 + m] = from_f32<T>(v);
      }
      static_cast<T*>(L.sout)[int64_t(tok) * H + r0 + m] = from_f32<T>(L.Is > 0 ? yk[K * RC] : 0.f);
    }
    return;
  }
  // ---- moe_combine for rows [r0, r0 + 16) of every token
  for (int i = tid; i < T_ * RC; i += DN_WARPS * 32) {
    const int tok = i / RC, m = i % RC;
    const float* yk = ys + tok * (K + 1) * RC + m;  // routed output k at yk[k * RC]
    const float sv = L.Is > 0 ? yk[K * RC] : 0.f;
    const float gv = L.Is > 0 ? round_to<T>(wts[T_ * K + tok]) : -INFINITY;
    static_cast<T*>(L.out)[int64_t(tok) * H + r0 + m] =
        from_f32<T>(combine_one<T, RC>(yk, wts + tok * K, K, gv, sv));
  }
  TRACE_POINT(2, 5);
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

// Blocks of `kern` (threads, dynamic shared memory) resident at once on the current device, 0 when CUDA cannot say;
// remembered per device, kernel and size (a launch asks for each layer)
static int resident_blocks(const void* kern, int threads, int smem) {
  struct Entry {
    int dev;
    const void* kern;
    int threads, smem, blocks;
  };
  static std::mutex m;
  static std::vector<Entry> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(m);
  for (const Entry& e : cache)
    if (e.dev == dev && e.kern == kern && e.threads == threads && e.smem == smem) return e.blocks;
  int per_sm = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, size_t(smem)) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  cache.push_back(Entry{dev, kern, threads, smem, per_sm * sms});
  return per_sm * sms;
}

template <int KGU, int KD, typename T>
static int run(LayerDev L, cudaStream_t s, int stage) {
  const int max_units = L.T * L.K + 1;
  const int gu_rs = int(std::max(L.rb_gu, L.rb_sgu));
  // down: a stage is one unit's 16 rows and its h; enough stages for every warp to hold one and the next in flight
  L.dn_stage = align16(RC * int(std::max(L.rb_d, L.rb_sd))) + align16(L.T * L.hstride * 2);
  const int dn_room = std::min(144 * 1024, 227 * 1024 - dn_smem(KD, L.T, L.K, L.dn_stage, 0).total);
  L.dn_stages = std::max(2, std::min({MAX_STAGES, max_units, dn_room / L.dn_stage}));
  if (L.dn_stages > DN_WARPS) L.dn_stages -= L.dn_stages % DN_WARPS;  // every warp the same number of stages
  // one down block an SM: two on one SM (where the gate/up blocks left room first) ran twice as long, and the
  // layer waits for the slowest; more than half an SM's shared memory keeps a second one off
  const int dn_total = std::max(dn_smem(KD, L.T, L.K, L.dn_stage, L.dn_stages).total, 116 * 1024);
  // gate/up: one block an item when every item of the largest window is resident at once, else looping blocks (as
  // many as are resident), whose sums take the rows' space
  const int gu_items = max_units * int(ceil_div(std::max(L.I, L.Is), RG));
  const int gu_one = gu_smem(KGU, L.T, L.H, gu_rs, false).total, gu_alias = gu_smem(KGU, L.T, L.H, gu_rs, true).total;
  if (gu_alias > 227 * 1024 || dn_total > 227 * 1024) return SC_ERR_SHAPE;

  auto kr = L.T == 1   ? route_kernel<T, 1>
            : L.T == 2 ? route_kernel<T, 2>
            : L.T <= 4 ? route_kernel<T, 4>
                       : route_kernel<T, MAXT>;
  auto kg1 = gate_up_kernel<KGU, KD, T, false>;
  auto kgl = gate_up_kernel<KGU, KD, T, true>;
  auto kd = down_kernel<KD, T>;
  // the dynamic shared memory a launch may take is raised to what it needs, per kernel: the gate/up and down
  // kernels are shared by the paths of several block-type mixes, each with its own sizes
  int resident = 0;
  if (gu_one <= 227 * 1024) {
    if (int rc = raise_smem(reinterpret_cast<const void*>(kg1), gu_one, "decode gate_up smem attribute")) return rc;
    resident = resident_blocks(reinterpret_cast<const void*>(kg1), WARPS * 32, gu_one);
  }
  const bool gu_loop = gu_items > resident;
  const int gu_total = gu_loop ? gu_alias : gu_one;
  auto kg = gu_loop ? kgl : kg1;
  int grid_g = gu_items;
  if (gu_loop) {
    if (int rc = raise_smem(reinterpret_cast<const void*>(kgl), gu_alias, "decode gate_up smem attribute")) return rc;
    grid_g = resident_blocks(reinterpret_cast<const void*>(kgl), WARPS * 32, gu_alias);
    if (grid_g <= 0) return cuda_failed(cudaGetLastError(), "decode gate_up occupancy");
  }
  if (int rc = raise_smem(reinterpret_cast<const void*>(kd), dn_total, "decode down smem attribute")) return rc;
  // route: the window's tokens in groups of two over as many groups of blocks (one token: one group)
  L.rt_groups = (L.T + 1) / 2;
  const int grid_r = int(ceil_div(L.E + 1, RT_WARPS)) * L.rt_groups;
  const int grid_d = L.H / RC;
  if (stage < 0 || stage == 0)
    if (cudaError_t e = launch_pdl(kr, grid_r, RT_THREADS, 0, s, L)) return cuda_failed(e, "decode route launch");
  if (stage < 0 || stage == 1)
    if (cudaError_t e = launch_pdl(kg, grid_g, WARPS * 32, gu_total, s, L)) return cuda_failed(e, "decode gate_up launch");
  if (stage < 0 || stage == 2)
    if (cudaError_t e = launch_pdl(kd, grid_d, DN_THREADS, dn_total, s, L)) return cuda_failed(e, "decode down launch");
  return SC_OK;
}

}  // namespace dl

#ifdef SC_TRACE
extern "C" SC_API int sc_trace_read(void* host) {
  return cudaMemcpyFromSymbol(host, dl::g_trace, sizeof(dl::g_trace)) == cudaSuccess ? 0 : -1;
}
extern "C" SC_API int sc_trace_clear() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, dl::g_trace) != cudaSuccess) return -1;
  return cudaMemset(p, 0, sizeof(dl::g_trace)) == cudaSuccess ? 0 : -1;
}
#endif

// Whether the three-kernel path takes the layer, and the scratch it needs beyond the common header.
bool v2_takes(const sc_moe_layer* L, int tokens) {
  auto mma_kind = [](int k) { return k == SC_Q2_0 || k == SC_IQ3_S || k == SC_IQ3_XXS; };
  if (L->dtype != SC_BF16 && L->dtype != SC_F16) return false;
  if (tokens < 1 || tokens > dl::MAXT || L->top_k > TOPK_MAX_K || tokens * L->top_k > dl::MAXU - 1) return false;
  if (L->experts > 1024) return false;  // the last route block's sixteen warps take 64 logits each
  if (!mma_kind(L->kind_gate) || L->kind_up != L->kind_gate || !mma_kind(L->kind_down)) return false;
  if (L->shared_inter > 0 && (L->kind_sgate != L->kind_gate || L->kind_sup != L->kind_gate || L->kind_sdown != L->kind_down))
    return false;
  if (L->hidden % 256 || L->hidden / 256 > dl::MAX_ROUTER_CHUNKS || L->hidden % dl::RC) return false;
  // the decoders take runs four at a time: rows of 128 weights
  if (L->inter % 128 || L->shared_inter % 128) return false;
  if (row_bytes(L->kind_gate, L->hidden) % 16) return false;  // 16-row bulk copies start on 16 bytes
  return true;
}

int v2_run(const sc_moe_layer* L, const void* x, int tokens, void* out, uint8_t* ws, const V2Offsets& o,
           cudaStream_t s, int stage, const V2Ep& ep) {
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
  d.e0 = ep.e0;
  d.e1 = ep.e1 < 0 ? L->experts : ep.e1;
  d.ypairs = ep.ypairs;
  d.sout = ws + o.sout;
  d.peers = ep.peers;
  d.G = ep.G;
  d.rank = ep.rank;
  d.tl = ep.tl;
  d.par = ep.par;
  d.xtarget = uint32_t(ep.G * ep::COMBINE_BLOCKS);
  d.step = ep.step;
  d.done = ep.done;
  int rc = SC_ERR_UNSUPPORTED;
  auto go = [&]<int KGU, int KD>() {
    if (L->dtype == SC_BF16) rc = dl::run<KGU, KD, __nv_bfloat16>(d, s, stage);
    else rc = dl::run<KGU, KD, __half>(d, s, stage);
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
