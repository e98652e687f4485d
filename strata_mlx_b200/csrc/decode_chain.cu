// The decode block as one persistent kernel over a chain of layers (strata_mlx/fused.py:487-497, _Routed.__call__,
// layer after layer for a window of 1..8 tokens): sc_moe_decode_chain.
//
// One block per SM, all resident (a cooperative launch), seventeen warps: sixteen consumer warps in two groups of
// eight and one producer warp that streams weight rows into a ring of four shared-memory stages with 1-D bulk
// copies. A layer is five phases separated by grid-wide barriers (a count in the workspace, bounded waits):
//
//   R  router rows: each block's share of the E router rows and the shared expert's gate row, copied into shared
//      memory by the producer during the previous layer, times the window -> logits (global)
//   -- barrier A
//   P  every block routes the whole window itself (decode_dev.cuh's route tail: top-k, softmax, the plan of units)
//   G  gate/up items (a unit's 16 gate rows and 16 up rows), split evenly over the blocks: a group's eight warps
//      split the columns, their sums meet in shared memory, swiglu as mlx-lm rounds it -> h (global)
//   -- barrier B
//   D  down items (a unit's 128 output rows and its h), split evenly: a warp per tile of 16 rows, the pair's
//      output rounded to the activations' type -> Y (global); the producer fetched the rows during G
//   -- barrier C
//   C  each block combines a slice of the window (moe_combine in MLX's add order) -> the next layer's window
//   -- barrier D (only when the next layer takes it: with refeed, or after the last layer, it is not needed)
//
// The arithmetic of an item is that of the three-kernel block (decode_layer.cu): the same fragment decoders, the
// same eight column slices summed in the same order, a unit's 16 rows of down by one warp, the same route tail and
// combine. The two give the same bits, which the expert-parallel path (built on the three kernels) relies on.
//
// Every wait is bounded (about a second): a wait that gives up records SC_ERR_TIMEOUT in the error word and the
// block leaves; the workspace must then be zeroed before its next use (the barrier's count is left mid-way).
#include <algorithm>

#include "matvec.cuh"
#include "frag_decode.cuh"
#include "decode_layer.cuh"
#include "decode_dev.cuh"

namespace sc {
namespace ck {

using dl::MAXT;
using dl::MAXU;
using dl::named_sync;

constexpr int MAXL = 64;                 // layers a launch takes
constexpr int GW = 8;                    // warps of a group (one item at a time)
constexpr int GROUPS = 2;
constexpr int CW = GW * GROUPS;          // consumer warps: the route tail's sixteen
constexpr int CT = CW * 32;
constexpr int THREADS = CT + 32;         // and the producer warp
constexpr int MAX_STAGES = 8;            // a ring of an even number of stages: stage s is group s % 2's
constexpr int DN_ROWS = GW * 16;         // output rows of a down item: a tile of 16 rows a warp
constexpr int RG = 16;                   // gate/up rows of an item
constexpr int CONS_BAR = 1;              // named barrier of the consumer threads; group g uses 2 + g
constexpr long long WAIT_LIMIT = 2000000000LL;  // clock cycles: about a second

// Phase stamps for a profiling build (-DSC_TRACE): %globaltimer per block, layer and phase. Compiled out otherwise.
#ifdef SC_TRACE
__device__ unsigned long long g_ctrace[160][MAXL][16];
#define CK_TRACE(l, p)                                                               \
  do {                                                                               \
    unsigned long long t_;                                                           \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                           \
    if (blockIdx.x < 160 && (l) < MAXL) g_ctrace[blockIdx.x][(l)][(p)] = t_;         \
  } while (0)
// per item of a layer (its index in the block's list, first 5): issued, data in, done
__device__ unsigned long long g_itrace[160][MAXL][16];
#define CK_ITRACE(l, i, p)                                                           \
  do {                                                                               \
    unsigned long long t_;                                                           \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                           \
    if (blockIdx.x < 160 && (l) < MAXL && (i) < 5) g_itrace[blockIdx.x][(l)][3 * (i) + (p)] = t_; \
  } while (0)
#else
#define CK_ITRACE(l, i, p) \
  do {                     \
  } while (0)
#define CK_TRACE(l, p) \
  do {                 \
  } while (0)
#endif

struct LayerW {
  const uint8_t *gate, *up, *down, *sgate, *sup, *sdown;
  const __half *router, *shared_gate;
  int kgu, kd;
  int rb_gu, rb_d, rb_sd;  // bytes of a row: gate / up (and the shared expert's), down, the shared expert's down
};

struct Args {
  LayerW w[MAXL];
  int L, T, H, I, Is, E, K, refeed, hstride, rt_rows, wmax, stages;
  const void* x;
  void* out;
  int* err;
  unsigned* bar;   // [0] arrivals (counted up within a launch), [1] blocks past the last barrier (resets both)
  float *logits, *gsh;
  uint32_t* idx;   // (L, T, K): every layer's routes
  float* wts;      // (L, T, K)
  void *h, *Y, *Xn;  // (MAXU, T, hstride), (T, K + 1, H), (T, H) of the activations' type
};

struct Smem {
  int bars, tabs, x, router, plan, routes, red, stages, stage, hoff, total;
};

__host__ __device__ inline Smem smem_of(int T, int H, int rt_rows, int wmax, int hstride, int stages) {
  Smem s;
  int o = 0;
  s.bars = o; o += (2 * MAX_STAGES + 8) * 8;
  s.tabs = o; o += align16(GRID_TAB_BYTES);
  s.x = o; o += align16(T * (H + 32) * 2);
  s.router = o; o += align16(rt_rows * H * 2);
  s.plan = o; o += align16(int(sizeof(dl::Plan)));
  s.routes = o; o += align16((MAXT * TOPK_MAX_K + MAXT) * 4);
  const int red = std::max(int(sizeof(dl::TailSmem)), GROUPS * GW * 32 * 8 * 4);
  s.red = o; o += align16(red);
  s.hoff = align16(wmax);
  s.stage = s.hoff + align16(T * hstride * 2);
  s.stages = align16(o); o = s.stages + stages * s.stage;
  s.total = o;
  return s;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// All blocks' consumer threads meet: this block's writes before it are visible to every block after it. Thread 0
// adds to the launch's arrival count and waits (bounded) for `target` arrivals. Returns false when a wait gave up.
__device__ __forceinline__ bool grid_barrier(unsigned* bar, unsigned target, int* err, int* s_abort) {
  named_sync(CONS_BAR, CT);
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    if (ld_acquire(bar) < target) {
      const long long start = clock64();
      while (ld_acquire(bar) < target) {
        if (clock64() - start > WAIT_LIMIT) {
          record_error(err, SC_ERR_TIMEOUT);
          *s_abort = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  named_sync(CONS_BAR, CT);
  return *s_abort == 0;
}

// The items of a layer: gate/up items (unit, 16 rows) and down items (unit, 128 output rows), unit 0 the shared
// expert (when there is one); block `cta` of G takes [n * cta / G, n * (cta + 1) / G) of each list.
struct Items {
  int g0, g1, d0, d1, nrb, nrbs, nd;
  __device__ void unit_row_gu(int j, int& u, int& r0) const {
    if (j < nrbs) { u = 0; r0 = RG * j; }
    else { u = 1 + (j - nrbs) / nrb; r0 = RG * ((j - nrbs) % nrb); }
  }
  __device__ void unit_row_dn(int j, bool shared, int& u, int& c0) const {
    const int q = j / nd;
    u = shared ? q : q + 1;
    c0 = DN_ROWS * (j % nd);
  }
};

__device__ __forceinline__ Items items_of(int units, int I, int Is, int H, int cta, int G) {
  Items it;
  it.nrb = I / RG;
  it.nrbs = Is / RG;
  it.nd = H / DN_ROWS;
  const int ngu = it.nrbs + (units - 1) * it.nrb;
  const int ndn = (Is > 0 ? units : units - 1) * it.nd;
  it.g0 = ngu * cta / G;
  it.g1 = ngu * (cta + 1) / G;
  it.d0 = ndn * cta / G;
  it.d1 = ndn * (cta + 1) / G;
  return it;
}

// ---- the producer warp: router rows one layer ahead, then the layer's items into the ring

template <typename T>
__device__ void producer(const Args& A, uint8_t* smem, const Smem& S, int r_lo, int r_hi) {
  const int STAGES = A.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S.bars);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* rt_full = empty + MAX_STAGES;
  uint64_t* rt_free = rt_full + 1;
  uint64_t* plan_ready = rt_free + 1;
  uint64_t* hready = plan_ready + 1;
  uint64_t* prod_done = hready + 1;
  const dl::Plan* plan = reinterpret_cast<const dl::Plan*>(smem + S.plan);
  uint8_t* rt = smem + S.router;
  uint8_t* stage0 = smem + S.stages;
  const int H = A.H, E = A.E, T_ = A.T;
  const uint32_t hbytes = uint32_t(T_ * A.hstride * 2);
  uint32_t issued = 0;  // items issued, for the drain at the end

  auto router = [&](int l) {
    const LayerW& w = A.w[l];
    uint32_t bytes = 0;
    for (int r = r_lo; r < r_hi; ++r)
      if (r < E || A.Is > 0) bytes += uint32_t(H * 2);
    if (bytes == 0) {
      mbar_arrive(rt_full);
      return;
    }
    mbar_arrive_expect_tx(rt_full, bytes);
    for (int r = r_lo; r < r_hi; ++r) {
      const __half* src = r < E ? w.router + int64_t(r) * H : (A.Is > 0 ? w.shared_gate : nullptr);
      if (src) bulk_load(rt + (r - r_lo) * H * 2, src, uint32_t(H * 2), rt_full);
    }
  };

  router(0);
  uint32_t it = 0;
  bool ok = true;
  for (int l = 0; l < A.L && ok; ++l) {
    const LayerW& w = A.w[l];
    if (!(ok = mbar_wait(plan_ready, l & 1, A.err))) break;
    CK_TRACE(l, 11);
    if (l + 1 < A.L) {
      if (!(ok = mbar_wait(rt_free, l & 1, A.err))) break;
      router(l + 1);
    }
    CK_TRACE(l, 15);
    const uint32_t it_layer = it;
    const int units = plan->units;
    const Items I_ = items_of(units, A.I, A.Is, H, blockIdx.x, gridDim.x);
    const int rb_gu = w.rb_gu, rb_d = w.rb_d, rb_sgu = w.rb_gu, rb_sd = w.rb_sd;
    auto slot = [&](int s) -> bool {
      if (it >= uint32_t(STAGES) && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, A.err)) return false;
      return true;
    };
    for (int j = I_.g0; j < I_.g1; ++j, ++it) {
      int u, r0;
      I_.unit_row_gu(j, u, r0);
      const int s = int(it % STAGES);
      if (!(ok = slot(s))) break;
      uint8_t* dst = stage0 + s * S.stage;
      const bool sh = u == 0 && A.Is > 0;
      const int rb = sh ? rb_sgu : rb_gu;
      const uint32_t bytes = uint32_t(RG * rb);
      mbar_arrive_expect_tx(&full[s], 2 * bytes);
      if (sh) {
        bulk_load(dst, w.sgate + r0 * rb, bytes, &full[s]);
        bulk_load(dst + align16(int(bytes)), w.sup + r0 * rb, bytes, &full[s]);
      } else {
        const int64_t e = plan->unit[u].expert;
        bulk_load(dst, w.gate + (e * A.I + r0) * rb, bytes, &full[s]);
        bulk_load(dst + align16(int(bytes)), w.up + (e * A.I + r0) * rb, bytes, &full[s]);
      }
      issued = it + 1;
      CK_ITRACE(l, it - it_layer, 0);
    }
    if (!ok) break;
    CK_TRACE(l, 12);
    bool have_h = false;
    for (int j = I_.d0; j < I_.d1; ++j, ++it) {
      int u, c0;
      I_.unit_row_dn(j, A.Is > 0, u, c0);
      const int s = int(it % STAGES);
      if (!(ok = slot(s))) break;
      uint8_t* dst = stage0 + s * S.stage;
      const bool sh = u == 0;
      const int rb = sh ? rb_sd : rb_d;
      const uint32_t bytes = uint32_t(DN_ROWS * rb);
      mbar_arrive_expect_tx(&full[s], bytes + hbytes);
      if (sh) bulk_load(dst, w.sdown + c0 * rb, bytes, &full[s]);
      else bulk_load(dst, w.down + (int64_t(plan->unit[u].expert) * H + c0) * rb, bytes, &full[s]);
      if (!have_h) {  // the units' h are complete once every block passed barrier B
        if (!(ok = mbar_wait(hready, l & 1, A.err))) break;
        fence_proxy_async();  // h was written by other blocks' threads; the bulk copy reads it as the async proxy
        have_h = true;
        CK_TRACE(l, 13);
      }
      bulk_load(dst + S.hoff, static_cast<const uint8_t*>(A.h) + size_t(u) * hbytes, hbytes, &full[s]);
      issued = it + 1;
      CK_ITRACE(l, it - it_layer, 0);
    }
    if (!ok) break;
    CK_TRACE(l, 14);
    if (!have_h && !(ok = mbar_wait(hready, l & 1, A.err))) break;  // every phase of hready is waited once
    mbar_arrive(prod_done);
  }
  // leave no copy in flight: wait (bounded) for the last phase each stage was filled for
  for (uint32_t i = issued > uint32_t(STAGES) ? issued - STAGES : 0; i < issued; ++i)
    mbar_wait(&full[i % STAGES], (i / STAGES) & 1, A.err);
}

// ---- consumers: a gate/up item is split over a group's eight warps by runs, four at a time (the three-kernel
// block's gate_up_kernel split); a down item gives each warp a tile of 16 rows over every run (its down_piece)

__device__ __forceinline__ void gu_runs(int H, int w, int& n0, int& n1) {
  const int q4 = H / 128;
  n0 = 4 * (w * q4 / GW);
  n1 = 4 * ((w + 1) * q4 / GW);
}

template <typename F>
__device__ __forceinline__ void by_kind(int kind, F&& f) {
  if (kind == SC_Q2_0) f.template operator()<SC_Q2_0>();
  else if (kind == SC_IQ3_S) f.template operator()<SC_IQ3_S>();
  else f.template operator()<SC_IQ3_XXS>();
}

template <typename T, int MT>
__global__ void __launch_bounds__(THREADS, 1) chain_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int T_ = A.T, H = A.H, E = A.E, K = A.K;
  const Smem S = smem_of(T_, H, A.rt_rows, A.wmax, A.hstride, A.stages);
  const int STAGES = A.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S.bars);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* rt_full = empty + MAX_STAGES;
  uint64_t* rt_free = rt_full + 1;
  uint64_t* plan_ready = rt_free + 1;
  uint64_t* hready = plan_ready + 1;
  uint64_t* prod_done = hready + 1;
  __shared__ int s_abort;
  const int r_lo = int(int64_t(E + 1) * cta / G), r_hi = int(int64_t(E + 1) * (cta + 1) / G);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GW);  // a stage is a group's: each of its warps arrives once done with it
    }
    mbar_init(rt_full, 1);
    mbar_init(rt_free, 1);
    mbar_init(plan_ready, 1);
    mbar_init(hready, 1);
    mbar_init(prod_done, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  // the codebooks of every kind a layer may have, expanded to four values of T an entry (Q2_0 needs none)
  build_grid_tabs<T>(reinterpret_cast<uint2*>(smem + S.tabs), tid, THREADS);
  __syncthreads();
  if (warp == CW) {
    if (lane == 0) producer<T>(A, smem, S, r_lo, r_hi);
    return;
  }

  // ---- consumers
  const uint2* tabs = reinterpret_cast<const uint2*>(smem + S.tabs);
  T* xs = reinterpret_cast<T*>(smem + S.x);
  const uint8_t* rt = smem + S.router;
  dl::Plan* plan = reinterpret_cast<dl::Plan*>(smem + S.plan);
  float* s_wts = reinterpret_cast<float*>(smem + S.routes);
  float* s_gsh = s_wts + MAXT * TOPK_MAX_K;
  float* red = reinterpret_cast<float*>(smem + S.red);
  dl::TailSmem& TS = *reinterpret_cast<dl::TailSmem*>(smem + S.red);
  uint8_t* stage0 = smem + S.stages;
  const int grp = warp / GW, gw = warp % GW;
  T* h = static_cast<T*>(A.h);
  T* Y = static_cast<T*>(A.Y);
  unsigned nbar = 0;
  uint32_t it = 0;
  auto barrier = [&]() -> bool { return grid_barrier(A.bar, ++nbar * unsigned(G), A.err, &s_abort); };
  auto sync = [] { named_sync(CONS_BAR, CT); };

  for (int l = 0; l < A.L; ++l) {
    const LayerW& w = A.w[l];
    const int rb_gu = w.rb_gu, rb_d = w.rb_d, rb_sd = w.rb_sd;
    // ---- the window: the chain's input, or the previous layer's combined outputs
    if (tid == 0) CK_TRACE(l, 0);
    const bool fresh = l == 0 || (A.refeed > 0 && l % A.refeed == 0);
    const bool pairs = x_pairs(w.kgu);
    stage_x<T>(static_cast<const T*>(fresh ? A.x : A.Xn), T_, H, xs, H + 32, tid, CT, pairs);
    sync();
    if (tid == 0) CK_TRACE(l, 1);
    // ---- R: this block's router rows
    if (!mbar_wait(rt_full, l & 1, A.err)) s_abort = 1;
    // warp w takes router row w % nrows for one group of the window's tokens (groups of tpg), so that every warp
    // has a share when the block holds fewer rows than warps
    const int nrows = r_hi - r_lo, ngroups = nrows > 0 ? max(1, CW / nrows) : 1;
    const int tpg = (T_ + ngroups - 1) / ngroups, rl = nrows > 0 ? warp % nrows : 0, tg = nrows > 0 ? warp / nrows : 0;
    if (nrows > 0 && tg < ngroups && s_abort == 0) {
      const int row = r_lo + rl;
      const uint4* wv = reinterpret_cast<const uint4*>(rt + rl * H * 2) + lane;
      for (int t = tg * tpg; t < min(T_, (tg + 1) * tpg); ++t) {
        const uint4* xr = reinterpret_cast<const uint4*>(xs + t * (H + 32)) + lane;
        float acc = 0.f;
        for (int c = 0; c < H / 256; ++c) {
          const uint4 o = xr[32 * c];  // eight activations, stored as (0,4) (1,5) (2,6) (3,7) for a Q2_0 layer
          const uint4 v = pairs ? make_uint4(__byte_perm(o.x, o.y, 0x5410), __byte_perm(o.z, o.w, 0x5410),
                                             __byte_perm(o.x, o.y, 0x7632), __byte_perm(o.z, o.w, 0x7632))
                                : o;
          acc += dl::dot8_half<T>(wv[32 * c], v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
          if (row < E) A.logits[int64_t(t) * E + row] = acc;
          else A.gsh[t] = acc;
        }
      }
    }
    sync();
    if (tid == 0) {
      mbar_arrive(rt_free);
      CK_TRACE(l, 2);
    }
    if (!barrier()) return;  // A
    if (tid == 0) CK_TRACE(l, 3);
    // ---- P: the window's routes and plan, in every block
    const int units = dl::route_tail<MT>(A.logits, T_, E, K, 0, E, TS, tid, sync);
    for (int u = tid; u < units; u += CT) {
      dl::Unit v;
      v.expert = u == 0 ? -1 : TS.s_expert[u];
      v.tokmask = u == 0 ? (A.Is > 0 ? (1u << T_) - 1u : 0u) : TS.s_mask[u];
      v.kpack = u == 0 ? 0u : TS.s_kpack[u];
      v.pad = 0;
      plan->unit[u] = v;
    }
    for (int p = tid; p < T_ * K; p += CT) {
      s_wts[p] = TS.s_w[p];
      if (cta == 0) {
        A.idx[(int64_t(l) * T_) * K + p] = TS.s_idx[p];
        A.wts[(int64_t(l) * T_) * K + p] = TS.s_w[p];
      }
    }
    for (int t = tid; t < T_; t += CT) s_gsh[t] = A.Is > 0 ? __ldcg(A.gsh + t) : -INFINITY;
    if (tid == 0) {
      plan->units = units;
      if (l > 0 && !mbar_wait(prod_done, (l - 1) & 1, A.err)) s_abort = 1;
    }
    sync();
    if (s_abort) return;
    if (tid == 0) {
      mbar_arrive(plan_ready);
      CK_TRACE(l, 4);
    }
    const Items I_ = items_of(units, A.I, A.Is, H, cta, G);
    const uint32_t it_layer = it;
    // ---- G: gate/up items; item `it` goes to the group of its stage's parity
    for (int j = I_.g0; j < I_.g1; ++j, ++it) {
      const int s = int(it % STAGES);
      if ((s & 1) != grp) continue;
      int u, r0;
      I_.unit_row_gu(j, u, r0);
      const dl::Unit un = plan->unit[u];
      const int rb = rb_gu;  // the shared expert's gate / up rows are of the routed experts' kind
      const uint8_t* wg = stage0 + s * S.stage;
      const uint8_t* wu = wg + align16(int(RG * rb));
      float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
      const bool got = mbar_wait_sleep(&full[s], (it / STAGES) & 1, A.err, WAIT_LIMIT, 20000);
      if (gw == 0 && lane == 0) CK_ITRACE(l, it - it_layer, 1);
      if (got) {
        int n0, n1;
        gu_runs(H, gw, n0, n1);
        const int g = lane >> 2;
        const T* xg = g < T_ ? xs + g * (H + 32) : nullptr;
        by_kind(w.kgu, [&]<int KIND>() {
          frag_runs2<KIND, T>(wg + g * rb, wg + (g + 8) * rb, wu + g * rb, wu + (g + 8) * rb, xg, n0, n1, lane,
                              grid_tab<KIND>(tabs), accg, accu);
        });
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      float* rg = red + grp * (GW * 32 * 8);
      rg[((0 + 0) * GW + gw) * 32 + lane] = accg[0];
      rg[((0 + 1) * GW + gw) * 32 + lane] = accg[1];
      rg[((0 + 2) * GW + gw) * 32 + lane] = accg[2];
      rg[((0 + 3) * GW + gw) * 32 + lane] = accg[3];
      rg[((4 + 0) * GW + gw) * 32 + lane] = accu[0];
      rg[((4 + 1) * GW + gw) * 32 + lane] = accu[1];
      rg[((4 + 2) * GW + gw) * 32 + lane] = accu[2];
      rg[((4 + 3) * GW + gw) * 32 + lane] = accu[3];
      named_sync(2 + grp, GW * 32);
      const int gt = gw * 32 + lane;
      if (gt < 128 && got) {
        const int Lq = gt & 31, q = gt >> 5;
        float sg = 0.f, su = 0.f;
#pragma unroll
        for (int v = 0; v < GW; ++v) {
          sg += rg[(q * GW + v) * 32 + Lq];
          su += rg[((4 + q) * GW + v) * 32 + Lq];
        }
        const int m = (q < 2 ? 0 : 8) + (Lq >> 2), tok = 2 * (Lq & 3) + (q & 1);
        if (tok < T_ && ((un.tokmask >> tok) & 1u)) {
          // h in the order its consumer (the down product's decoder) wants
          h[(int64_t(u) * T_ + tok) * A.hstride + x_col(r0 + m, x_pairs(w.kd))] = from_f32<T>(swiglu_mlx<T>(sg, su));
        }
      }
      if (!got) s_abort = 1;
      named_sync(2 + grp, GW * 32);
      if (gw == 0 && lane == 0) CK_ITRACE(l, it - it_layer, 2);
    }
    if (tid == 0) CK_TRACE(l, 5);
    if (!barrier()) return;  // B: every unit's h
    if (tid == 0) {
      mbar_arrive(hready);
      CK_TRACE(l, 6);
    }
    // ---- D: down items
    for (int j = I_.d0; j < I_.d1; ++j, ++it) {
      const int s = int(it % STAGES);
      if ((s & 1) != grp) continue;
      int u, c0;
      I_.unit_row_dn(j, A.Is > 0, u, c0);
      const dl::Unit un = plan->unit[u];
      const bool sh = u == 0;
      const int rb = sh ? rb_sd : rb_d;
      const uint8_t* st = stage0 + s * S.stage;
      const T* hs = reinterpret_cast<const T*>(st + S.hoff);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const bool got = mbar_wait_sleep(&full[s], (it / STAGES) & 1, A.err, WAIT_LIMIT, 20000);
      if (gw == 0 && lane == 0) CK_ITRACE(l, it - it_layer, 1);
      if (got) {
        const int g = lane >> 2;
        const bool mine = g < T_ && ((un.tokmask >> g) & 1u);
        const uint8_t* st0 = st + gw * 16 * rb;
        by_kind(w.kd, [&]<int KIND>() {
          frag_runs<KIND, T>(st0 + g * rb, st0 + (g + 8) * rb, mine ? hs + g * A.hstride : nullptr, 0,
                             (sh ? A.Is : A.I) / 32, lane, grid_tab<KIND>(tabs), acc);
        });
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (!got) {
        s_abort = 1;
        continue;
      }
      const int g = lane >> 2, t = lane & 3;
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // C fragment: rows g, g + 8; tokens 2t, 2t + 1
        const int m = (q < 2 ? 0 : 8) + g, tok = 2 * t + (q & 1);
        if (tok < T_ && ((un.tokmask >> tok) & 1u)) {
          const int k = sh ? K : int((un.kpack >> (4 * tok)) & 15u);
          Y[(int64_t(tok) * (K + 1) + k) * H + c0 + gw * 16 + m] = from_f32<T>(acc[q]);
        }
      }
      if (gw == 0 && lane == 0) CK_ITRACE(l, it - it_layer, 2);
    }
    const bool last = l == A.L - 1;
    const bool next_fresh = !last && A.refeed > 0 && (l + 1) % A.refeed == 0;
    if (tid == 0) CK_TRACE(l, 7);
    if (next_fresh) continue;  // the next layer takes the chain's input again: this layer's outputs are not needed
    if (!barrier()) return;  // C: every pair's output
    if (tid == 0) CK_TRACE(l, 8);
    // ---- C: this block's slice of the window (moe_combine, fused.py:448-462), an output a thread
    const int n_out = T_ * H;
    const int q0 = int(int64_t(n_out) * cta / G), q1 = int(int64_t(n_out) * (cta + 1) / G);
    T* dst = static_cast<T*>(last ? A.out : A.Xn);
    for (int q = q0 + tid; q < q1; q += CT) {
      const int tok = q / H, c = q % H;
      float yk[TOPK_MAX_K];
      const T* yt = Y + int64_t(tok) * (K + 1) * H + c;
#pragma unroll
      for (int k = 0; k < TOPK_MAX_K; ++k)
        if (k < K) yk[k] = to_f32(__ldcg(yt + int64_t(k) * H));
      const float sv = A.Is > 0 ? to_f32(__ldcg(yt + int64_t(K) * H)) : 0.f;
      const float gv = A.Is > 0 ? round_to<T>(s_gsh[tok]) : -INFINITY;
      dst[q] = from_f32<T>(combine_one<T>(yk, s_wts + tok * K, K, gv, sv));
    }
    if (tid == 0) CK_TRACE(l, 9);
    if (last) break;
    if (!barrier()) return;  // D: the next layer's window
    if (tid == 0) CK_TRACE(l, 10);
  }
  // every block past the launch's last barrier: the last one resets the count for the next launch
  sync();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(A.bar + 1, 1u) == unsigned(G) - 1) {
      A.bar[0] = 0;
      A.bar[1] = 0;
      __threadfence();
    }
  }
}

}  // namespace ck

// ---------------------------------------------------------------------------------------------------- host

struct ChainWs {
  size_t err, bar, logits, gsh, idx, wts, h, Y, Xn, total;
};

static ChainWs chain_ws(const sc_moe_layer* L, int n_layers, int tokens) {
  const size_t T = size_t(tokens), K = size_t(L->top_k), E = size_t(L->experts), H = size_t(L->hidden);
  ChainWs m{};
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o += (bytes + 255) & ~size_t(255); return at; };
  m.err = take(16);
  m.bar = take(16);
  m.logits = take(T * E * 4);
  m.gsh = take(T * 4);
  m.idx = take(size_t(n_layers) * T * K * 4);
  m.wts = take(size_t(n_layers) * T * K * 4);
  m.h = take(size_t(tokens * L->top_k + 1) * T * size_t(v2_hstride(L)) * 2);
  m.Y = take(T * (K + 1) * H * 2);
  m.Xn = take(T * H * 2);
  m.total = o;
  return m;
}

// The layers the chain kernel takes: those of the three-kernel block, one shape for all, hidden by 128.
static int chain_check(const sc_moe_layer* layers, int n, int tokens) {
  if (!layers || n < 1) return SC_ERR_ARG;
  if (n > ck::MAXL) return SC_ERR_SHAPE;
  const sc_moe_layer& a = layers[0];
  for (int l = 0; l < n; ++l) {
    const sc_moe_layer& b = layers[l];
    if (!b.gate || !b.up || !b.down || !b.router) return SC_ERR_ARG;
    if (b.shared_inter && (!b.sgate || !b.sup || !b.sdown || !b.shared_gate)) return SC_ERR_ARG;
    if (b.hidden != a.hidden || b.inter != a.inter || b.experts != a.experts || b.top_k != a.top_k ||
        b.shared_inter != a.shared_inter || b.dtype != a.dtype)
      return SC_ERR_SHAPE;
    if (!v2_takes(&b, tokens)) return SC_ERR_UNSUPPORTED;
    if (b.hidden % ck::DN_ROWS) return SC_ERR_UNSUPPORTED;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(b.gate) || !al(b.up) || !al(b.down) || !al(b.router)) return SC_ERR_ALIGN;
    if (b.shared_inter && (!al(b.sgate) || !al(b.sup) || !al(b.sdown) || !al(b.shared_gate))) return SC_ERR_ALIGN;
  }
  return SC_OK;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return n;
}

}  // namespace sc

using namespace sc;

#ifdef SC_TRACE
extern "C" SC_API int sc_chain_trace_read(void* host) {
  return cudaMemcpyFromSymbol(host, ck::g_ctrace, sizeof(ck::g_ctrace)) == cudaSuccess ? 0 : -1;
}
extern "C" SC_API int sc_chain_itrace_read(void* host) {
  return cudaMemcpyFromSymbol(host, ck::g_itrace, sizeof(ck::g_itrace)) == cudaSuccess ? 0 : -1;
}
#endif

extern "C" size_t sc_moe_decode_chain_workspace(const sc_moe_layer* layers, int n_layers, int tokens) {
  if (chain_check(layers, n_layers, tokens) != SC_OK) return 0;
  return chain_ws(layers, n_layers, tokens).total;
}

extern "C" int sc_moe_decode_chain_routes(const sc_moe_layer* layers, int n_layers, int tokens, size_t* idx_offset,
                                          size_t* weight_offset) {
  if (int rc = chain_check(layers, n_layers, tokens)) return rc;
  const ChainWs m = chain_ws(layers, n_layers, tokens);
  if (idx_offset) *idx_offset = m.idx;
  if (weight_offset) *weight_offset = m.wts;
  return SC_OK;
}

extern "C" int sc_moe_decode_chain(const sc_moe_layer* layers, int n_layers, const void* x, int tokens, int refeed,
                                   void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = chain_check(layers, n_layers, tokens)) return rc;
  if (!x || !out || refeed < 0) return SC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) return SC_ERR_ALIGN;
  const ChainWs m = chain_ws(layers, n_layers, tokens);
  if (!workspace || workspace_bytes < m.total) return SC_ERR_WORKSPACE;
  const int G = sm_count();
  if (G <= 0) return SC_ERR_CUDA;
  const sc_moe_layer& a = layers[0];
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  ck::Args A{};  // copied into the launch's parameters
  A.L = n_layers;
  A.T = tokens;
  A.H = a.hidden;
  A.I = a.inter;
  A.Is = a.shared_inter;
  A.E = a.experts;
  A.K = a.top_k;
  A.refeed = refeed;
  A.hstride = v2_hstride(&a);
  A.rt_rows = int(ceil_div(a.experts + 1, G));
  int wmax = 0;
  for (int l = 0; l < n_layers; ++l) {
    const sc_moe_layer& b = layers[l];
    ck::LayerW& w = A.w[l];
    w.gate = static_cast<const uint8_t*>(b.gate);
    w.up = static_cast<const uint8_t*>(b.up);
    w.down = static_cast<const uint8_t*>(b.down);
    w.sgate = static_cast<const uint8_t*>(b.sgate);
    w.sup = static_cast<const uint8_t*>(b.sup);
    w.sdown = static_cast<const uint8_t*>(b.sdown);
    w.router = static_cast<const __half*>(b.router);
    w.shared_gate = static_cast<const __half*>(b.shared_gate);
    w.kgu = b.kind_gate;
    w.kd = b.kind_down;
    w.rb_gu = int(row_bytes(b.kind_gate, b.hidden));
    w.rb_d = int(row_bytes(b.kind_down, b.inter));
    w.rb_sd = b.shared_inter ? int(row_bytes(b.kind_sdown, b.shared_inter)) : 0;
    const int gu = 2 * align16(int(ck::RG * row_bytes(b.kind_gate, b.hidden)));
    const int dn = int(ck::DN_ROWS * row_bytes(b.kind_down, b.inter));
    const int dns = b.shared_inter ? int(ck::DN_ROWS * row_bytes(b.kind_sdown, b.shared_inter)) : 0;
    wmax = std::max({wmax, gu, dn, dns});
  }
  A.wmax = wmax;
  A.x = x;
  A.out = out;
  A.err = reinterpret_cast<int*>(ws + m.err);
  A.bar = reinterpret_cast<unsigned*>(ws + m.bar);
  A.logits = reinterpret_cast<float*>(ws + m.logits);
  A.gsh = reinterpret_cast<float*>(ws + m.gsh);
  A.idx = reinterpret_cast<uint32_t*>(ws + m.idx);
  A.wts = reinterpret_cast<float*>(ws + m.wts);
  A.h = ws + m.h;
  A.Y = ws + m.Y;
  A.Xn = ws + m.Xn;
  // as many stages as fit (an even number, 4 .. 8): small windows then fetch every item of a layer at once
  const ck::Smem S0 = ck::smem_of(tokens, a.hidden, A.rt_rows, wmax, A.hstride, 0);
  A.stages = std::min(ck::MAX_STAGES, ((227 * 1024 - 256 - S0.total) / S0.stage) & ~1);
  if (A.stages < 4) return SC_ERR_SHAPE;
  const ck::Smem S = ck::smem_of(tokens, a.hidden, A.rt_rows, wmax, A.hstride, A.stages);
  // one block an SM: more than half an SM's shared memory keeps a second block off
  const int smem = std::max(S.total, 116 * 1024);
  if (smem > 227 * 1024) return SC_ERR_SHAPE;
  int rc = SC_ERR_UNSUPPORTED;
  auto go = [&]<typename T>() {
    auto kern = tokens == 1 ? ck::chain_kernel<T, 1>
                : tokens == 2 ? ck::chain_kernel<T, 2>
                : tokens <= 4 ? ck::chain_kernel<T, 4>
                              : ck::chain_kernel<T, dl::MAXT>;
    if ((rc = raise_smem(reinterpret_cast<const void*>(kern), smem, "decode chain smem attribute"))) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(ck::THREADS);
    cfg.dynamicSmemBytes = size_t(smem);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every block resident at once: the grid barriers need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaError_t e = cudaLaunchKernelEx(&cfg, kern, A)) rc = cuda_failed(e, "decode chain launch");
    else rc = SC_OK;
  };
  if (a.dtype == SC_BF16) go.template operator()<__nv_bfloat16>();
  else go.template operator()<__half>();
  return rc;
}
