// The reference's unfused expert products for a batch of pairs (BlockSwitchLinear.__call__, strata_mlx/blocks.py:
// 407-440; its gate/up fused form :808-818; matvec_glu :222-259) when the activations are 16-bit floats and the
// block type has a fragment decoder (Q2_0, IQ3_S, IQ3_XXS): the pairs are grouped by expert, each expert's blocks
// are read once per group of up to eight pairs, and decoded straight into tensor-core fragments (frag_decode.cuh)
// that multiply all of the group's activations at once. The exact float32 kernel (matvec_impl.cuh) stays for
// float32 activations, for the other block types and for small calls.
//
// One persistent block per SM, seventeen warps: sixteen consumer warps in two groups of eight and a producer warp.
//   plan   every block works out the same plan from the pairs' experts (a bitmap; prefix sums over the block):
//          the distinct experts (units, ascending), each unit's pairs (slots, in pair order), and groups of up to
//          eight slots
//   items  (group, 16 weight rows) -- or, for a product of fewer than 1,024 columns, (group, 128 rows) --
//          group-major; block b of G takes [n b / G, n (b + 1) / G)
//   ring   the producer streams each item's rows (gate and up rows for the gate/up form) into a ring of
//          shared-memory stages with 1-D bulk copies; items alternate between the two consumer groups
//   items  a group's eight warps split the columns (runs by fours), stage the group's activations when the item's
//          group of pairs changes, and sum their parts through shared memory in warp order -> out (pairs, rows);
//          a 128-row item gives each warp 16 rows over every column instead (no sums to meet)
//
// Results: float32 sums of exact products (the weights enter the tensor core as small integers of the
// activations' type, the run scales applied to the run sums), rounded once to the activations' type; the gate/up
// form applies mlx-lm's swiglu to the rounded gate and up sums, so it gives the bits of the two products apart.
// Bits do not depend on which pairs share a group (each pair is its own column of the product).
#include <algorithm>

#include "matvec.cuh"
#include "frag_decode.cuh"

namespace sc {
namespace gm {

constexpr int GW = 8;                  // warps of a consumer group
constexpr int GROUPS = 2;
constexpr int CW = GW * GROUPS;
constexpr int THREADS = (CW + 1) * 32;  // and the producer warp
constexpr int RG = 16;                 // weight rows an item
constexpr int SLOTS = 8;               // pairs a group of pairs holds: the tensor core's n
constexpr int MAX_STAGES = 8;
constexpr int MAX_PAIRS = 1024;        // pairs a launch takes (the host splits larger calls)
constexpr int FROM = 32;               // pairs from which a call takes this path

struct Args {
  const uint8_t* w;   // the stack (gate/up form: the gate stack)
  const uint8_t* w2;  // gate/up form: the up stack
  const uint32_t* idx;
  const void* x;      // (x rows, cols); GLU_IN: the gate activations (pairs, cols)
  const void* x2;     // GLU_IN: the up activations (pairs, cols)
  void* out;          // (pairs, rows)
  int* err;
  int64_t rb;         // bytes of a weight row
  int experts, rows, cols, pairs, share, stages, stage_bytes;
  int item_rows;      // RG (a group's warps split the columns) or GW * RG (a warp a tile of 16 rows, every column)
};

struct Layout {
  int bars, tabs, bitmap, wpre, ucnt, uoff, ufill, uexp, goff, gdesc, slots, sidx, xs, xs_group, red, stages, total;
};

// The codebook an IQ3 kind reads in REP copies (Q2_0 has none)
constexpr int REP = 16;
__host__ __device__ constexpr int tab_bytes(int kind) {
  return kind == SC_IQ3_S ? 512 * REP * 8 : kind == SC_IQ3_XXS ? 256 * REP * 8 : 0;
}
// Whether a group's activations are staged in shared memory: Q2_0 wants them reordered, the down product of the
// swiglu form computes them; otherwise the warps read them from global memory (L1) in place.
__host__ __device__ constexpr bool stages_x(int kind, int mode) { return kind == SC_Q2_0 || mode == MV_GLU_IN; }

__host__ __device__ inline Layout layout_of(int kind, int mode, int experts, int pairs, int cols, int stage_bytes,
                                            int stages) {
  Layout L;
  int o = 0;
  const int words = (experts + 31) / 32;
  const int umax = experts < pairs ? experts : pairs;
  L.bars = o; o += align16(2 * MAX_STAGES * 8);
  L.tabs = o; o += tab_bytes(kind);
  L.bitmap = o; o += align16(4 * words);
  L.wpre = o; o += align16(4 * words);
  L.ucnt = o; o += align16(4 * umax);
  L.uoff = o; o += align16(4 * umax);
  L.ufill = o; o += align16(4 * umax);
  L.uexp = o; o += align16(4 * umax);
  L.goff = o; o += align16(4 * umax);
  L.gdesc = o; o += align16(8 * pairs);  // a group: (first slot << 4 | pairs), expert
  L.slots = o; o += align16(4 * pairs);  // a slot: (x row << 16) | pair
  L.sidx = o; o += align16(4 * pairs);   // the pairs' experts
  L.xs_group = stages_x(kind, mode) ? align16(SLOTS * (cols + 32) * 2) : 0;
  L.xs = o; o += GROUPS * L.xs_group;
  L.red = o; o += GROUPS * GW * 32 * 8 * 4;
  L.stages = align16(o); o = L.stages + stages * stage_bytes;
  L.total = o;
  return L;
}

__device__ __forceinline__ void named_sync_group(int grp) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(GW * 32) : "memory");
}

// Exclusive prefix sums of v(i), i < n, into out[i] (out may be nullptr); returns the total. Every thread of the
// block calls it; wsum holds 72 ints of shared memory.
template <typename F>
__device__ int block_scan(int n, F v, int* out, int* wsum) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int per = (n + int(blockDim.x) - 1) / int(blockDim.x);
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  int mine = 0;
  for (int i = i0; i < i1; ++i) mine += v(i);
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < nw ? wsum[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    wsum[32 + lane] = wi - w;
    if (lane == 31) wsum[64] = wi;
  }
  __syncthreads();
  int run = wsum[32 + warp] + incl - mine;
  if (out)
    for (int i = i0; i < i1; ++i) {
      out[i] = run;
      run += v(i);
    }
  const int total = wsum[64];
  __syncthreads();
  return total;
}

// eight activations (one 16-byte piece) into the order a kind's decoder wants them
__device__ __forceinline__ uint4 in_order(uint4 v, bool pairs) {
  if (!pairs) return v;
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);  // (0, 4)
  o.y = __byte_perm(v.x, v.z, 0x7632);  // (1, 5)
  o.z = __byte_perm(v.y, v.w, 0x5410);  // (2, 6)
  o.w = __byte_perm(v.y, v.w, 0x7632);  // (3, 7)
  return o;
}

template <int KIND, typename T, int MODE>
__global__ void __launch_bounds__(THREADS, 1) gm_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int wsum[72];
  __shared__ int s_units, s_groups, s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S_ = A.stages;
  const Layout L = layout_of(KIND, MODE, A.experts, A.pairs, A.cols, A.stage_bytes, S_);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + MAX_STAGES;
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  int* wpre = reinterpret_cast<int*>(smem + L.wpre);
  int* ucnt = reinterpret_cast<int*>(smem + L.ucnt);
  int* uoff = reinterpret_cast<int*>(smem + L.uoff);
  int* ufill = reinterpret_cast<int*>(smem + L.ufill);
  int* uexp = reinterpret_cast<int*>(smem + L.uexp);
  int* goff = reinterpret_cast<int*>(smem + L.goff);
  int2* gdesc = reinterpret_cast<int2*>(smem + L.gdesc);
  uint32_t* slots = reinterpret_cast<uint32_t*>(smem + L.slots);
  uint32_t* sidx = reinterpret_cast<uint32_t*>(smem + L.sidx);
  uint8_t* stage0 = smem + L.stages;
  const int words = (A.experts + 31) / 32;
  const int umax = min(A.experts, A.pairs);

  if (tid == 0) {
    for (int s = 0; s < S_; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GW);  // a stage is a consumer group's: each of its warps arrives once done with it
    }
    fence_mbar_init();
    s_abort = 0;
  }
  if constexpr (KIND != SC_Q2_0) build_grid_tab_rep<T, KIND, REP>(reinterpret_cast<uint2*>(smem + L.tabs), tid, THREADS);

  // ---- the plan
  for (int i = tid; i < words; i += THREADS) bitmap[i] = 0;
  for (int u = tid; u < umax; u += THREADS) ucnt[u] = ufill[u] = 0;
  __syncthreads();
  for (int p = tid; p < A.pairs; p += THREADS) {
    const uint32_t e = __ldg(A.idx + p);
    sidx[p] = e;
    if (e < uint32_t(A.experts)) atomicOr(&bitmap[e >> 5], 1u << (e & 31));
    else record_error(A.err, SC_ERR_INDEX);
  }
  __syncthreads();
  const int units = block_scan(words, [&](int i) { return __popc(bitmap[i]); }, wpre, wsum);
  auto unit_of = [&](uint32_t e) { return wpre[e >> 5] + __popc(bitmap[e >> 5] & ((1u << (e & 31)) - 1u)); };
  for (int p = tid; p < A.pairs; p += THREADS) {
    const uint32_t e = sidx[p];
    if (e < uint32_t(A.experts)) {
      const int u = unit_of(e);
      atomicAdd(&ucnt[u], 1);
      uexp[u] = int(e);
    }
  }
  __syncthreads();
  block_scan(units, [&](int u) { return ucnt[u]; }, uoff, wsum);
  const int groups = block_scan(units, [&](int u) { return (ucnt[u] + SLOTS - 1) / SLOTS; }, goff, wsum);
  if (warp == 0) {
    // a unit's slots in the order of their pairs, the same in every block: a unit of more than eight pairs is
    // several groups, and every block must put the same pairs in each (one warp, 32 pairs a step, equal experts
    // found with a match and counted in lane order)
    for (int base = 0; base < A.pairs; base += 32) {
      const int p = base + lane;
      const uint32_t e = p < A.pairs ? sidx[p] : 0xffffffffu;
      const bool ok = e < uint32_t(A.experts);
      const uint32_t peers = __match_any_sync(0xffffffffu, ok ? e : 0xffffffffu);
      const int leader = __ffs(peers) - 1;
      const int u = ok ? unit_of(e) : 0;
      int before = 0;
      if (ok && lane == leader) {
        before = ufill[u];
        ufill[u] = before + __popc(peers);
      }
      before = __shfl_sync(0xffffffffu, before, leader);
      if (ok) {
        const int at = uoff[u] + before + __popc(peers & ((1u << lane) - 1u));
        const int xrow = MODE == MV_GLU_IN ? p : p / A.share;
        slots[at] = (uint32_t(xrow) << 16) | uint32_t(p);
      }
      __syncwarp();
    }
  }
  for (int u = tid; u < units; u += THREADS) {
    const int c = ucnt[u];
    for (int k = 0; k * SLOTS < c; ++k)
      gdesc[goff[u] + k] = make_int2(((uoff[u] + k * SLOTS) << 4) | min(SLOTS, c - k * SLOTS), uexp[u]);
  }
  if (tid == 0) {
    s_units = units;
    s_groups = groups;
  }
  __syncthreads();

  const int IR = A.item_rows;
  const bool by_rows = IR != RG;
  const int nrb = A.rows / IR;
  const int64_t items = int64_t(s_groups) * nrb;
  const int64_t c0 = items * blockIdx.x / gridDim.x, c1 = items * (blockIdx.x + 1) / gridDim.x;
  const int parts = MODE == MV_GATEUP ? 2 : 1;
  const uint32_t bytes = uint32_t(IR * A.rb);
  const int rs = int(A.rb);
  const int up_at = align16(int(bytes));

  if (warp == CW) {
    // ---- producer: one lane issues the bulk copies; every copy it issued has landed before it leaves
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t j = c0; j < c1; ++j, ++it) {
        const int s = int(it % S_);
        if (it >= uint32_t(S_) && !mbar_wait(&empty[s], ((it / S_) - 1) & 1, A.err)) break;
        const int2 gd = gdesc[j / nrb];
        const int64_t row0 = int64_t(gd.y) * A.rows + (j % nrb) * IR;
        uint8_t* dst = stage0 + s * A.stage_bytes;
        mbar_arrive_expect_tx(&full[s], bytes * parts);
        bulk_load(dst, A.w + row0 * A.rb, bytes, &full[s]);
        if constexpr (MODE == MV_GATEUP) bulk_load(dst + up_at, A.w2 + row0 * A.rb, bytes, &full[s]);
      }
      for (uint32_t i = it > uint32_t(S_) ? it - S_ : 0; i < it; ++i) mbar_wait(&full[i % S_], (i / S_) & 1, A.err);
    }
    return;
  }

  // ---- consumers
  const int grp = warp / GW, gw = warp % GW, g = lane >> 2;
  const int cols = A.cols, xstride = cols + 32;
  T* xs = reinterpret_cast<T*>(smem + L.xs + grp * L.xs_group);
  float* rg = reinterpret_cast<float*>(smem + L.red) + grp * (GW * 32 * 8);
  const uint2* tab = rep_tab<REP>(reinterpret_cast<const uint2*>(smem + L.tabs), lane);
  constexpr bool STAGE = stages_x(KIND, MODE);
  const bool pairs = x_pairs(KIND);
  const int q4 = cols / 128, n0 = 4 * (gw * q4 / GW), n1 = 4 * ((gw + 1) * q4 / GW);  // runs, by fours
  const int gt = gw * 32 + lane;
  int cur = -1;
  uint32_t it = 0;
  for (int64_t j = c0; j < c1; ++j, ++it) {
    const int s = int(it % S_);
    if ((s & 1) != grp) continue;
    const int gi = int(j / nrb), r0 = int(j % nrb) * IR;
    const int2 gd = gdesc[gi];
    const int cnt = gd.x & 15, first = gd.x >> 4;
    if (STAGE && gi != cur) {  // the group's activations (by columns, the previous item ended with the group's barrier)
      if (by_rows) named_sync_group(grp);
      const int pieces = cols / 8;
      for (int i = gt; i < cnt * pieces; i += GW * 32) {
        const int k = i / pieces, c = i % pieces;
        const int xrow = int(slots[first + k] >> 16);
        uint4 v;
        if constexpr (MODE == MV_GLU_IN) {
          const uint4 gv = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(A.x) + int64_t(xrow) * cols) + c);
          const uint4 uv = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(A.x2) + int64_t(xrow) * cols) + c);
          const T* ge = reinterpret_cast<const T*>(&gv);
          const T* ue = reinterpret_cast<const T*>(&uv);
          T* ve = reinterpret_cast<T*>(&v);
#pragma unroll
          for (int e = 0; e < 8; ++e) ve[e] = from_f32<T>(swiglu_mlx<T>(to_f32(ge[e]), to_f32(ue[e])));
        } else {
          v = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(A.x) + int64_t(xrow) * cols) + c);
        }
        *reinterpret_cast<uint4*>(xs + k * xstride + 8 * c) = in_order(v, pairs);
      }
      named_sync_group(grp);
      cur = gi;
    }
    const uint8_t* st = stage0 + s * A.stage_bytes;
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    const bool got = s_abort == 0 && mbar_wait(&full[s], (it / S_) & 1, A.err);
    if (by_rows) {
      // ---- a warp a tile of 16 rows, every column: the eight column slices' sums of the split by columns, in the
      // same order, so that both splits give the same bits (a call's form does not decide its bits)
      if (got) {
        const T* xg = g >= cnt ? nullptr
                      : STAGE ? xs + g * xstride
                              : static_cast<const T*>(A.x) + int64_t(slots[first + g] >> 16) * cols;
        const uint8_t* t0 = st + gw * RG * rs;
        const uint8_t* u0 = st + up_at + gw * RG * rs;
        for (int v = 0; v < GW; ++v) {
          const int m0 = 4 * (v * q4 / GW), m1 = 4 * ((v + 1) * q4 / GW);
          float pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
          if constexpr (MODE == MV_GATEUP)
            frag_runs2<KIND, T, REP>(t0 + g * rs, t0 + (g + 8) * rs, u0 + g * rs, u0 + (g + 8) * rs, xg, m0, m1, lane, tab,
                                pa, pb);
          else
            frag_runs<KIND, T, REP>(t0 + g * rs, t0 + (g + 8) * rs, xg, m0, m1, lane, tab, pa);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[q] += pa[q];
            if constexpr (MODE == MV_GATEUP) acc2[q] += pb[q];
          }
        }
      } else {
        s_abort = 1;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (got) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // C fragment: rows g, g + 8; pairs 2t, 2t + 1 of the group
          const int m = (q < 2 ? 0 : 8) + g, tok = 2 * (lane & 3) + (q & 1);
          if (tok < cnt) {
            const int p = int(slots[first + tok] & 0xffffu);
            const float y = MODE == MV_GATEUP ? swiglu_mlx<T>(acc[q], acc2[q]) : acc[q];
            static_cast<T*>(A.out)[int64_t(p) * A.rows + r0 + gw * RG + m] = from_f32<T>(y);
          }
        }
      }
      continue;
    }
    if (got) {
      const T* xg = g >= cnt ? nullptr
                    : STAGE ? xs + g * xstride
                            : static_cast<const T*>(A.x) + int64_t(slots[first + g] >> 16) * cols;
      if constexpr (MODE == MV_GATEUP)
        frag_runs2<KIND, T, REP>(st + g * rs, st + (g + 8) * rs, st + up_at + g * rs, st + up_at + (g + 8) * rs, xg, n0,
                            n1, lane, tab, acc, acc2);
      else
        frag_runs<KIND, T, REP>(st + g * rs, st + (g + 8) * rs, xg, n0, n1, lane, tab, acc);
    } else {
      s_abort = 1;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      rg[(q * GW + gw) * 32 + lane] = acc[q];
      if constexpr (MODE == MV_GATEUP) rg[((4 + q) * GW + gw) * 32 + lane] = acc2[q];
    }
    named_sync_group(grp);
    if (gt < 128 && s_abort == 0) {
      const int Lq = gt & 31, q = gt >> 5;
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int v = 0; v < GW; ++v) {  // the eight column slices' sums, in warp order
        sa += rg[(q * GW + v) * 32 + Lq];
        if constexpr (MODE == MV_GATEUP) sb += rg[((4 + q) * GW + v) * 32 + Lq];
      }
      const int m = (q < 2 ? 0 : 8) + (Lq >> 2), tok = 2 * (Lq & 3) + (q & 1);
      if (tok < cnt) {
        const int p = int(slots[first + tok] & 0xffffu);
        const float y = MODE == MV_GATEUP ? swiglu_mlx<T>(sa, sb) : sa;
        static_cast<T*>(A.out)[int64_t(p) * A.rows + r0 + m] = from_f32<T>(y);
      }
    }
    named_sync_group(grp);
  }
}

// ---- host side

template <int KIND, typename T, int MODE>
static int launch(Args a, int grid, cudaStream_t s) {
  const Layout L = layout_of(KIND, MODE, a.experts, a.pairs, a.cols, a.stage_bytes, a.stages);
  auto kern = gm_kernel<KIND, T, MODE>;
  if (int rc = raise_smem(reinterpret_cast<const void*>(kern), L.total, "grouped matvec smem attribute")) return rc;
  kern<<<grid, THREADS, L.total, s>>>(a);
  if (cudaError_t e = cudaGetLastError()) return cuda_failed(e, "grouped matvec launch");
  return SC_OK;
}

template <typename T, int MODE>
static int by_kind(int kind, const Args& a, int grid, cudaStream_t s) {
  if (kind == SC_Q2_0) return launch<SC_Q2_0, T, MODE>(a, grid, s);
  if (kind == SC_IQ3_S) return launch<SC_IQ3_S, T, MODE>(a, grid, s);
  return launch<SC_IQ3_XXS, T, MODE>(a, grid, s);
}

template <typename T>
static int by_mode(int kind, int mode, const Args& a, int grid, cudaStream_t s) {
  if (mode == MV_PLAIN) return by_kind<T, MV_PLAIN>(kind, a, grid, s);
  if (mode == MV_GATEUP) return by_kind<T, MV_GATEUP>(kind, a, grid, s);
  return by_kind<T, MV_GLU_IN>(kind, a, grid, s);
}

static int stages_for(int kind, int mode, int experts, int pairs, int cols, int stage_bytes, int least) {
  for (int st = MAX_STAGES; st >= least; st -= 2)
    if (layout_of(kind, mode, experts, pairs, cols, stage_bytes, st).total <= 225 * 1024) return st;  // + static
  return 0;
}

}  // namespace gm

int gm_matvec(int kind, int mode, int dtype, const void* w, const void* w2, int experts, int rows, int cols,
              const uint32_t* idx, int pairs, int share, int glu, const void* x, const void* x2, void* out, int* err,
              cudaStream_t s) {
  using namespace gm;
  if (kind != SC_Q2_0 && kind != SC_IQ3_S && kind != SC_IQ3_XXS) return GM_DECLINED;
  if (dtype != SC_F16 && dtype != SC_BF16) return GM_DECLINED;
  if (pairs < FROM || rows % RG || cols % 128 || share > MAX_PAIRS || (mode == MV_GLU_IN && glu)) return GM_DECLINED;
  const auto mis = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (mis(w) || (w2 && mis(w2)) || mis(x) || (x2 && mis(x2))) return GM_DECLINED;
  const int64_t rb = row_bytes(kind, cols);
  const int parts = mode == MV_GATEUP ? 2 : 1;
  const int chunk = MAX_PAIRS - MAX_PAIRS % share;
  const int most = std::min(pairs, chunk);
  // whether the path takes a call does not depend on which of the gate/up form and the plain product it is (the two
  // must agree bit for bit): where the gate/up form's smallest ring fits, the plain product's does; the swiglu
  // form, which stages its activations, decides for itself (it agrees with the plain product where both take it)
  const int dmode = mode == MV_GLU_IN ? MV_GLU_IN : MV_GATEUP;
  if (stages_for(kind, dmode, experts, most, cols, (dmode == MV_GATEUP ? 2 : 1) * align16(int(RG * rb)), 2) == 0)
    return GM_DECLINED;
  // narrow products (fewer runs of four than a group has warps) give each warp whole rows instead of columns,
  // where a ring of four such stages fits; the bits are the same either way
  int item_rows = RG;
  if (cols / 128 < GW && rows % (GW * RG) == 0 &&
      stages_for(kind, mode, experts, most, cols, parts * align16(int(GW * RG * rb)), 4) > 0)
    item_rows = GW * RG;
  const int stage_bytes = parts * align16(int(item_rows * rb));
  const int least = stages_for(kind, mode, experts, most, cols, stage_bytes, 4) > 0 ? 4 : 2;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  for (int p0 = 0; p0 < pairs; p0 += chunk) {
    const int n = std::min(chunk, pairs - p0);
    Args a{};
    a.w = static_cast<const uint8_t*>(w);
    a.w2 = static_cast<const uint8_t*>(w2);
    a.idx = idx + p0;
    a.x = static_cast<const uint8_t*>(x) + int64_t(mode == MV_GLU_IN ? p0 : p0 / share) * cols * 2;
    a.x2 = x2 ? static_cast<const uint8_t*>(x2) + int64_t(p0) * cols * 2 : nullptr;
    a.out = static_cast<uint8_t*>(out) + int64_t(p0) * rows * 2;
    a.err = err;
    a.rb = rb;
    a.experts = experts; a.rows = rows; a.cols = cols; a.pairs = n; a.share = share;
    a.stage_bytes = stage_bytes;
    a.item_rows = item_rows;
    a.stages = stages_for(kind, mode, experts, n, cols, stage_bytes, least);
    const int grid = int(std::min<int64_t>(sms, int64_t(n) * (rows / item_rows)));
    const int rc = dtype == SC_BF16 ? by_mode<__nv_bfloat16>(kind, mode, a, grid, s) : by_mode<__half>(kind, mode, a, grid, s);
    if (rc != SC_OK) return rc;
  }
  return SC_OK;
}

}  // namespace sc
