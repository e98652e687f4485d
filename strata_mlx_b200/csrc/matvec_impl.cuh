// The decode matvec kernel and its launcher, included by matvec_kind.cu, which the build compiles once per
// block type (-DMV_KIND=k) so that the variants compile in parallel.
#pragma once

#include <algorithm>
#include <numeric>

#include "matvec.cuh"

namespace sc {

template <int KIND, typename InT, int MODE, int SG>
__global__ void __launch_bounds__(MV_THREADS) mv_kernel(MvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int xrows = MODE == MV_PLAIN || MODE == MV_GATEUP ? (a.pairs + a.share - 1) / a.share : a.pairs;
  const int experts = a.bases ? a.pairs : a.experts;
  const MvLayout L = mv_layout<KIND>(a.bases ? 1 : experts, a.pairs, xrows, a.cols, a.stage_bytes, a.stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + MV_MAX_STAGES;
  int* sh_count = reinterpret_cast<int*>(empty + MV_MAX_STAGES);  // [0] = units
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  const uint8_t** ubase = reinterpret_cast<const uint8_t**>(smem + L.units);
  const uint8_t** ubase2 = ubase + a.pairs;
  int* uoff = reinterpret_cast<int*>(ubase2 + a.pairs);
  int* ucnt = uoff + a.pairs;
  uint32_t* slots = reinterpret_cast<uint32_t*>(smem + L.slots);
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  uint8_t* stage0 = smem + L.stages;

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MV_WARPS);
    }
    fence_mbar_init();
  }
  const Tabs tabs = load_tabs<KIND>(smem + L.tabs);

  // ---- the plan: units (distinct experts, ascending) and their slots (x row, out row)
  const int words = (experts + 31) / 32;
  if (a.bases) {
    for (int p = tid; p < a.pairs; p += blockDim.x) {
      ubase[p] = a.bases[p];
      uoff[p] = p;
      ucnt[p] = 1;
      slots[p] = (uint32_t(p / a.share) << 16) | uint32_t(p);
    }
    if (tid == 0) sh_count[0] = a.pairs;
  } else {
    for (int i = tid; i < words; i += blockDim.x) bitmap[i] = 0;
    for (int i = tid; i < a.pairs; i += blockDim.x) ucnt[i] = 0;
    __syncthreads();
    for (int p = tid; p < a.pairs; p += blockDim.x) {
      const uint32_t e = a.idx ? a.idx[p] : 0u;
      if (e < uint32_t(experts)) atomicOr(&bitmap[e >> 5], 1u << (e & 31));
      else record_error(a.err, SC_ERR_INDEX);
    }
    __syncthreads();
    // exclusive prefix of the bitmap's popcounts, by warp 0: lane l sums words [l*per, (l+1)*per)
    uint32_t* wpre = bitmap + words;  // exclusive prefix of the popcounts, per word
    if (warp == 0) {
      const int per = (words + 31) / 32;
      int mine = 0;
      for (int i = lane * per; i < min(words, (lane + 1) * per); ++i) mine += __popc(bitmap[i]);
      int incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      int run = incl - mine;
      for (int i = lane * per; i < min(words, (lane + 1) * per); ++i) {
        wpre[i] = run;
        run += __popc(bitmap[i]);
      }
      if (lane == 31) sh_count[0] = incl;
    }
    __syncthreads();
    for (int p = tid; p < a.pairs; p += blockDim.x) {
      const uint32_t e = a.idx ? a.idx[p] : 0u;
      if (e < uint32_t(experts)) {
        const int u = wpre[e >> 5] + __popc(bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
        ubase[u] = a.w + int64_t(e) * a.rows * a.rbytes;
        if (MODE == MV_GATEUP) ubase2[u] = a.w2 + int64_t(e) * a.rows * a.rbytes;
        atomicAdd(&ucnt[u], 1);
      }
    }
    __syncthreads();
    if (tid == 0) {  // offsets of the units' slot lists (units <= pairs <= MV_MAX_PAIRS)
      int run = 0;
      for (int u = 0; u < sh_count[0]; ++u) {
        uoff[u] = run;
        run += ucnt[u];
        ucnt[u] = 0;
      }
    }
    __syncthreads();
    for (int p = tid; p < a.pairs; p += blockDim.x) {
      const uint32_t e = a.idx ? a.idx[p] : 0u;
      if (e < uint32_t(experts)) {
        const int u = wpre[e >> 5] + __popc(bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
        const int at = uoff[u] + atomicAdd(&ucnt[u], 1);
        slots[at] = (uint32_t(p / a.share) << 16) | uint32_t(p);
      }
    }
  }
  // ---- activations as float32, in the bank-spread layout of xs_index
  const int runs = a.cols / 32;
  for (int i = tid; i < xrows * runs * 8; i += blockDim.x) {
    const int c = i & 7, n = (i >> 3) % runs, r = (i >> 3) / runs;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t at = int64_t(r) * a.cols + n * 32 + c * 4 + j;
      if constexpr (MODE == MV_GLU_IN) {
        const float g = to_f32(static_cast<const InT*>(a.x)[at]), u = to_f32(static_cast<const InT*>(a.x2)[at]);
        v[j] = a.glu ? swiglu_f32(g, u) : swiglu_mlx<InT>(g, u);
      } else {
        v[j] = to_f32(static_cast<const InT*>(a.x)[at]);
      }
    }
    *reinterpret_cast<float4*>(xs + xs_index(r, n, c, a.cols)) = make_float4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();

  // ---- this block's share of the (unit, chunk) list
  const int units = sh_count[0];
  const int per_unit = int(ceil_div(a.rows, a.chunk_rows));
  const int64_t total = int64_t(units) * per_unit;
  const int64_t c0 = total * blockIdx.x / gridDim.x, c1 = total * (blockIdx.x + 1) / gridDim.x;
  const int64_t part_bytes = int64_t(a.chunk_rows) * a.rbytes;
  const int part_stride = align16(int(part_bytes) + 16);  // GATEUP: where the up rows start in a stage

  if (warp == MV_WARPS) {
    // ---- producer warp: lane 0 issues bulk copies; the whole warp copies chunks that are not 16-byte aligned
    for (int64_t c = c0; c < c1; ++c) {
      const int i = int(c - c0), s = i % a.stages;
      if (i >= a.stages) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&empty[s], ((i / a.stages) - 1) & 1, a.err);
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        __syncwarp();
      }
      const int u = int(c / per_unit), rc = int(c % per_unit);
      const int r0 = rc * a.chunk_rows, nr = min(a.chunk_rows, a.rows - r0);
      const uint32_t bytes = uint32_t(int64_t(nr) * a.rbytes);
      uint8_t* dst = stage0 + int64_t(s) * a.stage_bytes;
      const uint8_t* src[2] = {ubase[u] + int64_t(r0) * a.rbytes, MODE == MV_GATEUP ? ubase2[u] + int64_t(r0) * a.rbytes : nullptr};
      const int parts = MODE == MV_GATEUP ? 2 : 1;
      bool aligned = (bytes & 15) == 0;
      for (int q = 0; q < parts; ++q) aligned = aligned && ((reinterpret_cast<uintptr_t>(src[q]) & 15) == 0);
      if (aligned) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], bytes * parts);
          for (int q = 0; q < parts; ++q) bulk_load(dst + q * part_stride, src[q], bytes, &full[s]);
        }
      } else {
        for (int q = 0; q < parts; ++q)
          for (uint32_t b = lane; b < bytes; b += 32) dst[q * part_stride + b] = src[q][b];
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);  // release: the warp's stores above are visible to the waiters
      }
    }
    return;
  }

  // ---- consumer warps
  const int P = a.lanes, rows_per_warp = 32 / P;
  const int part = lane % P, sub = lane / P;
  for (int64_t c = c0; c < c1; ++c) {
    const int i = int(c - c0), s = i % a.stages;
    if (!mbar_wait(&full[s], (i / a.stages) & 1, a.err)) break;
    const int u = int(c / per_unit), rc = int(c % per_unit);
    const int r0 = rc * a.chunk_rows, nr = min(a.chunk_rows, a.rows - r0);
    const uint8_t* stage = stage0 + int64_t(s) * a.stage_bytes;
    const int ns = ucnt[u], so = uoff[u];
    for (int lr = warp * rows_per_warp + sub; lr - sub < nr; lr += MV_WARPS * rows_per_warp) {
      const bool live = lr < nr;
      const uint8_t* row = stage + int64_t(live ? lr : 0) * a.rbytes;
      for (int g0 = 0; g0 < ns; g0 += SG) {
        float acc[SG], acc2[SG];
        int xr[SG];
#pragma unroll
        for (int q = 0; q < SG; ++q) {
          acc[q] = 0.f;
          acc2[q] = 0.f;
          xr[q] = g0 + q < ns ? int(slots[so + g0 + q] >> 16) : 0;
        }
        if (live) {
          for (int n = part; n < runs; n += P) {
            float w[32];
            unpack32<KIND>(row, n, w, tabs);
            float w2[MODE == MV_GATEUP ? 32 : 1];
            if constexpr (MODE == MV_GATEUP) unpack32<KIND>(row + part_stride, n, w2, tabs);
#pragma unroll
            for (int q = 0; q < SG; ++q) {
              if (g0 + q < ns) {
                float sum = 0.f, sum2 = 0.f;
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                  const float4 v = *reinterpret_cast<const float4*>(xs + xs_index(xr[q], n, cc, a.cols));
                  sum = fmaf(w[4 * cc], v.x, sum);
                  sum = fmaf(w[4 * cc + 1], v.y, sum);
                  sum = fmaf(w[4 * cc + 2], v.z, sum);
                  sum = fmaf(w[4 * cc + 3], v.w, sum);
                  if constexpr (MODE == MV_GATEUP) {
                    sum2 = fmaf(w2[4 * cc], v.x, sum2);
                    sum2 = fmaf(w2[4 * cc + 1], v.y, sum2);
                    sum2 = fmaf(w2[4 * cc + 2], v.z, sum2);
                    sum2 = fmaf(w2[4 * cc + 3], v.w, sum2);
                  }
                }
                acc[q] += sum;
                if constexpr (MODE == MV_GATEUP) acc2[q] += sum2;
              }
            }
          }
        }
#pragma unroll
        for (int q = 0; q < SG; ++q) {
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            if (o < P) {
              acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], o);
              if constexpr (MODE == MV_GATEUP) acc2[q] += __shfl_xor_sync(0xffffffffu, acc2[q], o);
            }
          }
        }
        if (live && part == 0) {
#pragma unroll
          for (int q = 0; q < SG; ++q) {
            if (g0 + q < ns) {
              const int orow = int(slots[so + g0 + q] & 0xffffu);
              float v = acc[q];
              if constexpr (MODE == MV_GATEUP) v = swiglu_mlx<InT>(acc[q], acc2[q]);
              static_cast<InT*>(a.out)[int64_t(orow) * a.rows + r0 + lr] = from_f32<InT>(v);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// ---- host side

struct MvPlan {
  int chunk_rows, stage_bytes, stages, grid, smem;
};

template <int KIND>
static MvPlan mv_plan(const MvArgs& a, int mode, int units_max, int xrows) {
  MvPlan p{};
  const int parts = mode == MV_GATEUP ? 2 : 1;
  const int64_t target = 8192;  // bytes of a stack a chunk carries
  // a chunk: whole passes of the consumer warps over rows, and rows that end on 16 bytes (bulk copies)
  const int per_pass = MV_WARPS * (32 / mv_lanes(a.cols));
  const int align_rows = 16 / std::gcd(int(a.rbytes % 16), 16);
  const int unit = std::lcm(per_pass, align_rows);
  int cr = unit * int(std::max<int64_t>(1, target / (int64_t(unit) * a.rbytes * parts)));
  cr = std::min(cr, a.rows);
  p.chunk_rows = cr;
  const int part_stride = align16(int(int64_t(cr) * a.rbytes) + 16);
  p.stage_bytes = parts * part_stride;
  const int budget = 100 * 1024;
  p.stages = std::max(2, std::min(MV_MAX_STAGES, budget / p.stage_bytes));
  const MvLayout L = mv_layout<KIND>(a.bases ? 1 : a.experts, a.pairs, xrows, a.cols, p.stage_bytes, p.stages);
  p.smem = L.total;
  const int64_t chunks = int64_t(units_max) * ceil_div(a.rows, cr);
  p.grid = int(std::min<int64_t>(chunks, 148 * 2));
  return p;
}

template <int KIND, typename InT, int MODE>
static int mv_launch(MvArgs a, int units_max, int sg_hint, cudaStream_t s) {
  const int xrows = MODE == MV_PLAIN || MODE == MV_GATEUP ? (a.pairs + a.share - 1) / a.share : a.pairs;
  MvPlan p = mv_plan<KIND>(a, MODE, units_max, xrows);
  if (p.smem > 227 * 1024) return SC_ERR_SHAPE;
  a.chunk_rows = p.chunk_rows;
  a.stage_bytes = p.stage_bytes;
  a.stages = p.stages;
  a.lanes = mv_lanes(a.cols);
  auto go = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
    kern<<<p.grid, MV_THREADS, p.smem, s>>>(a);
  };
  if (sg_hint <= 1) go(mv_kernel<KIND, InT, MODE, 1>);
  else if (sg_hint <= 2) go(mv_kernel<KIND, InT, MODE, 2>);
  else if (sg_hint <= 4) go(mv_kernel<KIND, InT, MODE, 4>);
  else go(mv_kernel<KIND, InT, MODE, 8>);
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

template <int KIND>
int mv_dispatch(MvArgs a, int mode, int dtype, int units_max, int sg_hint, cudaStream_t s) {
  int rc = SC_ERR_DTYPE;
  dispatch_dtype(dtype, [&]<typename InT>() {
    if (mode == MV_PLAIN) rc = mv_launch<KIND, InT, MV_PLAIN>(a, units_max, sg_hint, s);
    else if (mode == MV_GLU_IN) rc = mv_launch<KIND, InT, MV_GLU_IN>(a, units_max, sg_hint, s);
    else if (mode == MV_GATEUP) rc = mv_launch<KIND, InT, MV_GATEUP>(a, units_max, sg_hint, s);
    else rc = SC_ERR_ARG;
  });
  return rc;
}

}  // namespace sc
