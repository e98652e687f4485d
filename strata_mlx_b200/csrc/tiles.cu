// Prefill: a chunk's (token, expert) pairs sorted into tiles of 16 slots, each tile one expert's
// (strata_mlx/blocks.py:539-563 tiles_of), and the tile product on the CUDA cores for float32 activations
// (blocks.py:465-536 tile_matmul; bfloat16/float16 go to the tcgen05 kernel of tile_mma.cu).
#include <algorithm>

#include "decode.cuh"
#include "tiles.cuh"

namespace sc {

// ---- tiles_of: one block of 1024 threads; counts per expert in the workspace, a block-wide scan of the
// experts' tile counts, then every pair takes the next slot of its expert (the order of slots inside an expert's
// tiles is not fixed; every pair's product is the same wherever its slot is)

template <typename IdxT>
__global__ void __launch_bounds__(1024) tiles_of_kernel(const IdxT* __restrict__ idx, int pairs, int k, int experts,
                                                        uint32_t* __restrict__ tile_expert, uint32_t* __restrict__ token,
                                                        uint32_t* __restrict__ where, int* __restrict__ counts,
                                                        int* __restrict__ start) {
  __shared__ int part[1024];
  const int tid = threadIdx.x, nt = blockDim.x;
  const int most = pairs / TOKENS_TILE + min(experts, pairs);
  for (int e = tid; e < experts; e += nt) counts[e] = 0;
  for (int i = tid; i < most * TOKENS_TILE; i += nt) token[i] = 0;
  __syncthreads();
  for (int p = tid; p < pairs; p += nt) {
    const int64_t e = int64_t(idx[p]);
    if (e >= 0 && e < experts) atomicAdd(&counts[e], 1);
  }
  __syncthreads();
  // exclusive scan of ceil(count / 16) over experts: thread t takes a contiguous segment
  const int per = (experts + nt - 1) / nt;
  const int e0 = min(experts, tid * per), e1 = min(experts, e0 + per);
  int mine = 0;
  for (int e = e0; e < e1; ++e) mine += (counts[e] + TOKENS_TILE - 1) / TOKENS_TILE;
  part[tid] = mine;
  __syncthreads();
  for (int o = 1; o < nt; o <<= 1) {
    const int v = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  int run = part[tid] - mine;
  const int used = part[nt - 1];
  for (int e = e0; e < e1; ++e) {
    const int tiles = (counts[e] + TOKENS_TILE - 1) / TOKENS_TILE;
    start[e] = run;
    for (int t = 0; t < tiles; ++t) tile_expert[run + t] = uint32_t(e);
    run += tiles;
    counts[e] = 0;  // from here on: slots taken
  }
  for (int t = used + tid; t < most; t += nt) tile_expert[t] = uint32_t(experts);
  __syncthreads();
  for (int p = tid; p < pairs; p += nt) {
    const int64_t e = int64_t(idx[p]);
    if (e >= 0 && e < experts) {
      const int slot = start[e] * TOKENS_TILE + atomicAdd(&counts[e], 1);
      where[p] = uint32_t(slot);
      token[slot] = uint32_t(p / k);
    } else {
      where[p] = 0xffffffffu;
    }
  }
}

// ---- the tile product on the CUDA cores: a block takes 64 weight rows of one tile's expert, decodes 64
// columns at a time into shared memory (rounded to the activations' type, blocks.py:492) and multiplies the
// tile's 16 tokens by them

template <int KIND, typename InT>
__global__ void __launch_bounds__(256) tile_simt_kernel(const uint8_t* __restrict__ blocks, int experts, int rows,
                                                        int cols, int64_t rbytes, const InT* __restrict__ a,
                                                        const uint32_t* __restrict__ tile_expert, float* __restrict__ c) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t e = tile_expert[blockIdx.y];
  if (e >= uint32_t(experts)) return;  // a tile beyond those the pairs fill
  const Tabs tabs = load_tabs<KIND>(smem);
  float* ws = reinterpret_cast<float*>(smem + align16(table_bytes(KIND) + 8));  // [64][65]
  float* as = ws + 64 * 65;                                                     // [16][64]
  const int tid = threadIdx.x;
  const int r0 = blockIdx.x * 64;
  const uint8_t* wrows = blocks + (int64_t(e) * rows + r0) * rbytes;
  const InT* arows = a + int64_t(blockIdx.y) * TOKENS_TILE * cols;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int tok = tid / 16, rr = tid % 16;
  __syncthreads();
  for (int k0 = 0; k0 < cols; k0 += 64) {
    if (tid < 128) {
      const int r = tid / 2, n = k0 / 32 + (tid % 2);
      float w[32];
      unpack32<KIND>(wrows + int64_t(r) * rbytes, n, w, tabs);
#pragma unroll
      for (int j = 0; j < 32; ++j) ws[r * 65 + (tid % 2) * 32 + j] = round_to<InT>(w[j]);
    }
    for (int i = tid; i < TOKENS_TILE * 64; i += blockDim.x) as[i] = to_f32(arows[int64_t(i / 64) * cols + k0 + i % 64]);
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 64; ++kk) {
      const float av = as[tok * 64 + kk];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(av, ws[(rr + 16 * j) * 65 + kk], acc[j]);
    }
    __syncthreads();
  }
  const int64_t p = int64_t(blockIdx.y) * TOKENS_TILE + tok;
#pragma unroll
  for (int j = 0; j < 4; ++j) c[p * rows + r0 + rr + 16 * j] = acc[j];
}

template <int KIND, typename InT>
int tile_simt_launch(const uint8_t* blocks, int experts, int rows, int cols, int64_t rb, const void* a, int P,
                     const uint32_t* tile_expert, float* c, cudaStream_t s) {
  const int smem = align16(table_bytes(KIND) + 8) + (64 * 65 + 16 * 64) * 4;
  auto kern = tile_simt_kernel<KIND, InT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(rows / 64, P / TOKENS_TILE);
  kern<<<grid, 256, smem, s>>>(blocks, experts, rows, cols, rb, static_cast<const InT*>(a), tile_expert, c);
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

}  // namespace sc

using namespace sc;

extern "C" size_t sc_tiles_of_workspace(int experts) { return size_t(std::max(experts, 0)) * 8 + 64; }

extern "C" int sc_tiles_of(const void* idx, int idx_dtype, int pairs, int k, int experts, uint32_t* tile_expert,
                           uint32_t* token, uint32_t* where, void* workspace, size_t workspace_bytes, void* stream) {
  if (!idx || !tile_expert || !token || !where || pairs < 0 || k < 1 || experts < 1) return SC_ERR_ARG;
  if (!workspace || workspace_bytes < sc_tiles_of_workspace(experts)) return SC_ERR_WORKSPACE;
  if (pairs == 0) return SC_OK;
  int* counts = static_cast<int*>(workspace);
  int* start = counts + experts;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (idx_dtype) {
    case SC_I32:
      tiles_of_kernel<int32_t><<<1, 1024, 0, s>>>(static_cast<const int32_t*>(idx), pairs, k, experts, tile_expert, token,
                                                 where, counts, start);
      break;
    case SC_U32:
      tiles_of_kernel<uint32_t><<<1, 1024, 0, s>>>(static_cast<const uint32_t*>(idx), pairs, k, experts, tile_expert,
                                                  token, where, counts, start);
      break;
    case SC_I64:
      tiles_of_kernel<int64_t><<<1, 1024, 0, s>>>(static_cast<const int64_t*>(idx), pairs, k, experts, tile_expert, token,
                                                 where, counts, start);
      break;
    default:
      return SC_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

extern "C" int sc_tile_matmul_path(int kind, int experts, int rows, int cols, int a_dtype, int P, const void* a,
                                   const void* blocks) {
  return tile_mma_takes(kind, experts, rows, cols, a_dtype, P, a, blocks) ? 1 : 0;
}

extern "C" int sc_tile_matmul(int kind, const void* blocks, int experts, int rows, int cols, const void* a, int a_dtype,
                              int P, const uint32_t* tile_expert, float* c, int* err, void* stream) {
  if (!blocks || !a || !tile_expert || !c || experts < 1 || P < 0) return SC_ERR_ARG;
  if (block_info(kind).per_block == 0) return SC_ERR_KIND;
  if (!tileable(kind, rows, cols) || P % TOKENS_TILE) return SC_ERR_SHAPE;
  if (P == 0) return SC_OK;
  const int64_t rb = row_bytes(kind, cols);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a_dtype != SC_F32) {
    TileOut to{};
    to.mode = 0;
    to.c = c;
    const int rc = tile_mma_launch(kind, static_cast<const uint8_t*>(blocks), experts, rows, cols, rb, a, a_dtype, P,
                                   tile_expert, to, err, s);
    if (rc != SC_ERR_UNSUPPORTED) return rc;
  }
  int rc = SC_ERR_DTYPE;
  dispatch_kind(kind, [&]<int KIND>() {
    dispatch_dtype(a_dtype, [&]<typename InT>() {
      rc = tile_simt_launch<KIND, InT>(static_cast<const uint8_t*>(blocks), experts, rows, cols, rb, a, P, tile_expert, c, s);
    });
  });
  return rc;
}

// ---- a prompt's three tile products in one call (blocks.py:566-576 _tiled_glu): gate and up in A's type, their
// swiglu (sc_swiglu, mlx-lm's rounding), down written in the pairs' order; the same bits as the three tile_matmul
// calls, the swiglu and the unsort

__global__ void slot_pairs_kernel(const uint32_t* __restrict__ where, int pairs, int P, int* __restrict__ pos) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p < pairs && where[p] < uint32_t(P)) pos[where[p]] = p;
}

static size_t glu_part(int P, int inter) { return (size_t(P) * inter * 2 + 15) / 16 * 16; }

extern "C" size_t sc_tile_glu_workspace(int P, int inter, int a_dtype) {
  if (P < 0 || inter < 1 || (a_dtype != SC_F16 && a_dtype != SC_BF16)) return 0;
  return 3 * glu_part(P, inter) + (size_t(P) * 4 + 15) / 16 * 16;
}

extern "C" int sc_tile_glu(int kind_gate, const void* gate, int kind_up, const void* up, int kind_down, const void* down,
                           int experts, int hidden, int inter, const void* a, int a_dtype, int P,
                           const uint32_t* tile_expert, const uint32_t* where, int pairs, void* out, void* workspace,
                           size_t workspace_bytes, int* err, void* stream) {
  if (!gate || !up || !down || !a || !tile_expert || !where || !out || experts < 1 || P < 0 || pairs < 0)
    return SC_ERR_ARG;
  if (a_dtype != SC_F16 && a_dtype != SC_BF16) return SC_ERR_UNSUPPORTED;
  if (P % TOKENS_TILE) return SC_ERR_SHAPE;
  if (!workspace || workspace_bytes < sc_tile_glu_workspace(P, inter, a_dtype)) return SC_ERR_WORKSPACE;
  if (!tile_mma_takes(kind_gate, experts, inter, hidden, a_dtype, P, a, gate) ||
      !tile_mma_takes(kind_up, experts, inter, hidden, a_dtype, P, a, up) ||
      !tile_mma_takes(kind_down, experts, hidden, inter, a_dtype, P, workspace, down))
    return SC_ERR_UNSUPPORTED;
  if (P == 0) return SC_OK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* h = ws;                               // (P, inter): swiglu, the down product's A
  void* g = ws + glu_part(P, inter);          // (P, inter): the gate product in A's type
  void* u = ws + 2 * glu_part(P, inter);      // (P, inter): the up product
  int* pos = reinterpret_cast<int*>(ws + 3 * glu_part(P, inter));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(pos, 0xFF, size_t(P) * 4, s) != cudaSuccess) return SC_ERR_CUDA;
  if (pairs > 0) slot_pairs_kernel<<<int(ceil_div(pairs, 256)), 256, 0, s>>>(where, pairs, P, pos);
  if (cudaGetLastError() != cudaSuccess) return SC_ERR_CUDA;
  TileOut to{};
  to.mode = 1;
  to.out = g;
  if (int rc = tile_mma_launch(kind_gate, static_cast<const uint8_t*>(gate), experts, inter, hidden,
                               row_bytes(kind_gate, hidden), a, a_dtype, P, tile_expert, to, err, s))
    return rc;
  to.out = u;
  if (int rc = tile_mma_launch(kind_up, static_cast<const uint8_t*>(up), experts, inter, hidden,
                               row_bytes(kind_up, hidden), a, a_dtype, P, tile_expert, to, err, s))
    return rc;
  if (int rc = sc_swiglu(g, u, int64_t(P) * inter, a_dtype, h, stream)) return rc;
  to.mode = 2;
  to.out = out;
  to.pair_of_slot = pos;
  return tile_mma_launch(kind_down, static_cast<const uint8_t*>(down), experts, hidden, inter,
                         row_bytes(kind_down, inter), h, a_dtype, P, tile_expert, to, err, s);
}
