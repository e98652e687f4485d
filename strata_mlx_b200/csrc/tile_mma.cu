// The tile product on the fifth-generation tensor cores: C (P, rows) float32 = A (P, cols) . W[e]^T for tiles of
// 16 slots that each belong to one expert e (strata_mlx/blocks.py:465-536 tile_matmul). A is float16 or bfloat16;
// the weights are decoded from their blocks and rounded to A's type before they multiply (blocks.py:492); sums are
// float32 in tensor memory.
//
// One persistent block per SM. A work item is (group, 128-row block): a group is up to 8 consecutive tiles of one
// expert (N = 16..128 slots), so an expert's weights are decoded once for all of its slots. Per item, 256 columns
// (a chunk) at a time:
//   - the producer warp brings the 128 weight rows' blocks of the chunk into shared memory by TMA (a row's blocks
//     for 256 columns are contiguous; rows whose chunks start at the same offset modulo 16 bytes come in one 2-D box,
//     so one to eight boxes per chunk) and, by TMA, the slots' 64-column slices of A (128-byte swizzle, K-major: the
//     MMA's B operand, one box per power-of-two run of tiles);
//   - a decoder warpgroup (two of them take alternate chunks) decodes the chunk with one thread per weight row and
//     stores the row's 256 weights, rounded to A's type, straight into tensor memory: the MMA's A operand, so
//     decoded weights never pass through shared memory;
//   - one thread issues 128 x N x 16 MMAs (A from tensor memory, B from shared memory) into a tensor-memory
//     accumulator;
//   - four epilogue warps move a finished accumulator to C while the next item fills the other one.
// Tensor memory (512 columns): accumulators at columns 0 and 128, decoded weights of two chunks at 256 and 384.
// Every wait is bounded; a wait that gives up records SC_ERR_TIMEOUT and the block winds down.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "decode.cuh"
#include "tiles.cuh"

namespace sc {
namespace tm {

// Event stamps of block 0 for a profiling build (-DSC_TRACE): %globaltimer per event kind and counter.
#ifdef SC_TRACE
__device__ unsigned long long g_tt[16][1024];
__device__ int g_tt_block;
__device__ unsigned long long g_acc[4][1024];  // per block: decode time, w_empty wait, raw wait, chunks
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define TT(k, i)                                                      \
  do {                                                                \
    if (int(blockIdx.x) == g_tt_block && (i) < 1024) {                \
      unsigned long long t_;                                          \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));          \
      g_tt[k][i] = t_;                                                \
    }                                                                 \
  } while (0)
#else
#define TT(k, i) \
  do {           \
  } while (0)
#endif

constexpr int BM = 128;       // weight rows of an item: the MMA's M, one tensor-memory lane each
constexpr int SUBK = 64;      // columns of a B stage: one 128-byte swizzle atom of 16-bit values
constexpr int CHK = 256;      // columns of a chunk
constexpr int NMAX = 128;     // slots of a group: the MMA's largest N here
constexpr int GROUP_TILES = NMAX / TOKENS_TILE;
constexpr int BSTAGES = 8;    // B stages (A's 64-column slices): enough in flight to cover the loads' latency
// warps: 0 weight-block producer, 1 MMA, 2-5 and 6-9 decoder warpgroups, 10-13 epilogue, 14 A producer
constexpr int EPI_WARP0 = 10, APROD_WARP = 14;
constexpr int WARPS = APROD_WARP + 1;
constexpr int THREADS = WARPS * 32;
constexpr int MAX_TILES = 4096;  // tiles of a call (P <= 65536 slots)
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0, WCOL = 2 * NMAX;  // accumulators; decoded weights (two chunks of 128 columns)
constexpr int B_STAGE = NMAX * SUBK * 2;      // 16 KB

__host__ __device__ constexpr int chunk_bytes(int kind) {
  return CHK / block_info(kind).per_block * block_info(kind).block_bytes;
}
// a row's chunk starts on an even byte, so its 16-byte aligned cover is at most align16(bytes + 14) long; a raw box
// row is this wide, an odd number of 16-byte units, so that eight consecutive rows' 16-byte loads fall in distinct
// banks
__host__ __device__ constexpr int slot_bytes(int kind) {
  return align16(chunk_bytes(kind) + 14) + ((align16(chunk_bytes(kind) + 14) / 16) % 2 == 0 ? 16 : 0);
}

// kinds decoded from registers with a grid table replicated 16 times (lane l reads copy l % 16: at most two lanes
// of a warp on one bank)
constexpr int GRID_COPIES = 16;
__host__ __device__ constexpr bool fast_kind(int kind) { return kind == SC_IQ3_XXS; }
__host__ __device__ constexpr int tab_bytes(int kind) {
  return fast_kind(kind) ? 256 * 4 * GRID_COPIES : table_bytes(kind);
}

struct Layout {
  int b, raw, tabs, groups, bars, total;
};

__host__ __device__ constexpr Layout layout(int kind, int raw_stages) {
  Layout l{};
  l.b = 0;
  l.raw = l.b + BSTAGES * B_STAGE;
  l.tabs = l.raw + raw_stages * BM * slot_bytes(kind);
  l.groups = align16(l.tabs + tab_bytes(kind) + 8);
  l.bars = l.groups + MAX_TILES * 4;
  l.total = l.bars + 512 + 1024;  // barriers and scratch, plus the slack to align the base to 1024 bytes
  return l;
}

constexpr int SMEM_LIMIT = 227 * 1024;
__host__ __device__ constexpr int raw_stages_for(int kind) {
  return layout(kind, 4).total <= SMEM_LIMIT ? 4 : layout(kind, 3).total <= SMEM_LIMIT ? 3 : 2;
}

// ---- PTX wrappers

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// K-major operand in 128-byte swizzle atoms (8 rows x 128 bytes, atoms 1024 bytes apart), version 1 (sm_100)
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  return uint64_t((smem_u32(p) & 0x3FFFF) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16 instruction descriptor: float32 accumulator, A and B of the activations' type, both K-major
template <typename T>
__device__ __forceinline__ uint32_t instr_desc(int n) {
  constexpr uint32_t fmt = std::is_same_v<T, __nv_bfloat16> ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

// D (tensor memory) (+)= A (tensor memory, 128 lanes x 16 values) . B (shared memory)^T; no output lane disabled
// (the form with the disable-output-lane operand issued faster than the form without it, measured here)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ bool elect_one() {
  uint32_t p;
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, e;\n\t}"
      : "=r"(p));
  return p != 0;
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 columns of this thread's lane into registers
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 columns of this thread's lane from registers; waits until the store is done
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

// block-wide scans over THREADS threads; `sh` holds WARPS ints
__device__ __forceinline__ int block_excl_sum(int v, int* sh, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  int before = 0;
  total = 0;
  for (int w = 0; w < WARPS; ++w) {
    const int t = sh[w];
    if (w < warp) before += t;
    total += t;
  }
  __syncthreads();
  return before + x - v;
}
__device__ __forceinline__ int block_excl_max(int v, int* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x = max(x, y);
  }
  int prev = __shfl_up_sync(0xffffffffu, x, 1);
  if (lane == 0) prev = -1;
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  for (int w = 0; w < warp; ++w) prev = max(prev, sh[w]);
  __syncthreads();
  return prev;
}

// ---- IQ3_XXS from registers (strata_mlx/blocks.py:103-115): the block's 98 bytes as words (byte i at
// word i / 4, bits 8 (i % 4)). Weight j of grid entry l of run r is d_r * grid[qs[8 r + l]] byte j, negated when bit j
// of sign nibble l is set; d_r = d (0.5 + aux_r >> 28) 0.5 in float32, as unpack32 computes it.
//   - the product: fma(2^23 + byte, d_r, -2^23 d_r) is d_r * byte rounded once (2^23 + byte and 2^23 d_r are
//     exact), with 2^23 + byte made by one byte permute, two weights per packed float32x2 fma;
//   - the sign: applied to the rounded pair (rounding to nearest commutes with negation), the pair's two sign bits
//     moved to bits 15 and 31 by one multiply (bit b to 15 and bit b + 1 to 31: s8 * (2^(15-b) + 2^(30-b)));
//   - ksigns[i] = i | parity(i) << 7 (gguf-py's table; the sign bytes have even parity).
// `grid` is this lane's copy of the replicated grid table (entry e at grid[GRID_COPIES e]).
// `q` holds the block's bytes from 16 i (i = the slice) on, so that run r (0 or 1 of the slice) has its grid
// indices at bytes 2 + 8 r .. 9 + 8 r of q; aux is the run's sign and scale word.
template <typename T>
__device__ __forceinline__ void iq3xxs_run(const uint32_t (&q)[17], uint32_t aux, int r, float d,
                                           const uint32_t* grid, uint32_t* out /* 16 pairs */) {
  const float dr = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, float(aux >> 28))), 0.5f);
  const float2 dd = make_float2(dr, dr), cc = make_float2(dr * -8388608.0f, dr * -8388608.0f);
#pragma unroll
  for (int k = 0; k < 4; ++k) {  // grid entries 2k and 2k + 1 share a sign byte
    const uint32_t s7 = (aux >> (7 * k)) & 127u;
    const uint32_t s8 = s7 | ((__popc(s7) & 1u) << 7);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int l = 2 * k + h, qb = 2 + 8 * r + l;  // the grid index byte
      const uint32_t g = grid[__byte_perm(q[qb >> 2], 0u, 0x4440u | uint32_t(qb & 3)) * GRID_COPIES];
      const float2 a0 = make_float2(__uint_as_float(__byte_perm(g, 0x4B000000u, 0x7540u)),
                                    __uint_as_float(__byte_perm(g, 0x4B000000u, 0x7541u)));
      const float2 a1 = make_float2(__uint_as_float(__byte_perm(g, 0x4B000000u, 0x7542u)),
                                    __uint_as_float(__byte_perm(g, 0x4B000000u, 0x7543u)));
      const float2 v0 = __ffma2_rn(a0, dd, cc), v1 = __ffma2_rn(a1, dd, cc);
      constexpr uint32_t M[4] = {0x40008000u, 0x10002000u, 0x04000800u, 0x01000200u};  // bits 0, 2, 4, 6
      out[2 * l] = pack2<T>(v0.x, v0.y) ^ ((s8 * M[2 * h]) & 0x80008000u);
      out[2 * l + 1] = pack2<T>(v1.x, v1.y) ^ ((s8 * M[2 * h + 1]) & 0x80008000u);
    }
  }
}

// 32 columns of this thread's lane from registers, not waited for (tcgen05.wait::st does)
__device__ __forceinline__ void tmem_st32_async(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int KIND, typename T, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    tile_mma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap16,
                    const __grid_constant__ CUtensorMap amap32, const __grid_constant__ CUtensorMap amap64,
                    const __grid_constant__ CUtensorMap amap128, const uint8_t* __restrict__ blocks, int experts,
                    int rows, int cols, int64_t rbytes, int phases, int P, const uint32_t* __restrict__ tile_expert,
                    const TileOut to, int* err, int raw_stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = layout(KIND, raw_stages);
  constexpr int SLOT = slot_bytes(KIND), CB = chunk_bytes(KIND);
  uint8_t* bst = smem + L.b;
  uint8_t* raw = smem + L.raw;
  uint32_t* groups = reinterpret_cast<uint32_t*>(smem + L.groups);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* b_full = bars;                  // [BSTAGES]: the producer's expect_tx
  uint64_t* b_empty = b_full + BSTAGES;     // [BSTAGES]: the MMAs of the stage
  uint64_t* raw_full = b_empty + BSTAGES;   // [4]: the raw boxes
  uint64_t* raw_empty = raw_full + 4;       // [4]: the 4 warps of the decoding warpgroup
  uint64_t* w_full = raw_empty + 4;         // [2][4]: a chunk's 64-column slice in tensor memory, 4 warps
  uint64_t* w_empty = w_full + 8;           // [2]: the MMAs of the chunk
  uint64_t* acc_full = w_empty + 2;         // [2]: the item's MMAs
  uint64_t* acc_empty = acc_full + 2;       // [2]: 4 epilogue warps
  uint64_t* done = acc_empty + 2;           // the last MMAs, before tensor memory is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* scan = reinterpret_cast<int*>(tmem_slot + 1);  // [WARPS]
  int* ngroups = scan + WARPS;
  volatile int* bail = ngroups + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#ifdef SC_TRACE
  if (tid == 0) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g_tt[14][blockIdx.x % 1024]));
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_tt[13][blockIdx.x % 1024] = smid;
  }
#endif
  Tabs tabs{};
  uint32_t* grid_rep = reinterpret_cast<uint32_t*>(smem + L.tabs);
  if constexpr (fast_kind(KIND)) {
    for (int i = tid; i < 256 * GRID_COPIES; i += THREADS) grid_rep[i] = IQ3XXS_GRID[i / GRID_COPIES];
  } else {
    tabs = load_tabs<KIND>(smem + L.tabs);
  }
  if (tid == 0) {
    for (int i = 0; i < BSTAGES; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 4);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&w_full[i], 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(done, 1);
    *bail = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // ---- the groups: runs of tiles of one expert, split every GROUP_TILES tiles from the run's start; tiles of no
  // expert (>= experts) make no group. Every block works the list out the same way.
  const int T_ = P / TOKENS_TILE;
  const int per = (T_ + THREADS - 1) / THREADS;
  const int i0 = min(T_, tid * per), i1 = min(T_, i0 + per);
  int last_start = -1;
  for (int i = i0; i < i1; ++i)
    if (i == 0 || __ldg(tile_expert + i) != __ldg(tile_expert + i - 1)) last_start = i;
  int run = block_excl_max(last_start, scan);
  int mine = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t e = __ldg(tile_expert + i);
    if (i == 0 || e != __ldg(tile_expert + i - 1)) run = i;
    mine += e < uint32_t(experts) && (i - run) % GROUP_TILES == 0;
  }
  int total;
  int at = block_excl_sum(mine, scan, total);
  run = block_excl_max(last_start, scan);
  for (int i = i0; i < i1; ++i) {
    const uint32_t e = __ldg(tile_expert + i);
    if (i == 0 || e != __ldg(tile_expert + i - 1)) run = i;
    if (e < uint32_t(experts) && (i - run) % GROUP_TILES == 0) {
      int n = 1;
      while (n < GROUP_TILES && i + n < T_ && __ldg(tile_expert + i + n) == e) ++n;
      groups[at++] = uint32_t(i) | (uint32_t(n - 1) << 12) | (e << 16);
    }
  }
  if (tid == 0) *ngroups = total;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int RB = rows / BM, KC = cols / CHK;
  const int items = *ngroups * RB;

  if (warp == 0) {
    // ---- weight-block producer: per chunk, the item's 128 rows' blocks
    uint32_t rc = 0;
    bool ok = true;
    if (lane == 0) {
      for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x) {
        const uint32_t g = groups[item / RB];
        const int r0 = (item % RB) * BM, e = int(g >> 16);
        const int y0 = int((int64_t(e) * rows + r0) / phases);  // the item's first row of phase rows
        for (int j = 0; j < KC; ++j) {
          const int rs = int(rc % uint32_t(raw_stages));
          if (!(ok = mbar_wait_sleep(&raw_empty[rs], ((rc / raw_stages) & 1) ^ 1, err))) break;
          // phase k: the rows r with r % phases == k, whose chunk j starts k * rbytes + j * CB into a phase row
          mbar_arrive_expect_tx(&raw_full[rs], uint32_t(BM * SLOT));
          for (int k = 0; k < phases; ++k)
            tma_load_2d(raw + (rs * BM + k * (BM / phases)) * SLOT, &wmap,
                        int((k * rbytes + int64_t(j) * CB) & ~int64_t(15)), y0, &raw_full[rs]);
          TT(0, rc);
          ++rc;
        }
      }
      if (!ok) *bail = 1;
      // in-flight copies land before the block may end: wait (briefly) for the last phase of every stage armed
      for (uint32_t i = rc > uint32_t(raw_stages) ? rc - raw_stages : 0; i < rc; ++i)
        mbar_wait_sleep(&raw_full[i % raw_stages], (i / raw_stages) & 1, nullptr, 20000000LL);
    }
    __syncwarp();
  } else if (warp == APROD_WARP) {
    // ---- A producer: per chunk, the group's four 64-column slices of A
    uint32_t bc = 0;
    bool ok = true;
    if (lane == 0) {
      for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x) {
        const uint32_t g = groups[item / RB];
        const int st = int(g & 0xfff), nt = int((g >> 12) & 15) + 1;
        for (int j = 0; j < KC && ok; ++j) {
          for (int i = 0; i < CHK / SUBK; ++i) {
            const int bs = int(bc % BSTAGES);
            if (!(ok = mbar_wait_sleep(&b_empty[bs], ((bc / BSTAGES) & 1) ^ 1, err))) break;
            mbar_arrive_expect_tx(&b_full[bs], uint32_t(nt * TOKENS_TILE * SUBK * 2));
            int at = 0;  // the group's tiles in runs of 8, 4, 2 and 1 tiles, one box each
#pragma unroll
            for (int b = 3; b >= 0; --b)
              if ((nt >> b) & 1) {
                const CUtensorMap* map = b == 3 ? &amap128 : b == 2 ? &amap64 : b == 1 ? &amap32 : &amap16;
                tma_load_2d(bst + bs * B_STAGE + at * TOKENS_TILE * 128, map, j * CHK + i * SUBK,
                            (st + at) * TOKENS_TILE, &b_full[bs]);
                at += 1 << b;
              }
            TT(1, bc);
            ++bc;
          }
        }
      }
      if (!ok) *bail = 1;
      for (uint32_t i = bc > uint32_t(BSTAGES) ? bc - BSTAGES : 0; i < bc; ++i)
        mbar_wait_sleep(&b_full[i % BSTAGES], (i / BSTAGES) & 1, nullptr, 20000000LL);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: the whole warp follows the loop and waits (a wait that gives up in any lane ends the loop in
    // all of them); one elected lane issues. All 512 columns are
    // this block's, so tensor memory starts at address 0: the MMAs' addresses are loop constants.
    const bool leader = elect_one();
    uint32_t bc = 0, jc = 0, ic = 0;
    bool ok = tmem == 0;
    if (!ok) record_error(err, SC_ERR_CUDA);
    for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x, ++ic) {
      const uint32_t g = groups[item / RB];
      const int nt = int((g >> 12) & 15) + 1;
      const int b = int(ic & 1);
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[b], ((ic >> 1) & 1) ^ 1, err)))) break;
      if (leader) TT(5, ic);
      tc_fence_after();
      const uint32_t d = uint32_t(ACC_COL + b * NMAX);
      const uint32_t idesc = instr_desc<T>(nt * TOKENS_TILE);
      for (int j = 0; j < KC && ok; ++j, ++jc) {
        const int wr = int(jc & 1);
        for (int i = 0; i < CHK / SUBK; ++i) {
          const int bs = int(bc % BSTAGES);
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&w_full[wr * 4 + i], (jc >> 1) & 1, err)))) break;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&b_full[bs], (bc / BSTAGES) & 1, err)))) break;
          if (leader) TT(4, bc);
          tc_fence_after();
          const uint32_t a = uint32_t(WCOL + wr * 128 + i * 32);
          const uint64_t bd = smem_desc(bst + bs * B_STAGE);
          if (leader) {
#pragma unroll
            for (int k = 0; k < SUBK / 16; ++k) mma_ts(d, a + 8 * k, bd + 2 * k, idesc, (j | i | k) != 0);
            mma_commit(&b_empty[bs]);
          }
          __syncwarp();
          ++bc;
        }
        if (ok && leader) mma_commit(&w_empty[wr]);
        __syncwarp();
      }
      if (ok && leader) mma_commit(&acc_full[b]);
      __syncwarp();
    }
    if (!ok) *bail = 1;
    if (leader) {
      mma_commit(done);  // arrives once every MMA this thread issued has finished
      mbar_wait(done, 0, nullptr, 20000000LL);
    }
    __syncwarp();
  } else if (warp >= 2 && warp < EPI_WARP0) {
    // ---- decoders: warpgroup wg takes the chunks jc with jc % 2 == wg; thread = weight row = tensor-memory lane
    const int wg = (warp - 2) >> 2, quarter = warp & 3;
    const int m = 32 * quarter + lane;
    const int phase = m % phases, slot = phase * (BM / phases) + m / phases;  // where the raw boxes put row m
    const uint32_t lane_addr = tmem + (uint32_t(32 * quarter) << 16);
    uint32_t jc = 0, rc = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x) {
      for (int j = 0; j < KC; ++j, ++jc, ++rc) {
        if (int(jc & 1) != wg) continue;
        const int rs = int(rc % uint32_t(raw_stages));
        const int wr = int(jc & 1);
#ifdef SC_TRACE
        const unsigned long long t_a = gtime();
#endif
        if (!(ok = mbar_wait_sleep(&raw_full[rs], (rc / raw_stages) & 1, err))) break;
        if (lane == 0 && quarter == 0) TT(8, jc);
#ifdef SC_TRACE
        const unsigned long long t_b = gtime();
#endif
        if (!(ok = mbar_wait_sleep(&w_empty[wr], ((jc >> 1) & 1) ^ 1, err))) break;
        if (lane == 0 && quarter == 0) TT(2, jc);
#ifdef SC_TRACE
        const unsigned long long t_c = gtime();
#endif
        tc_fence_after();
        const uint8_t* row = raw + (rs * BM + slot) * SLOT;
        const int s = int((phase * rbytes + int64_t(j) * CB) & 15);
        if constexpr (fast_kind(KIND)) {
          // the row's cover into registers, then shifted so that word 0 starts at the block
          uint32_t w[28];
#pragma unroll
          for (int q = 0; q < 7; ++q) {
            const uint4 v = *reinterpret_cast<const uint4*>(row + 16 * q);
            w[4 * q] = v.x, w[4 * q + 1] = v.y, w[4 * q + 2] = v.z, w[4 * q + 3] = v.w;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[rs]);  // the shared-memory copy is no longer needed
          if (s & 8) {
#pragma unroll
            for (int q = 0; q < 26; ++q) w[q] = w[q + 2];
          }
          if (s & 4) {
#pragma unroll
            for (int q = 0; q < 27; ++q) w[q] = w[q + 1];
          }
          if (s & 2) {
#pragma unroll
            for (int q = 0; q < 27; ++q) w[q] = __byte_perm(w[q], w[q + 1], 0x5432);
          }
          const float d = half_bits(w[0] & 0xffffu);
          const uint32_t* grid = grid_rep + (lane % GRID_COPIES);
          // The slice loop stays rolled, so that the decoders' code fits the instruction cache: q and x slide down
          // by one slice's bytes each iteration instead of being indexed by the slice. Slice i's store is waited
          // for after slice i + 1 is decoded, so that the store's latency hides behind the work.
          uint32_t q[17], x[9];
#pragma unroll
          for (int k = 0; k < 17; ++k) q[k] = w[k];
#pragma unroll
          for (int k = 0; k < 9; ++k) x[k] = w[16 + k];
#pragma unroll 1
          for (int i = 0; i < 4; ++i) {
            uint32_t out[32];
            iq3xxs_run<T>(q, __byte_perm(x[0], x[1], 0x5432), 0, d, grid, out);
            iq3xxs_run<T>(q, __byte_perm(x[1], x[2], 0x5432), 1, d, grid, out + 16);
#pragma unroll
            for (int k = 0; k < 13; ++k) q[k] = q[k + 4];
#pragma unroll
            for (int k = 0; k < 7; ++k) x[k] = x[k + 2];
            if (i > 0) {
              tmem_st_wait();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&w_full[wr * 4 + i - 1]);
            }
            tmem_st32_async(lane_addr + uint32_t(WCOL + wr * 128 + 32 * i), out);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&w_full[wr * 4 + 3]);
          if (lane == 0 && quarter == 0) TT(3, jc);
#ifdef SC_TRACE
          if (lane == 0 && quarter == 0) {
            atomicAdd(&g_acc[0][blockIdx.x % 1024], gtime() - t_c);
            atomicAdd(&g_acc[1][blockIdx.x % 1024], t_c - t_b);
            atomicAdd(&g_acc[2][blockIdx.x % 1024], t_b - t_a);
            atomicAdd(&g_acc[3][blockIdx.x % 1024], 1ull);
          }
#endif
        } else {
          const uint8_t* blk = row + s;
#pragma unroll 1
          for (int i = 0; i < 4; ++i) {
            uint32_t out[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float v[32];
              unpack32<KIND>(blk, 2 * i + h, v, tabs);
#pragma unroll
              for (int p = 0; p < 16; ++p) out[16 * h + p] = pack2<T>(v[2 * p], v[2 * p + 1]);
            }
            tmem_st32(lane_addr + uint32_t(WCOL + wr * 128 + 32 * i), out);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_full[wr * 4 + i]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[rs]);
        }
      }
    }
    if (!ok) *bail = 1;
  } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + 4) {
    // ---- epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31, the item's rows r0 + 32 (w % 4) + lane
    const int quarter = warp & 3;
    uint32_t ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x, ++ic) {
      const uint32_t g = groups[item / RB];
      const int r0 = (item % RB) * BM, st = int(g & 0xfff), nt = int((g >> 12) & 15) + 1;
      const int b = int(ic & 1);
      if (!(ok = mbar_wait_sleep(&acc_full[b], (ic >> 1) & 1, err))) break;
      if (lane == 0 && quarter == 0) TT(6, ic);
      tc_fence_after();
      const int row = r0 + 32 * quarter + lane;
      for (int n0 = 0; n0 < nt * TOKENS_TILE; n0 += 32) {
        float v[32];
        tmem_ld32(tmem + (uint32_t(32 * quarter) << 16) + uint32_t(ACC_COL + b * NMAX + n0), v);
        const int n = min(32, nt * TOKENS_TILE - n0);
        const int64_t at = (int64_t(st) * TOKENS_TILE + n0) * rows + row;  // slot st 16 + n0 (+ i), row
        if constexpr (MODE == 0) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < n) to.c[at + int64_t(i) * rows] = v[i];
        } else if constexpr (MODE == 1) {
          T* o = static_cast<T*>(to.out) + at;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < n) o[int64_t(i) * rows] = from_f32<T>(v[i]);
        } else {
          // lane j holds the pair of slot st 16 + n0 + j; the pairs go to every lane by shuffles
          const int mine = lane < n ? to.pair_of_slot[st * TOKENS_TILE + n0 + lane] : -1;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int p = __shfl_sync(0xffffffffu, mine, i);
            if (p >= 0) static_cast<T*>(to.out)[int64_t(p) * rows + row] = from_f32<T>(v[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (lane == 0 && quarter == 0) TT(7, ic);
    }
    if (!ok) *bail = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
#ifdef SC_TRACE
  if (tid == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g_tt[15][blockIdx.x % 1024]));
#endif
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time dependence on its version)
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_tiled() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

// rows whose chunks start at the same offset modulo 16 bytes: rows r and r + phases(rb)
inline int phases_of(int64_t rb) {
  int64_t g = rb & 15;
  int64_t a = 16;
  while (g) {  // gcd(rb mod 16, 16)
    const int64_t t = a % g;
    a = g;
    g = t;
  }
  return int(16 / a);
}

template <int KIND, typename T>
int launch(const uint8_t* blocks, int experts, int rows, int cols, int64_t rb, const void* a, int P,
           const uint32_t* tile_expert, const TileOut& to, int* err, cudaStream_t s) {
  EncodeTiled enc = encode_tiled();
  if (!enc) return SC_ERR_CUDA;
  const cuuint32_t estr[2] = {1, 1};
  // A: (P, cols) of T, boxes of 64 columns x 16, 32, 64 or 128 slots, 128-byte swizzle
  CUtensorMap amaps[4];
  const CUtensorMapDataType dt =
      std::is_same_v<T, __nv_bfloat16> ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t adims[2] = {cuuint64_t(cols), cuuint64_t(P)};
  const cuuint64_t astrides[1] = {cuuint64_t(cols) * 2};
  for (int b = 0; b < 4; ++b) {
    const cuuint32_t box[2] = {SUBK, cuuint32_t(TOKENS_TILE << b)};
    if (enc(&amaps[b], dt, 2, const_cast<void*>(a), adims, astrides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return SC_ERR_CUDA;
  }
  // the blocks as bytes in phase rows of `phases` weight rows; boxes of slot_bytes x 128 / phases
  const int phases = phases_of(rb);
  CUtensorMap wmap;
  const cuuint64_t wdims[2] = {cuuint64_t(phases * rb), cuuint64_t(int64_t(experts) * rows / phases)};
  const cuuint64_t wstrides[1] = {cuuint64_t(phases * rb)};
  const cuuint32_t wbox[2] = {cuuint32_t(slot_bytes(KIND)), cuuint32_t(BM / phases)};
  if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(blocks), wdims, wstrides, wbox, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return SC_ERR_CUDA;
  constexpr int RS = raw_stages_for(KIND);
  constexpr int smem = layout(KIND, RS).total;
  static_assert(smem <= SMEM_LIMIT, "tile_mma shared memory");
  auto kern = to.mode == 0 ? tile_mma_kernel<KIND, T, 0>
            : to.mode == 1 ? tile_mma_kernel<KIND, T, 1>
                           : tile_mma_kernel<KIND, T, 2>;
  static bool set[3][64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64 || to.mode < 0 || to.mode > 2) return SC_ERR_CUDA;
  if (!set[to.mode][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return SC_ERR_CUDA;
    set[to.mode][dev] = true;
  }
  const int grid = sm_count();
  if (grid <= 0) return SC_ERR_CUDA;
  kern<<<grid, THREADS, smem, s>>>(wmap, amaps[0], amaps[1], amaps[2], amaps[3], blocks, experts, rows, cols, rb,
                                   phases, P, tile_expert, to, err, RS);
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

}  // namespace tm

#ifdef SC_TRACE
extern "C" SC_API void sc_tt_read(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, tm::g_tt, sizeof(tm::g_tt));
}
extern "C" SC_API void sc_acc_read(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, tm::g_acc, sizeof(tm::g_acc));
}
extern "C" SC_API void sc_tt_clear(int block) {
  static unsigned long long zero[16][1024];
  cudaMemcpyToSymbol(tm::g_tt, zero, sizeof(zero));
  cudaMemcpyToSymbol(tm::g_acc, zero, sizeof(tm::g_acc));
  cudaMemcpyToSymbol(tm::g_tt_block, &block, sizeof(int));
}
#endif

bool tile_mma_takes(int kind, int experts, int rows, int cols, int a_dtype, int P, const void* a, const void* blocks) {
  // Q8_0 (a dense type) is not a tile type: its 256-column chunk is wider than a TMA box row
  return (a_dtype == SC_F16 || a_dtype == SC_BF16) && block_info(kind).per_block && kind != SC_Q8_0 &&
         tm::slot_bytes(kind) <= 256 && rows % tm::BM == 0 &&
         cols % tm::CHK == 0 && P / TOKENS_TILE <= tm::MAX_TILES && experts <= 65535 &&
         reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(blocks) % 16 == 0;
}

int tile_mma_launch(int kind, const uint8_t* blocks, int experts, int rows, int cols, int64_t rbytes, const void* a,
                    int a_dtype, int P, const uint32_t* tile_expert, const TileOut& to, int* err, cudaStream_t s) {
  if (!tile_mma_takes(kind, experts, rows, cols, a_dtype, P, a, blocks)) return SC_ERR_UNSUPPORTED;
  int rc = SC_ERR_UNSUPPORTED;
  dispatch_kind(kind, [&]<int KIND>() {
    if (a_dtype == SC_BF16)
      rc = tm::launch<KIND, __nv_bfloat16>(blocks, experts, rows, cols, rbytes, a, P, tile_expert, to, err, s);
    else
      rc = tm::launch<KIND, __half>(blocks, experts, rows, cols, rbytes, a, P, tile_expert, to, err, s);
  });
  return rc;
}

}  // namespace sc
