// The tile product on the fifth-generation tensor cores: C (P, rows) float32 = A (P, cols) . W[e]^T for tiles of
// 16 slots that each belong to one expert e (strata_mlx/blocks.py:465-536 tile_matmul). A is float16 or bfloat16;
// the weights are decoded from their blocks and rounded to A's type before they multiply (blocks.py:492); sums are
// float32 in tensor memory.
//
// One persistent block per SM. A work item is (group, 128-row block): a group is up to 8 consecutive tiles of one
// expert (N = 16..128 slots), so an expert's weights are decoded once for all of its slots. Per item:
//   - the producer warp brings the item's weight rows through shared memory 256 columns at a time (one bulk copy
//     per row: a row's blocks for 256 columns are contiguous), and the slots' 64-column slices of A by TMA;
//   - eight decoder warps turn each 64-column slice of the 128 rows into a 128 x 64 operand tile (K-major, 128-byte
//     swizzle) with the same unpack32 the other kernels use, rounded to A's type;
//   - one thread issues four 128 x N x 16 MMAs per slice into a tensor-memory accumulator;
//   - four epilogue warps move a finished accumulator to C while the next item fills the other one.
// Every wait is bounded; a wait that gives up records SC_ERR_TIMEOUT and the block winds down.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "decode.cuh"
#include "tiles.cuh"

namespace sc {
namespace tm {

constexpr int BM = 128;       // weight rows of an item: the MMA's M
constexpr int SUBK = 64;      // columns of an operand stage: one 128-byte swizzle atom of 16-bit values
constexpr int CHK = 256;      // columns of a raw stage
constexpr int NMAX = 128;     // slots of a group: the MMA's largest N here
constexpr int GROUP_TILES = NMAX / TOKENS_TILE;
constexpr int STAGES = 4;     // operand stages (decoded weights + A slices)
constexpr int DEC_WARPS = 8;  // 256 decoder threads: one 32-weight run of one row each per stage
constexpr int EPI_WARP0 = 2 + DEC_WARPS;
constexpr int WARPS = EPI_WARP0 + 4;
constexpr int THREADS = WARPS * 32;
constexpr int MAX_TILES = 4096;  // tiles of a call (P <= 65536 slots)
constexpr int ACC_COLS = 2 * NMAX;
constexpr int W_STAGE = BM * SUBK * 2;    // 16 KB
constexpr int A_STAGE = NMAX * SUBK * 2;  // 16 KB

__host__ __device__ constexpr int chunk_bytes(int kind) {
  return CHK / block_info(kind).per_block * block_info(kind).block_bytes;
}
// a row's chunk starts anywhere on an even byte; its 16-byte aligned cover is at most this long
__host__ __device__ constexpr int slot_bytes(int kind) { return align16(chunk_bytes(kind) + 15); }

struct Layout {
  int w, a, raw, tabs, groups, bars, total, raw_stages;
};

__host__ __device__ constexpr Layout layout(int kind, int raw_stages) {
  Layout l{};
  l.raw_stages = raw_stages;
  l.w = 0;
  l.a = l.w + STAGES * W_STAGE;
  l.raw = l.a + STAGES * A_STAGE;
  l.tabs = l.raw + raw_stages * BM * slot_bytes(kind);
  l.groups = align16(l.tabs + table_bytes(kind) + 8);
  l.bars = l.groups + MAX_TILES * 4;
  l.total = l.bars + 256 + 1024;  // barriers and scratch, plus the slack to align the base to 1024 bytes
  return l;
}

constexpr int SMEM_LIMIT = 227 * 1024;

__host__ __device__ constexpr int raw_stages_for(int kind) {
  return layout(kind, 3).total <= SMEM_LIMIT ? 3 : 2;
}

// ---- PTX wrappers

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
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

__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
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

template <int KIND, typename T>
__global__ void __launch_bounds__(THREADS, 1)
    tile_mma_kernel(const __grid_constant__ CUtensorMap amap, const uint8_t* __restrict__ blocks, int experts, int rows,
                    int cols, int64_t rbytes, int P, const uint32_t* __restrict__ tile_expert, float* __restrict__ c,
                    int* err, int raw_stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = layout(KIND, raw_stages);
  constexpr int SLOT = slot_bytes(KIND), CB = chunk_bytes(KIND);
  uint8_t* wst = smem + L.w;
  uint8_t* ast = smem + L.a;
  uint8_t* raw = smem + L.raw;
  uint32_t* groups = reinterpret_cast<uint32_t*>(smem + L.groups);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* full = bars;                  // [STAGES]: 8 decoder warps + the producer's expect_tx
  uint64_t* empty = full + STAGES;        // [STAGES]: the MMAs of the stage
  uint64_t* raw_full = empty + STAGES;    // [3]: the bulk copies
  uint64_t* raw_empty = raw_full + 3;     // [3]: 8 decoder warps
  uint64_t* acc_full = raw_empty + 3;     // [2]: the item's MMAs
  uint64_t* acc_empty = acc_full + 2;     // [2]: 4 epilogue warps
  uint64_t* done = acc_empty + 2;         // the last MMAs, before tensor memory is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* scan = reinterpret_cast<int*>(tmem_slot + 1);  // [WARPS]
  int* ngroups = scan + WARPS;
  volatile int* bail = ngroups + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Tabs tabs = load_tabs<KIND>(smem + L.tabs);
  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], DEC_WARPS + 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], DEC_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(done, 1);
    *bail = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ACC_COLS)
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
  const int RB = rows / BM, KS = cols / SUBK, KC = cols / CHK;
  const int items = *ngroups * RB;

  if (warp == 0) {
    // ---- producer
    uint32_t rc = 0, sc_ = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x) {
      const uint32_t g = groups[item / RB];
      const int r0 = (item % RB) * BM, st = int(g & 0xfff), nt = int((g >> 12) & 15) + 1, e = int(g >> 16);
      const uint8_t* wbase = blocks + (int64_t(e) * rows + r0) * rbytes;
      for (int j = 0; j < KC && ok; ++j) {
        const int rs = int(rc % uint32_t(raw_stages));
        if (!(ok = mbar_wait(&raw_empty[rs], ((rc / raw_stages) & 1) ^ 1, err))) break;
        uintptr_t from[4];
        uint32_t bytes[4], sum = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uintptr_t addr = reinterpret_cast<uintptr_t>(wbase + int64_t(lane + 32 * q) * rbytes + int64_t(j) * CB);
          from[q] = addr & ~uintptr_t(15);
          bytes[q] = uint32_t(((addr + CB + 15) & ~uintptr_t(15)) - from[q]);
          sum += bytes[q];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) mbar_arrive_expect_tx(&raw_full[rs], sum);
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 4; ++q)
          bulk_load(raw + (rs * BM + lane + 32 * q) * SLOT, reinterpret_cast<const void*>(from[q]), bytes[q],
                    &raw_full[rs]);
        ++rc;
        for (int kk = 4 * j; kk < 4 * j + 4; ++kk) {
          const int ws = int(sc_ % STAGES);
          if (!(ok = mbar_wait(&empty[ws], ((sc_ / STAGES) & 1) ^ 1, err))) break;
          if (lane == 0) {
            mbar_arrive_expect_tx(&full[ws], uint32_t(nt * TOKENS_TILE * SUBK * 2));
            for (int t = 0; t < nt; ++t)
              tma_load_2d(ast + ws * A_STAGE + t * TOKENS_TILE * 128, &amap, kk * SUBK, (st + t) * TOKENS_TILE,
                          &full[ws]);
          }
          __syncwarp();
          ++sc_;
        }
      }
    }
    if (!ok) *bail = 1;
    // in-flight copies land before the block may end: wait (briefly) for the last phase of every stage armed
    for (uint32_t i = rc > uint32_t(raw_stages) ? rc - raw_stages : 0; i < rc; ++i)
      mbar_wait(&raw_full[i % raw_stages], (i / raw_stages) & 1, nullptr, 20000000LL);
    for (uint32_t i = sc_ > uint32_t(STAGES) ? sc_ - STAGES : 0; i < sc_; ++i)
      mbar_wait(&full[i % STAGES], (i / STAGES) & 1, nullptr, 20000000LL);
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      uint32_t sc_ = 0, ic = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x, ++ic) {
        const uint32_t g = groups[item / RB];
        const int nt = int((g >> 12) & 15) + 1;
        const int b = int(ic & 1);
        if (!(ok = mbar_wait(&acc_empty[b], ((ic >> 1) & 1) ^ 1, err))) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(b * NMAX);
        const uint32_t idesc = instr_desc<T>(nt * TOKENS_TILE);
        for (int kk = 0; kk < KS; ++kk) {
          const int ws = int(sc_ % STAGES);
          if (!(ok = mbar_wait(&full[ws], (sc_ / STAGES) & 1, err))) break;
          tc_fence_after();
          const uint64_t ad = smem_desc(wst + ws * W_STAGE), bd = smem_desc(ast + ws * A_STAGE);
#pragma unroll
          for (int k = 0; k < SUBK / 16; ++k) mma_f16(d, ad + 2 * k, bd + 2 * k, idesc, (kk | k) != 0);
          mma_commit(&empty[ws]);
          ++sc_;
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      if (!ok) *bail = 1;
      mma_commit(done);  // arrives once every MMA this thread issued has finished
      mbar_wait(done, 0, nullptr, 20000000LL);
    }
    __syncwarp();
  } else if (warp < EPI_WARP0) {
    // ---- decoders: thread dt takes row dt % 128 and the run dt / 128 of each 64-column slice
    const int dt = tid - 64, m = dt % BM, half = dt / BM;
    const int r8 = m & 7;
    uint8_t* wrow = wst + (m >> 3) * 1024 + r8 * 128;
    uint32_t rc = 0, sc_ = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x) {
      const uint32_t g = groups[item / RB];
      const int r0 = (item % RB) * BM, e = int(g >> 16);
      const uint8_t* wsrc = blocks + (int64_t(e) * rows + r0 + m) * rbytes;
      for (int kk = 0; kk < KS; ++kk) {
        const int j = kk / 4, q = kk % 4;
        const int rs = int(rc % uint32_t(raw_stages));
        if (q == 0 && !(ok = mbar_wait(&raw_full[rs], (rc / raw_stages) & 1, err))) break;
        const int ws = int(sc_ % STAGES);
        if (!(ok = mbar_wait(&empty[ws], ((sc_ / STAGES) & 1) ^ 1, err))) break;
        const int s = int(reinterpret_cast<uintptr_t>(wsrc + int64_t(j) * CB) & 15);
        float w[32];
        unpack32<KIND>(raw + (rs * BM + m) * SLOT + s, 2 * q + half, w, tabs);
        uint8_t* dst = wrow + ws * W_STAGE;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int chunk = half * 4 + i;
          uint4 v;
          v.x = pack2<T>(w[8 * i + 0], w[8 * i + 1]);
          v.y = pack2<T>(w[8 * i + 2], w[8 * i + 3]);
          v.z = pack2<T>(w[8 * i + 4], w[8 * i + 5]);
          v.w = pack2<T>(w[8 * i + 6], w[8 * i + 7]);
          *reinterpret_cast<uint4*>(dst + ((chunk ^ r8) << 4)) = v;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[ws]);
        ++sc_;
        if (q == 3) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[rs]);
          ++rc;
        }
      }
    }
    if (!ok) *bail = 1;
  } else {
    // ---- epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31, the item's rows r0 + 32 (w % 4) + lane
    const int quarter = warp & 3;
    uint32_t ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok && !*bail; item += gridDim.x, ++ic) {
      const uint32_t g = groups[item / RB];
      const int r0 = (item % RB) * BM, st = int(g & 0xfff), nt = int((g >> 12) & 15) + 1;
      const int b = int(ic & 1);
      if (!(ok = mbar_wait(&acc_full[b], (ic >> 1) & 1, err))) break;
      tc_fence_after();
      const int row = r0 + 32 * quarter + lane;
      float* out = c + int64_t(st) * TOKENS_TILE * rows + row;
      for (int n0 = 0; n0 < nt * TOKENS_TILE; n0 += 16) {
        float v[16];
        tmem_ld16(tmem + (uint32_t(32 * quarter) << 16) + uint32_t(b * NMAX + n0), v);
#pragma unroll
        for (int i = 0; i < 16; ++i) out[int64_t(n0 + i) * rows] = v[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (!ok) *bail = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ACC_COLS) : "memory");
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

template <int KIND, typename T>
int launch(const uint8_t* blocks, int experts, int rows, int cols, int64_t rb, const void* a, int P,
           const uint32_t* tile_expert, float* c, int* err, cudaStream_t s) {
  EncodeTiled enc = encode_tiled();
  if (!enc) return SC_ERR_CUDA;
  CUtensorMap map;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(P)};
  const cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  const cuuint32_t box[2] = {SUBK, TOKENS_TILE};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      std::is_same_v<T, __nv_bfloat16> ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (enc(&map, dt, 2, const_cast<void*>(a), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return SC_ERR_CUDA;
  constexpr int RS = raw_stages_for(KIND);
  constexpr int smem = layout(KIND, RS).total;
  static_assert(smem <= SMEM_LIMIT, "tile_mma shared memory");
  auto kern = tile_mma_kernel<KIND, T>;
  static bool set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return SC_ERR_CUDA;
  if (!set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return SC_ERR_CUDA;
    set[dev] = true;
  }
  const int grid = sm_count();
  if (grid <= 0) return SC_ERR_CUDA;
  kern<<<grid, THREADS, smem, s>>>(map, blocks, experts, rows, cols, rb, P, tile_expert, c, err, RS);
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

}  // namespace tm

bool tile_mma_takes(int kind, int experts, int rows, int cols, int a_dtype, int P, const void* a, const void* blocks) {
  return (a_dtype == SC_F16 || a_dtype == SC_BF16) && block_info(kind).per_block && rows % tm::BM == 0 &&
         cols % tm::CHK == 0 && P / TOKENS_TILE <= tm::MAX_TILES && experts <= 65535 &&
         reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(blocks) % 16 == 0;
}

int tile_mma_launch(int kind, const uint8_t* blocks, int experts, int rows, int cols, int64_t rbytes, const void* a,
                    int a_dtype, int P, const uint32_t* tile_expert, float* c, int* err, cudaStream_t s) {
  if (!tile_mma_takes(kind, experts, rows, cols, a_dtype, P, a, blocks)) return SC_ERR_UNSUPPORTED;
  int rc = SC_ERR_UNSUPPORTED;
  dispatch_kind(kind, [&]<int KIND>() {
    if (a_dtype == SC_BF16)
      rc = tm::launch<KIND, __nv_bfloat16>(blocks, experts, rows, cols, rbytes, a, P, tile_expert, c, err, s);
    else
      rc = tm::launch<KIND, __half>(blocks, experts, rows, cols, rbytes, a, P, tile_expert, c, err, s);
  });
  return rc;
}

}  // namespace sc
