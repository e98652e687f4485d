// Paged grouped-query attention for the synthetic decoder around the MoE blocks (the decode and verify passes of
// BASELINE configurations 4 and 5): a window of T_q (1..8) new tokens of one sequence against its key/value cache
// held in pages of 16 tokens. Not the hot path of this library -- the MoE expert products are -- but the decoder
// needs it at 8K and 128K contexts, where reading the cache once is what the pass costs.
//
//   sc_paged_attention  flash-decoding: the context is cut into about 148 chunks a key/value head (whole pages, so
//                       that every SM has a block at 8K and 128K alike); a block per (chunk, key/value head) takes
//                       the 8 query heads of its group times the window as up to 64 rows,
//                       streams the chunk's pages through shared memory (cp.async, three stages), and keeps an online
//                       softmax: scores and the value product on mma.sync (bf16, f32 sums), probabilities rounded
//                       to bf16 for the value product. A second kernel, launched as its programmatic dependent,
//                       merges the chunks' partial results.
//
// Query token i sits at position ctx_len - T_q + i and sees keys 0 .. its position (the window's own keys included:
// they are in the cache before the call).
#include <algorithm>

#include "common.cuh"
#include "mma_decode.cuh"

namespace sc {
namespace at {

constexpr int D = 256;         // head dimension
constexpr int PAGE = 16;       // tokens a page
constexpr int GQA = 8;         // query heads a key/value head (16 / 2)
constexpr int MAXROWS = 64;    // GQA x 8 tokens
constexpr int WARPS = 8;       // warp w: query tile w / 2 (16 rows), dimension half w % 2 (128 dims)
constexpr int NST = 3;         // pipeline stages of (K page, V page)
constexpr int QSTRIDE = D + 8;  // bf16 elements a row of Q in shared memory (padded: no bank conflicts)
constexpr int KSTRIDE = D + 8;

struct Args {
  const __nv_bfloat16 *q, *k, *v;  // q (T_q, Hq, D); k, v (pages, PAGE, Hkv, D)
  const int32_t* table;            // the sequence's pages
  const int32_t* ctx_dev;          // tokens in the cache, read on the device
  int Tq, Hq, Hkv, chunks;         // chunks: of the largest context the call allows
  int cpages;                      // pages a chunk
  float scale_log2;                // softmax scale times log2(e)
  float* opart;                    // (chunks, Hkv, MAXROWS, D) unnormalized outputs
  float* mpart;                    // (chunks, Hkv, MAXROWS) running maxima (log2 domain)
  float* lpart;                    // (chunks, Hkv, MAXROWS) sums
  __nv_bfloat16* out;              // (T_q, Hq, D)
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&r);
}


__global__ void __launch_bounds__(WARPS * 32) attn_kernel(const Args A) {
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem);                     // (MAXROWS, QSTRIDE)
  __nv_bfloat16* ks = qs + MAXROWS * QSTRIDE;                                    // (NST, PAGE, KSTRIDE)
  __nv_bfloat16* vs = ks + NST * PAGE * KSTRIDE;                                 // (NST, PAGE, KSTRIDE)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int chunk = blockIdx.x, hk = blockIdx.y;
  const int rows = GQA * A.Tq, mtiles = (rows + 15) / 16;
  const int ctx = *A.ctx_dev;
  const int k0 = chunk * A.cpages * PAGE, k1 = min(ctx, k0 + A.cpages * PAGE);
  const int pages = k1 > k0 ? (k1 - k0 + PAGE - 1) / PAGE : 0;
  pdl_launch_dependents();  // the merge's blocks may be placed as this grid's blocks leave
  // Q rows: row r = token (r / GQA), query head hk * GQA + r % GQA
  for (int i = tid; i < MAXROWS * (D / 8); i += blockDim.x) {
    const int r = i / (D / 8), c = (i % (D / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < rows) v = *reinterpret_cast<const uint4*>(A.q + (int64_t(r / GQA) * A.Hq + hk * GQA + r % GQA) * D + c);
    *reinterpret_cast<uint4*>(qs + r * QSTRIDE + c) = v;
  }
  auto load_page = [&](int p, int st) {  // page p of the chunk into stage st: its 16 keys and values of head hk
    const int page = A.table[(k0 / PAGE) + p];
    for (int i = tid; i < 2 * PAGE * (D / 8); i += blockDim.x) {
      const int kv = i / (PAGE * (D / 8)), j = (i / (D / 8)) % PAGE, c = (i % (D / 8)) * 8;
      const __nv_bfloat16* src = (kv ? A.v : A.k) + ((int64_t(page) * PAGE + j) * A.Hkv + hk) * D + c;
      __nv_bfloat16* dst = (kv ? vs : ks) + (st * PAGE + j) * KSTRIDE + c;
      cp_async16(dst, src);
    }
  };
  for (int p = 0; p < NST - 1; ++p) {
    if (p < pages) load_page(p, p);
    cp_commit();
  }
  const int mt = warp >> 1, dh = warp & 1;
  const bool active = mt < mtiles;
  // the rows this lane's fragments hold and their positions
  const int ra = mt * 16 + g, rb = ra + 8;
  const int pa = ctx - A.Tq + min(ra, rows - 1) / GQA, pb = ctx - A.Tq + min(rb, rows - 1) / GQA;
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float ma = -1e30f, mb = -1e30f, la = 0.f, lb = 0.f;
  for (int p = 0; p < pages; ++p) {
    if (p + NST - 1 < pages) load_page(p + NST - 1, (p + NST - 1) % NST);
    cp_commit();
    cp_wait<NST - 1>();
    __syncthreads();
    const int st = p % NST;
    if (active) {
      const __nv_bfloat16* kp = ks + st * PAGE * KSTRIDE;
      const __nv_bfloat16* vp = vs + st * PAGE * KSTRIDE;
      // scores of 16 rows x 16 keys: two n-tiles of 8 keys
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
      for (int kk = 0; kk < D / 16; ++kk) {
        const __nv_bfloat16* q0 = qs + (mt * 16 + g) * QSTRIDE + kk * 16 + 2 * t;
        const uint32_t a[4] = {*reinterpret_cast<const uint32_t*>(q0), *reinterpret_cast<const uint32_t*>(q0 + 8 * QSTRIDE),
                               *reinterpret_cast<const uint32_t*>(q0 + 8), *reinterpret_cast<const uint32_t*>(q0 + 8 * QSTRIDE + 8)};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const __nv_bfloat16* kr = kp + (8 * j + g) * KSTRIDE + kk * 16 + 2 * t;
          mma16816<__nv_bfloat16>(s[j], a, *reinterpret_cast<const uint32_t*>(kr),
                                  *reinterpret_cast<const uint32_t*>(kr + 8));
        }
      }
      // mask, the block's maxima, the online softmax's rescale
      const int kbase = k0 + p * PAGE;
      float bma = -1e30f, bmb = -1e30f;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kbase + 8 * j + 2 * t + e;
          s[j][e] = (ra < rows && key <= pa && key < ctx) ? s[j][e] * A.scale_log2 : -1e30f;
          s[j][2 + e] = (rb < rows && key <= pb && key < ctx) ? s[j][2 + e] * A.scale_log2 : -1e30f;
          bma = fmaxf(bma, s[j][e]);
          bmb = fmaxf(bmb, s[j][2 + e]);
        }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, off));
        bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, off));
      }
      const float na = fmaxf(ma, bma), nb = fmaxf(mb, bmb);
      const float ca = exp2f(ma - na), cb = exp2f(mb - nb);
      ma = na;
      mb = nb;
      la *= ca;
      lb *= cb;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        o[i][0] *= ca; o[i][1] *= ca; o[i][2] *= cb; o[i][3] *= cb;
      }
      float pr[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        pr[j][0] = s[j][0] > -1e29f ? exp2f(s[j][0] - na) : 0.f;
        pr[j][1] = s[j][1] > -1e29f ? exp2f(s[j][1] - na) : 0.f;
        pr[j][2] = s[j][2] > -1e29f ? exp2f(s[j][2] - nb) : 0.f;
        pr[j][3] = s[j][3] > -1e29f ? exp2f(s[j][3] - nb) : 0.f;
        la += pr[j][0] + pr[j][1];
        lb += pr[j][2] + pr[j][3];
      }
      // probabilities as the A operand (16 rows x 16 keys), values through ldmatrix.trans
      const uint32_t pa4[4] = {pack_bf16(pr[0][0], pr[0][1]), pack_bf16(pr[0][2], pr[0][3]), pack_bf16(pr[1][0], pr[1][1]),
                               pack_bf16(pr[1][2], pr[1][3])};
#pragma unroll
      for (int i = 0; i < 16; i += 2) {  // dims dh * 128 + 8 i .. + 16
        const int d0 = dh * 128 + 8 * i;
        const __nv_bfloat16* vr = vp + ((lane & 7) + ((lane >> 3) & 1) * 8) * KSTRIDE + d0 + (lane >> 4) * 8;
        uint32_t b[4];
        ldsm_x4_trans(b, vr);
        mma16816<__nv_bfloat16>(o[i], pa4, b[0], b[1]);
        mma16816<__nv_bfloat16>(o[i + 1], pa4, b[2], b[3]);
      }
    }
    __syncthreads();  // the stage is refilled next round
  }
  cp_wait<0>();
  if (!active) return;
  // the sums across the quad; partial results of this chunk
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);
  const int64_t base = (int64_t(chunk) * A.Hkv + hk) * MAXROWS;
  if (t == 0 && dh == 0) {
    if (ra < rows) { A.mpart[base + ra] = ma; A.lpart[base + ra] = la; }
    if (rb < rows) { A.mpart[base + rb] = mb; A.lpart[base + rb] = lb; }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int d = dh * 128 + 8 * i + 2 * t;
    if (ra < rows) *reinterpret_cast<float2*>(A.opart + (base + ra) * D + d) = make_float2(o[i][0], o[i][1]);
    if (rb < rows) *reinterpret_cast<float2*>(A.opart + (base + rb) * D + d) = make_float2(o[i][2], o[i][3]);
  }
}

// out[token, head, d] = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c over the chunks c: a block per (row, head,
// 32 dimensions), eight groups of 32 threads (a dimension each) taking every eighth chunk, so that the grid covers
// many SMs and many loads are in flight. It waits for the attention kernel's partial results before reading them.
constexpr int MERGE_DIMS = 32;
constexpr int MERGE_GROUPS = 8;

__global__ void __launch_bounds__(MERGE_GROUPS * MERGE_DIMS) merge_kernel(const Args A) {
  __shared__ float s_w[1024], s_num[MERGE_GROUPS][MERGE_DIMS], s_den[MERGE_GROUPS];
  const int row = blockIdx.x, hk = blockIdx.y, grp = threadIdx.x / MERGE_DIMS;
  const int d = blockIdx.z * MERGE_DIMS + threadIdx.x % MERGE_DIMS;
  pdl_wait();
  const int rows = GQA * A.Tq;
  if (row >= rows) return;
  const int ctx = *A.ctx_dev;
  const int chunks = min(A.chunks, (ctx + A.cpages * PAGE - 1) / (A.cpages * PAGE));  // later blocks wrote nothing
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) s_w[c] = A.mpart[(int64_t(c) * A.Hkv + hk) * MAXROWS + row];
  __syncthreads();
  float M = -1e30f;
  for (int c = 0; c < chunks; ++c) M = fmaxf(M, s_w[c]);  // a broadcast read of shared memory
  __syncthreads();
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) s_w[c] = exp2f(s_w[c] - M);
  __syncthreads();
  float num = 0.f, den = 0.f;
#pragma unroll 8
  for (int c = grp; c < chunks; c += MERGE_GROUPS) {
    const int64_t b = (int64_t(c) * A.Hkv + hk) * MAXROWS + row;
    num += s_w[c] * A.opart[b * D + d];
    den += s_w[c] * A.lpart[b];
  }
  s_num[grp][threadIdx.x % MERGE_DIMS] = num;
  if (threadIdx.x % MERGE_DIMS == 0) s_den[grp] = den;
  __syncthreads();
  if (grp == 0) {
    float n = 0.f, dd = 0.f;
#pragma unroll
    for (int g = 0; g < MERGE_GROUPS; ++g) {
      n += s_num[g][threadIdx.x % MERGE_DIMS];
      dd += s_den[g];
    }
    A.out[(int64_t(row / GQA) * A.Hq + hk * GQA + row % GQA) * D + d] = __float2bfloat16_rn(dd > 0.f ? n / dd : 0.f);
  }
}

// chunks of whole pages: about 148 a head (one block an SM over the heads' grid), at most 1024
inline void chunking(int max_ctx, int kv_heads, int& cpages, int& chunks) {
  const int pages = (max_ctx + PAGE - 1) / PAGE;
  const int want = std::max(1, (2 * 148 + kv_heads - 1) / kv_heads);
  cpages = std::max(1, (pages + want - 1) / want);
  chunks = (pages + cpages - 1) / cpages;
}

}  // namespace at
}  // namespace sc

using namespace sc;

extern "C" size_t sc_paged_attention_workspace(int ctx, int kv_heads) {
  if (ctx < 1 || kv_heads < 1) return 0;
  int cpages, chunks;
  at::chunking(ctx, kv_heads, cpages, chunks);
  const size_t n = size_t(chunks) * size_t(kv_heads) * at::MAXROWS;
  return n * at::D * 4 + 2 * n * 4 + 256;
}

extern "C" int sc_paged_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                                  const int32_t* ctx_dev, int max_ctx, int tokens, int q_heads, int kv_heads,
                                  int head_dim, float scale, void* out, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  if (!q || !k_cache || !v_cache || !block_table || !ctx_dev || !out || !workspace) return SC_ERR_ARG;
  if (head_dim != at::D || q_heads != at::GQA * kv_heads || tokens < 1 || tokens > 8 || max_ctx < tokens)
    return SC_ERR_SHAPE;
  const int ctx = max_ctx;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(workspace)) & 15)
    return SC_ERR_ALIGN;
  if (workspace_bytes < sc_paged_attention_workspace(ctx, kv_heads)) return SC_ERR_WORKSPACE;
  at::Args A{};
  A.q = static_cast<const __nv_bfloat16*>(q);
  A.k = static_cast<const __nv_bfloat16*>(k_cache);
  A.v = static_cast<const __nv_bfloat16*>(v_cache);
  A.table = block_table;
  A.ctx_dev = ctx_dev;
  A.Tq = tokens;
  A.Hq = q_heads;
  A.Hkv = kv_heads;
  at::chunking(ctx, kv_heads, A.cpages, A.chunks);
  if (A.chunks > 1024) return SC_ERR_SHAPE;
  A.scale_log2 = scale * 1.4426950408889634f;
  const size_t n = size_t(A.chunks) * size_t(kv_heads) * at::MAXROWS;
  A.opart = static_cast<float*>(workspace);
  A.mpart = A.opart + n * at::D;
  A.lpart = A.mpart + n;
  A.out = static_cast<__nv_bfloat16*>(out);
  const int smem = (at::MAXROWS * at::QSTRIDE + 2 * at::NST * at::PAGE * at::KSTRIDE) * 2;
  if (int rc = raise_smem(reinterpret_cast<const void*>(at::attn_kernel), smem, "attention smem attribute")) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  at::attn_kernel<<<dim3(A.chunks, kv_heads), at::WARPS * 32, smem, s>>>(A);
  {  // programmatic dependent launch: no gap between the two kernels
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(at::GQA * tokens), unsigned(kv_heads), unsigned(at::D / at::MERGE_DIMS));
    cfg.blockDim = dim3(at::MERGE_GROUPS * at::MERGE_DIMS);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaError_t e = cudaLaunchKernelEx(&cfg, at::merge_kernel, A))
      return cuda_failed(e, "attention merge launch");
  }
  if (cudaError_t e = cudaGetLastError()) return cuda_failed(e, "attention launch");
  return SC_OK;
}
