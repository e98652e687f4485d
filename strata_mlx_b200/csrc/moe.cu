// sc_moe_decode_layer: one MoE block in decode (strata_mlx/fused.py:487-497, _Routed.__call__) for a window of
// 1..8 tokens, run as a chain of the library's kernels on one stream: router logits and the shared expert's gate,
// top-k + softmax, the routed experts' fused gate/up/swiglu, their down products, the shared expert, and the
// combine. Nothing waits on the host; the chain can be captured in a CUDA graph.
#include <algorithm>

#include <cstdlib>

#include "decode_layer.cuh"
#include "ep.cuh"
#include "matvec.cuh"
#include "route.cuh"

namespace sc {

// moe_combine with the shared expert's gate given as float32 logits, rounded to T first (the reference's gate is
// a product in the activations' type, fused.py:493)
template <typename T>
__global__ void moe_combine_kernel(const T* __restrict__ y, const float* __restrict__ w, const float* __restrict__ g,
                                   const T* __restrict__ s, int rows, int k, int d, T* __restrict__ out) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= int64_t(rows) * d) return;
  const int t = int(i / d), c = int(i % d);
  float yk[16];
  for (int q = 0; q < k; ++q) yk[q] = to_f32(y[(int64_t(t) * k + q) * d + c]);
  const float gt = g ? round_to<T>(g[t]) : -INFINITY;
  const float st = s ? to_f32(s[i]) : 0.f;
  out[i] = from_f32<T>(combine_one<T>(yk, w + int64_t(t) * k, k, gt, st));
}

// The workspace: a header both paths share (error word, ticket, logits, the shared expert's gate logits, the routes,
// the plan), then the chain's buffers or the three-kernel path's h, whichever is larger.
struct MoeWs {
  size_t err, ticket, logits, w, g, idx, plan, zeros, h, y, hs, sh, gg, gu, h2, sout, total;
};

static MoeWs moe_ws(const sc_moe_layer* L, int tokens) {
  const size_t T = size_t(tokens), K = size_t(L->top_k), E = size_t(L->experts), H = size_t(L->hidden);
  const size_t I = size_t(L->inter), Is = size_t(L->shared_inter), es = L->dtype == SC_F32 ? 4 : 2;
  MoeWs m{};
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o += (bytes + 255) & ~size_t(255); return at; };
  m.err = take(16);
  m.ticket = take(16);
  m.logits = take(T * E * 4);
  m.g = take(T * 4);
  m.idx = take(T * K * 4);
  m.w = take(T * K * 4);
  m.plan = take(sizeof(dl::Plan));
  const size_t tail = o;
  m.zeros = take(T * 4);
  m.h = take(T * K * I * es);
  m.y = take(T * K * H * es);
  m.hs = take(T * Is * es);
  m.sh = take(T * H * es);
  const bool split_gu = L->kind_gate != L->kind_up || (Is && L->kind_sgate != L->kind_sup);
  m.gg = split_gu ? take(T * K * std::max(I, Is) * es) : 0;
  m.gu = split_gu ? take(T * K * std::max(I, Is) * es) : 0;
  const size_t chain_end = o;
  o = tail;
  m.h2 = take(v2_h_bytes(L, tokens));
  m.sout = take(T * H * es);  // expert parallel: the shared expert's output
  m.total = std::max(chain_end, o);
  return m;
}

// SC_DECODE_CHAIN=1 in the environment sends every layer through the chain of single-purpose kernels (the
// reference composition), so that the two paths can be compared
static bool chain_forced() {
  const char* v = std::getenv("SC_DECODE_CHAIN");
  return v && v[0] == '1';
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int check_layer(const sc_moe_layer* L, int tokens, bool pointers = true) {
  if (!L) return SC_ERR_ARG;
  if (tokens < 1 || tokens > ROUTER_MAX_TOKENS) return SC_ERR_SHAPE;
  if (L->hidden <= 0 || L->inter <= 0 || L->experts <= 0 || L->top_k <= 0 || L->shared_inter < 0) return SC_ERR_SHAPE;
  if (L->top_k > TOPK_MAX_K || L->top_k > L->experts || L->experts > TOPK_MAX_N) return SC_ERR_SHAPE;
  if (L->dtype != SC_F16 && L->dtype != SC_BF16) return SC_ERR_DTYPE;
  if (!L->gate || !L->up || !L->down || !L->router) return SC_ERR_ARG;
  if (row_bytes(L->kind_gate, L->hidden) < 0 || row_bytes(L->kind_up, L->hidden) < 0 ||
      row_bytes(L->kind_down, L->inter) < 0)
    return block_info(L->kind_gate).per_block && block_info(L->kind_up).per_block && block_info(L->kind_down).per_block
               ? SC_ERR_SHAPE : SC_ERR_KIND;
  if (L->shared_inter) {
    if (!L->sgate || !L->sup || !L->sdown || !L->shared_gate) return SC_ERR_ARG;
    if (row_bytes(L->kind_sgate, L->hidden) < 0 || row_bytes(L->kind_sup, L->hidden) < 0 ||
        row_bytes(L->kind_sdown, L->shared_inter) < 0)
      return SC_ERR_SHAPE;
  }
  // the router rows (and the shared expert's gate) are read 16 bytes at a time on every path
  if (pointers && (!aligned16(L->router) || (L->shared_inter && !aligned16(L->shared_gate)))) return SC_ERR_ALIGN;
  return SC_OK;
}

// The fused kernels copy expert rows into shared memory with 1-D bulk copies and read the window 16 bytes at a time:
// every expert stack and the window must start on 16 bytes (the chain of single-purpose kernels takes any offset).
static bool v2_aligned(const sc_moe_layer* L, const void* x) {
  bool ok = aligned16(L->gate) && aligned16(L->up) && aligned16(L->down) && aligned16(x);
  if (L->shared_inter) ok = ok && aligned16(L->sgate) && aligned16(L->sup) && aligned16(L->sdown);
  return ok;
}

// The entry points that only the fused kernels serve: SC_ERR_UNSUPPORTED for a layer they do not take,
// SC_ERR_ALIGN for one they take at an offset they cannot copy from.
static int v2_only(const sc_moe_layer* L, const void* x, int tokens) {
  if (!v2_takes(L, tokens)) return SC_ERR_UNSUPPORTED;
  return v2_aligned(L, x) ? SC_OK : SC_ERR_ALIGN;
}

}  // namespace sc

using namespace sc;

extern "C" size_t sc_moe_decode_workspace(const sc_moe_layer* layer, int tokens) {
  if (check_layer(layer, tokens, false) != SC_OK) return 0;
  return moe_ws(layer, tokens).total;
}

extern "C" int sc_moe_decode_routes(const sc_moe_layer* layer, int tokens, size_t* idx_offset, size_t* weight_offset) {
  if (int rc = check_layer(layer, tokens, false)) return rc;
  const MoeWs m = moe_ws(layer, tokens);
  if (idx_offset) *idx_offset = m.idx;
  if (weight_offset) *weight_offset = m.w;
  return SC_OK;
}

extern "C" int sc_moe_decode_stage(const sc_moe_layer* L, const void* x, int tokens, void* out, void* workspace,
                                   size_t workspace_bytes, int stage, void* stream) {
  if (int rc = check_layer(L, tokens)) return rc;
  if (!x || !out || stage < 0 || stage > 2) return SC_ERR_ARG;
  const MoeWs m = moe_ws(L, tokens);
  if (!workspace || workspace_bytes < m.total) return SC_ERR_WORKSPACE;
  if (int rc = v2_only(L, x, tokens)) return rc;
  const V2Offsets o{m.err, m.ticket, m.logits, m.g, m.idx, m.w, m.plan, m.h2, m.sout};
  return v2_run(L, x, tokens, out, static_cast<uint8_t*>(workspace), o, static_cast<cudaStream_t>(stream), stage);
}

extern "C" int sc_moe_decode_layer_ep(const sc_moe_layer* L, const void* x, int tokens, int expert_begin,
                                      int expert_end, void* y_pairs, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  if (int rc = check_layer(L, tokens)) return rc;
  if (!x || !y_pairs) return SC_ERR_ARG;
  if (expert_begin < 0 || expert_end <= expert_begin || expert_end > L->experts) return SC_ERR_SHAPE;
  const MoeWs m = moe_ws(L, tokens);
  if (!workspace || workspace_bytes < m.total) return SC_ERR_WORKSPACE;
  if (int rc = v2_only(L, x, tokens)) return rc;
  const V2Offsets o{m.err, m.ticket, m.logits, m.g, m.idx, m.w, m.plan, m.h2, m.sout};
  V2Ep ep;
  ep.e0 = expert_begin;
  ep.e1 = expert_end;
  ep.ypairs = y_pairs;
  return v2_run(L, x, tokens, nullptr, static_cast<uint8_t*>(workspace), o, static_cast<cudaStream_t>(stream), -1, ep);
}

extern "C" int sc_moe_decode_layer_ep_p2p(const sc_moe_layer* L, const sc_ep_exchange* ex, int expert_begin,
                                          int expert_end, int parity, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  if (!ex || !ex->peers || !ex->own || ex->ranks < 1 || ex->rank < 0 || ex->rank >= ex->ranks ||
      ex->tokens_per_rank < 1 || (parity != 0 && parity != 1))
    return SC_ERR_ARG;
  const int tokens = ex->ranks * ex->tokens_per_rank;
  if (int rc = check_layer(L, tokens)) return rc;
  if (expert_begin < 0 || expert_end <= expert_begin || expert_end > L->experts) return SC_ERR_SHAPE;
  const MoeWs m = moe_ws(L, tokens);
  if (!workspace || workspace_bytes < m.total) return SC_ERR_WORKSPACE;
  const void* window = reinterpret_cast<const void*>(ex->own + ep::xoff(parity, tokens, L->hidden));
  if (int rc = v2_only(L, window, tokens)) return rc;
  const V2Offsets o{m.err, m.ticket, m.logits, m.g, m.idx, m.w, m.plan, m.h2, m.sout};
  V2Ep e;
  e.e0 = expert_begin;
  e.e1 = expert_end;
  e.peers = ex->peers;
  e.G = ex->ranks;
  e.rank = ex->rank;
  e.tl = ex->tokens_per_rank;
  e.par = parity;
  e.step = reinterpret_cast<uint32_t*>(ex->own + ep::STEP_OFF);
  e.done = reinterpret_cast<uint32_t*>(ex->own + ep::DONE_OFF);
  return v2_run(L, window, tokens, nullptr, static_cast<uint8_t*>(workspace), o, static_cast<cudaStream_t>(stream), -1,
                e);
}

extern "C" int sc_ep_combine(const sc_moe_layer* L, const sc_ep_exchange* ex, int parity, int last, void* out,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (!ex || !ex->peers || !ex->own || ex->ranks < 1 || ex->rank < 0 || ex->rank >= ex->ranks ||
      ex->tokens_per_rank < 1 || (parity != 0 && parity != 1) || !out)
    return SC_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(out) & 15) return SC_ERR_ALIGN;  // written 16 bytes at a time
  const int tokens = ex->ranks * ex->tokens_per_rank;
  if (int rc = check_layer(L, tokens)) return rc;
  const MoeWs m = moe_ws(L, tokens);
  if (!workspace || workspace_bytes < m.total) return SC_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  ep::EpArgs A{};
  A.peers = ex->peers;
  A.G = ex->ranks, A.rank = ex->rank, A.tl = ex->tokens_per_rank, A.T = tokens;
  A.H = L->hidden, A.K = L->top_k, A.Is = L->shared_inter, A.par = parity, A.last = last;
  A.wts = reinterpret_cast<const float*>(ws + m.w);
  A.gsh = reinterpret_cast<const float*>(ws + m.g);
  A.sout = ws + m.sout;
  A.out = out;
  A.err = reinterpret_cast<int*>(ws + m.err);
  A.step = reinterpret_cast<const uint32_t*>(ex->own + ep::STEP_OFF);  // counts every layer call on the buffer
  A.done = reinterpret_cast<const uint32_t*>(ex->own + ep::DONE_OFF);
  A.dn_blocks = uint32_t(L->hidden / dl::RC);
  return ep::combine_launch(A, L->dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int sc_moe_decode_combine(const sc_moe_layer* L, const void* y_pairs, int tokens, void* out,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_layer(L, tokens)) return rc;
  if (!y_pairs || !out) return SC_ERR_ARG;
  const MoeWs m = moe_ws(L, tokens);
  if (!workspace || workspace_bytes < m.total) return SC_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int T = tokens, K = L->top_k, H = L->hidden, Is = L->shared_inter;
  const int64_t n = int64_t(T) * H;
  const float* wts = reinterpret_cast<const float*>(ws + m.w);
  const float* g = reinterpret_cast<const float*>(ws + m.g);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool ok = dispatch_dtype(L->dtype, [&]<typename OutT>() {
    moe_combine_kernel<OutT><<<int(ceil_div(n, 256)), 256, 0, s>>>(
        static_cast<const OutT*>(y_pairs), wts, Is ? g : nullptr, Is ? reinterpret_cast<const OutT*>(ws + m.sout) : nullptr,
        T, K, H, static_cast<OutT*>(out));
  });
  if (!ok) return SC_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

// gate/up/swiglu of one set of experts: fused when gate and up share a block type, else two products and a swiglu
static int gate_up(int kind_g, const void* g, int kind_u, const void* u, int experts, int rows, int cols,
                   const uint32_t* idx, int pairs, int share, const void* x, int dtype, void* h, void* tmp_g,
                   void* tmp_u, int* err, void* stream) {
  if (kind_g == kind_u)
    return sc_expert_gate_up(kind_g, g, u, experts, rows, cols, idx, pairs, share, x, dtype, h, err, stream);
  if (int rc = sc_expert_matvec(kind_g, g, experts, rows, cols, idx, pairs, share, x, dtype, tmp_g, err, stream)) return rc;
  if (int rc = sc_expert_matvec(kind_u, u, experts, rows, cols, idx, pairs, share, x, dtype, tmp_u, err, stream)) return rc;
  return sc_swiglu(tmp_g, tmp_u, int64_t(pairs) * rows, dtype, h, stream);
}

extern "C" int sc_moe_decode_layer(const sc_moe_layer* L, const void* x, int tokens, void* out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  if (int rc = check_layer(L, tokens)) return rc;
  if (!x || !out) return SC_ERR_ARG;
  const MoeWs m = moe_ws(L, tokens);
  if (!workspace || workspace_bytes < m.total) return SC_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!chain_forced() && v2_takes(L, tokens) && v2_aligned(L, x)) {
    const V2Offsets o{m.err, m.ticket, m.logits, m.g, m.idx, m.w, m.plan, m.h2, m.sout};
    return v2_run(L, x, tokens, out, ws, o, s);
  }
  int* err = reinterpret_cast<int*>(ws + m.err);
  float* logits = reinterpret_cast<float*>(ws + m.logits);
  uint32_t* idx = reinterpret_cast<uint32_t*>(ws + m.idx);
  float* wts = reinterpret_cast<float*>(ws + m.w);
  float* g = reinterpret_cast<float*>(ws + m.g);
  uint32_t* zeros = reinterpret_cast<uint32_t*>(ws + m.zeros);
  const int T = tokens, K = L->top_k, E = L->experts, H = L->hidden, I = L->inter, Is = L->shared_inter;
  const int pairs = T * K;
  if (cudaMemsetAsync(ws, 0, m.idx, s) != cudaSuccess) return SC_ERR_CUDA;  // error word, ticket, logits
  if (cudaMemsetAsync(zeros, 0, size_t(T) * 4, s) != cudaSuccess) return SC_ERR_CUDA;
  if (int rc = sc_router(L->router, E, H, x, L->dtype, T, logits, stream)) return rc;
  if (Is)
    if (int rc = sc_router(L->shared_gate, 1, H, x, L->dtype, T, g, stream)) return rc;
  if (int rc = sc_top_k_softmax(logits, T, E, K, idx, wts, stream)) return rc;
  if (int rc = gate_up(L->kind_gate, L->gate, L->kind_up, L->up, E, I, H, idx, pairs, K, x, L->dtype, ws + m.h,
                       ws + m.gg, ws + m.gu, err, stream))
    return rc;
  if (int rc = sc_expert_matvec(L->kind_down, L->down, E, H, I, idx, pairs, 1, ws + m.h, L->dtype, ws + m.y, err, stream))
    return rc;
  if (Is) {
    if (int rc = gate_up(L->kind_sgate, L->sgate, L->kind_sup, L->sup, 1, Is, H, zeros, T, 1, x, L->dtype, ws + m.hs,
                         ws + m.gg, ws + m.gu, err, stream))
      return rc;
    if (int rc = sc_window_matvec(L->kind_sdown, L->sdown, H, Is, ws + m.hs, L->dtype, T, ws + m.sh, err, stream)) return rc;
  }
  const int64_t n = int64_t(T) * H;
  bool ok = dispatch_dtype(L->dtype, [&]<typename OutT>() {
    moe_combine_kernel<OutT><<<int(ceil_div(n, 256)), 256, 0, s>>>(
        reinterpret_cast<const OutT*>(ws + m.y), wts, Is ? g : nullptr, Is ? reinterpret_cast<const OutT*>(ws + m.sh) : nullptr,
        T, K, H, static_cast<OutT*>(out));
  });
  if (!ok) return SC_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}
