// Expert parallel decode over peer memory (no counterpart in strata-mlx, which runs on one device): the kernels
// around the fused decode block that replace the collectives, and the CUDA IPC calls that map the ranks' exchange
// buffers into each other (layout and counters in ep.cuh).
//
//   ep_feed_kernel     a step's first window: this rank's tokens into every rank's X[0], then a count there
//   ep_combine_kernel  moe_combine of this rank's tokens (strata_mlx/fused.py:467-481, the fixed add order) from
//                      the words of Y[p] tagged with this call's step, into `out`, and, unless the layer is the
//                      chain's last, into every rank's X[p ^ 1] with a count there
// Every wait is bounded (ep::wait_count); a rank that never writes makes the others record SC_ERR_TIMEOUT and go on.
#include <cuda.h>

#include <cstring>

#include "decode.cuh"
#include "decode_layer.cuh"
#include "ep.cuh"
#include "route.cuh"

namespace sc {
namespace ep {

// Event stamps for a profiling build (-DSC_TRACE): %globaltimer per combine block and phase. Compiled out otherwise.
#ifdef SC_TRACE
__device__ unsigned long long g_eptrace[64][4];
#define EP_TRACE(p)                                                                     \
  do {                                                                                  \
    if (threadIdx.x == 0 && blockIdx.x < 64)                                            \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g_eptrace[blockIdx.x][p]));     \
  } while (0)
#else
#define EP_TRACE(p) \
  do {              \
  } while (0)
#endif

template <typename T>
__global__ void __launch_bounds__(256) ep_feed_kernel(EpArgs A) {
  const size_t xo = xoff(0, A.T, A.H);
  const int n = A.tl * A.H, n8 = n / 8;  // eight values (16 bytes) a store; hidden sizes are multiples of 256
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(A.x)[i];
    for (int g = 0; g < A.G; ++g)
      reinterpret_cast<uint4*>(reinterpret_cast<T*>(A.peers[g] + xo) + int64_t(A.rank) * n)[i] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_release_sys();
    for (int g = 0; g < A.G; ++g) count_relaxed(at_u32(A.peers[g], xcount_off(0)));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ep_combine_kernel(EpArgs A) {
  // Launched as a programmatic dependent of this rank's down kernel, with no wait on it: the words of Y carry the
  // step of the call that wrote them (the pairs' ranks' down kernels), and this rank's down kernel counts its
  // blocks once their shared expert outputs (local) are written; the routes were written before that.
  pdl_launch_dependents();  // the next layer's route kernel may load its weights now
  const uint64_t own = A.peers[A.rank];
  EP_TRACE(0);
  // the window's count of this layer: its route and gate/up kernels are done with it (they ran before this rank's
  // down kernel, which launched this one); no rank counts window p again before this rank's combine counted the
  // next window, below
  if (threadIdx.x == 0 && blockIdx.x == 0) *at_u32(own, xcount_off(A.par)) = 0;
  __shared__ uint32_t s_step;
  if (threadIdx.x == 0) {
    // the step is final: the route kernel counted it before the down kernel, which launched this one, started
    const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(A.step);
    s_step = step;
    // every down block of this call has written its rows (a monotonic count: dn_blocks a call)
    wait_count(A.done, step * A.dn_blocks, A.err);
  }
  __syncthreads();
  const uint32_t step = s_step;
  EP_TRACE(1);
  const uint64_t* y = reinterpret_cast<const uint64_t*>(own + yoff(A.par, A.T, A.tl, A.K, A.H));
  const size_t xo = xoff(A.par ^ 1, A.T, A.H);
  const int n = A.tl * A.H, n4 = n / 4;
  // four outputs a thread: every pair's two tagged words loaded at once, then checked (and waited for, rarely);
  // groups of four dealt over the blocks in turn, so that every block has a share of a small window
  for (int i = blockIdx.x + gridDim.x * threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
    const int j = (4 * i) / A.H, c = (4 * i) % A.H, tok = A.rank * A.tl + j;
    uint64_t w0[TOPK_MAX_K], w1[TOPK_MAX_K];
#pragma unroll
    for (int k = 0; k < TOPK_MAX_K; ++k)
      if (k < A.K) load_words2(y + (int64_t(j) * A.K + k) * (A.H / 2) + c / 2, w0[k], w1[k]);
    uint32_t yv[TOPK_MAX_K][2];
#pragma unroll
    for (int k = 0; k < TOPK_MAX_K; ++k)
      if (k < A.K) {
        const uint64_t* wk = y + (int64_t(j) * A.K + k) * (A.H / 2) + c / 2;
        yv[k][0] = uint32_t(w0[k] >> 32) == step ? uint32_t(w0[k]) : wait_tagged(wk, step, A.err);
        yv[k][1] = uint32_t(w1[k] >> 32) == step ? uint32_t(w1[k]) : wait_tagged(wk + 1, step, A.err);
      }
    uint2 sraw = make_uint2(0, 0);
    if (A.Is > 0) sraw = *reinterpret_cast<const uint2*>(static_cast<const T*>(A.sout) + int64_t(tok) * A.H + c);
    const float gv = A.Is > 0 ? round_to<T>(A.gsh[tok]) : -INFINITY;
    uint2 ov;
    T* o = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float yk[TOPK_MAX_K];
#pragma unroll
      for (int k = 0; k < TOPK_MAX_K; ++k)
        if (k < A.K) yk[k] = to_f32(reinterpret_cast<const T*>(&yv[k][q >> 1])[q & 1]);
      const float sv = A.Is > 0 ? to_f32(reinterpret_cast<const T*>(&sraw)[q]) : 0.f;
      o[q] = from_f32<T>(combine_one<T>(yk, A.wts + tok * A.K, A.K, gv, sv));
    }
    reinterpret_cast<uint2*>(A.out)[i] = ov;
    if (!A.last)
      for (int g = 0; g < A.G; ++g)
        reinterpret_cast<uint2*>(reinterpret_cast<T*>(A.peers[g] + xo) + int64_t(A.rank) * n)[i] = ov;
  }
  __syncthreads();
  if (!A.last && threadIdx.x == 0) {
    fence_release_sys();
    for (int g = 0; g < A.G; ++g) count_relaxed(at_u32(A.peers[g], xcount_off(A.par ^ 1)));
  }
  EP_TRACE(2);
}

int feed_launch(const EpArgs& A, int dtype, cudaStream_t s) {
  bool ok = dispatch_dtype(dtype, [&]<typename T>() { ep_feed_kernel<T><<<COMBINE_BLOCKS, 256, 0, s>>>(A); });
  if (!ok) return SC_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

int combine_launch(const EpArgs& A, int dtype, cudaStream_t s) {
  cudaError_t e = cudaSuccess;
  bool ok = dispatch_dtype(dtype, [&]<typename T>() {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(COMBINE_BLOCKS);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, ep_combine_kernel<T>, A);
  });
  if (!ok) return SC_ERR_DTYPE;
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

}  // namespace ep
}  // namespace sc

using namespace sc;

#ifdef SC_TRACE
extern "C" SC_API void sc_eptrace_read(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, ep::g_eptrace, sizeof(ep::g_eptrace));
}
#endif

// ---- CUDA IPC: a rank's exchange buffer for the others to map

// cuMemGetAddressRange through the runtime's driver entry point: the library keeps no link-time dependence on
// the driver library (it loads where no driver is installed)
using AddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddressRange address_range() {
  static AddressRange fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<AddressRange>(p);
    return AddressRange(nullptr);
  }();
  return fn;
}

extern "C" int sc_ipc_handle(const void* ptr, void* handle, size_t* offset) {
  if (!ptr || !handle || !offset) return SC_ERR_ARG;
  AddressRange range = address_range();
  if (!range) return SC_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return SC_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return SC_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  *offset = size_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return SC_OK;
}

extern "C" int sc_ipc_open(const void* handle, void** base) {
  if (!handle || !base) return SC_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

extern "C" int sc_ipc_close(void* base) {
  if (!base) return SC_ERR_ARG;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? SC_OK : SC_ERR_CUDA;
}

// ---- the exchange

static int check_ex(const sc_moe_layer* L, const sc_ep_exchange* X) {
  if (!L || !X || !X->peers || !X->own) return SC_ERR_ARG;
  if (X->ranks < 1 || X->rank < 0 || X->rank >= X->ranks || X->tokens_per_rank < 1) return SC_ERR_ARG;
  if (X->ranks * X->tokens_per_rank > ROUTER_MAX_TOKENS) return SC_ERR_SHAPE;
  return SC_OK;
}

extern "C" size_t sc_ep_exchange_bytes(const sc_moe_layer* layer, int ranks, int tokens_per_rank) {
  if (!layer || ranks < 1 || tokens_per_rank < 1) return 0;
  return ep::total_bytes(ranks * tokens_per_rank, tokens_per_rank, layer->top_k, layer->hidden);
}

extern "C" int sc_ep_feed(const sc_moe_layer* layer, const sc_ep_exchange* ex, const void* x, void* stream) {
  if (int rc = check_ex(layer, ex)) return rc;
  if (!x) return SC_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) & 15) return SC_ERR_ALIGN;  // read 16 bytes at a time
  ep::EpArgs A{};
  A.peers = ex->peers;
  A.G = ex->ranks, A.rank = ex->rank, A.tl = ex->tokens_per_rank, A.T = ex->ranks * ex->tokens_per_rank;
  A.H = layer->hidden, A.K = layer->top_k, A.x = x;
  return ep::feed_launch(A, layer->dtype, static_cast<cudaStream_t>(stream));
}
