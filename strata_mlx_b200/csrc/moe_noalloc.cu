// sc_moe_decode_layer_noalloc: the decode MoE block for callers that cannot allocate device memory.
//
// A caller with a fixed memory plan (a serving process that owns all device memory from start-up), or a binding
// from a language without a CUDA allocator, passes only the inputs and the output. The scratch the block needs
// (routes, logits, the experts' inner activations and outputs) comes from a static device array of this file,
// SC_NOALLOC_SCRATCH_BYTES long, instead of a caller-owned workspace. Nothing here calls an allocator: the array
// exists for as long as the library is loaded on a device, and the work is sc_moe_decode_layer's, unchanged.
#include <mutex>

#include "common.cuh"

namespace {

// The scratch of every call on a device. Calls share it: the decode layer clears its error word and logits
// at the start of each call; calls whose work overlaps on the GPU race on it.
__device__ __align__(256) uint8_t g_noalloc_scratch[SC_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
void* g_scratch[kMaxDevices] = {};

// The array's device address on the current device, looked up once per device (with that device current).
// Host code cannot use the symbol itself: on the host it names a stand-in, not device memory.
void* scratch_address(int device) {
  std::lock_guard<std::mutex> hold(g_lock);
  if (!g_scratch[device]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
      cudaGetLastError();  // take the (non-sticky) error off the thread, so that the next call may try again
      return nullptr;
    }
    g_scratch[device] = p;
  }
  return g_scratch[device];
}

}  // namespace

extern "C" int sc_moe_decode_layer_noalloc(const sc_moe_layer* layer, const void* x, int tokens, void* out,
                                           void* stream) {
  if (!layer || !x || !out) return SC_ERR_ARG;
  const size_t need = sc_moe_decode_workspace(layer, tokens);
  if (need == 0) return SC_ERR_SHAPE;  // a layer or token count sc_moe_decode_layer does not take
  if (need > SC_NOALLOC_SCRATCH_BYTES) return SC_ERR_SCRATCH;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0) return SC_ERR_CUDA;
  if (device >= kMaxDevices) return SC_ERR_UNSUPPORTED;
  void* scratch = scratch_address(device);
  if (!scratch) return SC_ERR_CUDA;
  return sc_moe_decode_layer(layer, x, tokens, out, scratch, SC_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int sc_moe_decode_noalloc_error(int* code, void* stream) {
  if (!code) return SC_ERR_ARG;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0) return SC_ERR_CUDA;
  if (device >= kMaxDevices) return SC_ERR_UNSUPPORTED;
  void* scratch = scratch_address(device);
  if (!scratch) return SC_ERR_CUDA;
  // the error word is the scratch's first int (the decode block's workspace layout puts it at offset 0)
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int word = 0;
  if (cudaMemcpyAsync(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return SC_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return SC_ERR_CUDA;
  if (word != 0 && cudaMemsetAsync(scratch, 0, sizeof(int), s) != cudaSuccess) return SC_ERR_CUDA;
  *code = word;
  return SC_OK;
}
