// Version, error strings and block-type sizes of the C ABI.
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace sc {
int cuda_failed(cudaError_t e, const char* where) {
  static const bool verbose = [] {
    const char* v = std::getenv("SC_VERBOSE");
    return v && v[0] == '1';
  }();
  if (verbose) std::fprintf(stderr, "strata_cuda: %s: %s (%s)\n", where, cudaGetErrorName(e), cudaGetErrorString(e));
  return SC_ERR_CUDA;
}

int raise_smem(const void* kern, int bytes, const char* where) {
  static std::mutex lock;
  static std::map<std::pair<int, const void*>, int> set;
  if (bytes <= 48 * 1024) return SC_OK;  // every kernel takes this much without asking
  int device = 0;
  if (cudaError_t e = cudaGetDevice(&device)) return cuda_failed(e, where);
  std::lock_guard<std::mutex> hold(lock);
  int& now = set[{device, kern}];
  if (bytes <= now) return SC_OK;
  if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))
    return cuda_failed(e, where);
  now = bytes;
  return SC_OK;
}
}  // namespace sc

using namespace sc;

extern "C" int sc_version(void) { return SC_ABI_VERSION; }

extern "C" const char* sc_error_string(int code) {
  switch (code) {
    case SC_OK: return "ok";
    case SC_ERR_KIND: return "unknown block type";
    case SC_ERR_SHAPE: return "a row does not end on a block, or a size is out of range";
    case SC_ERR_DTYPE: return "activation type not taken by this entry point";
    case SC_ERR_ALIGN: return "a pointer or size is not aligned as the entry point needs";
    case SC_ERR_ARG: return "a NULL or negative argument";
    case SC_ERR_CUDA: return "a CUDA launch failed";
    case SC_ERR_WORKSPACE: return "the workspace is too small";
    case SC_ERR_UNSUPPORTED: return "a combination this build does not take";
    case SC_ERR_TIMEOUT: return "a kernel gave up a bounded wait";
    case SC_ERR_INDEX: return "an expert id is not below the number of experts";
    case SC_ERR_SCRATCH: return "the call needs more than the library's static scratch (SC_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown error code";
  }
}

extern "C" int sc_block_info(int kind, int* per_block, int* block_bytes) {
  const BlockInfo b = block_info(kind);
  if (b.per_block == 0) return SC_ERR_KIND;
  if (per_block) *per_block = b.per_block;
  if (block_bytes) *block_bytes = b.block_bytes;
  return SC_OK;
}
