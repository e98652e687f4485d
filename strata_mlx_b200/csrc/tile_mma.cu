// The tcgen05 tile product: placeholder until the tensor-core kernel lands; every call goes to the CUDA cores.
#include "tiles.cuh"

namespace sc {

int tile_mma_launch(int, const uint8_t*, int, int, int, int64_t, const void*, int, int, const uint32_t*, float*,
                    cudaStream_t) {
  return SC_ERR_UNSUPPORTED;
}

}  // namespace sc
