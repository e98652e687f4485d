// Prefill tile geometry (strata_mlx/blocks.py:462-463, :511-513) and the tensor-core tile product's launcher.
#pragma once

#include "common.cuh"

namespace sc {

constexpr int TOKENS_TILE = 16;  // slots of a tile (blocks.py:463 TOKENS_TILE)

// blocks.py:511-513 tileable: rows by 64, columns by 64, and rows that end on a block
inline bool tileable(int kind, int rows, int cols) {
  const BlockInfo b = block_info(kind);
  return b.per_block && rows > 0 && cols > 0 && rows % 64 == 0 && cols % 64 == 0 && cols % b.per_block == 0;
}

// The tcgen05 tile product (tile_mma.cu) for float16 / bfloat16 activations; SC_ERR_UNSUPPORTED where it
// does not take the call (tile_mma_takes false: the caller then runs the CUDA-core kernel). Bounded waits that give up record
// SC_ERR_TIMEOUT in *err (when err is not null).
// What the tile product's epilogue writes: 0 C float32 (P, rows); 1 C in A's type (P, rows); 2 C in A's type at row
// pair_of_slot[slot] of `out` (pairs, rows), nothing for slots of no pair. (A swiglu of the gate product in the up
// product's epilogue measured 2.4x slower than the plain epilogue: it runs as its own pass.)
struct TileOut {
  int mode;
  float* c;
  void* out;
  const int* pair_of_slot;
};

bool tile_mma_takes(int kind, int experts, int rows, int cols, int a_dtype, int P, const void* a, const void* blocks);
int tile_mma_launch(int kind, const uint8_t* blocks, int experts, int rows, int cols, int64_t rbytes, const void* a,
                    int a_dtype, int P, const uint32_t* tile_expert, const TileOut& o, int* err, cudaStream_t s);

}  // namespace sc
