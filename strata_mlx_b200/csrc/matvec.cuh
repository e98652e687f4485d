// Expert matvec machinery shared by the decode kernels: the per-block plan (which experts the pairs name, each
// read once), the shared-memory layout, activations staged as float32, and the ring of bulk copies that streams
// expert rows from HBM into shared memory while the consumer warps decode and multiply.
#pragma once

#include "decode.cuh"

namespace sc {

constexpr int MV_WARPS = 8;                       // consumer warps
constexpr int MV_THREADS = (MV_WARPS + 1) * 32;   // + one producer warp
constexpr int MV_MAX_PAIRS = 512;                 // pairs one launch takes (the host splits larger calls)
constexpr int MV_MAX_EXPERTS = 8192;              // experts a stack may have (bitmap of 256 words)
constexpr int MV_MAX_STAGES = 8;

enum MvMode { MV_PLAIN = 0, MV_GLU_IN = 1, MV_GATEUP = 2 };

struct MvArgs {
  const uint8_t* w;             // stack base (GATEUP: the gate stack)
  const uint8_t* w2;            // GATEUP: the up stack
  const uint8_t* const* bases;  // per-pair expert buffers (matvec_separate), or nullptr
  const uint32_t* idx;          // pairs' experts, or nullptr: every pair is expert 0 (window_matvec)
  const void* x;                // PLAIN / GATEUP: (x rows, cols); GLU_IN: the gate activations (pairs, cols)
  const void* x2;               // GLU_IN: the up activations (pairs, cols)
  void* out;                    // (pairs, rows)
  int* err;
  int64_t rbytes;               // bytes of a row
  int experts, rows, cols, pairs, share, glu;
  int chunk_rows;               // rows a chunk (one bulk copy per stack) carries
  int stage_bytes;              // shared-memory bytes of a stage, a multiple of 16
  int stages;
  int lanes;                    // lanes that share a row: a power of two <= 32
};

// lanes per row: as many as leave each lane at least two runs of 32 weights (mirrors the reference's rule,
// strata_mlx/blocks.py:303-308, with a B200 warp of 32)
inline int mv_lanes(int cols) {
  int runs = cols / 32, p = 1;
  while (p < 32 && runs % (2 * p) == 0 && runs / (2 * p) >= 2) p *= 2;
  return p;
}

// shared-memory carve-up; offsets in bytes, each 16-aligned
struct MvLayout {
  int bars, tabs, bitmap, units, slots, xs, stages, total;
};

template <int KIND>
__host__ __device__ inline MvLayout mv_layout(int experts, int pairs, int xrows, int cols, int stage_bytes, int stages) {
  MvLayout L;
  int o = 0;
  L.bars = o;   o += align16(2 * MV_MAX_STAGES * 8 + 16);
  L.tabs = o;   o += align16(table_bytes(KIND) + 8);
  L.bitmap = o; o += align16(8 * ((experts + 31) / 32 + 1));  // bitmap words, then their prefix counts
  L.units = o;  o += align16(pairs * (8 + 8 + 4 + 4) + 16);   // base, base2, slot offset, count
  L.slots = o;  o += align16(pairs * 4 + 4);                  // (x row << 16 | out row) low/high 16 bits
  L.xs = o;     o += align16(xrows * cols * 4);
  L.stages = o; o += stage_bytes * stages;
  L.total = o;
  return L;
}

// x row r, run n, chunk c (16 bytes) lives at slot (c + n) % 8 of the run: lanes that read the same chunk of
// consecutive runs then hit different banks
__device__ __forceinline__ int xs_index(int r, int n, int c, int cols) { return r * cols + n * 32 + (((c + n) & 7) << 2); }

// mlx-lm's swiglu (strata_mlx/blocks.py:230-238): sigmoid in float32 from |g|, rounded to T, then g * sig and
// that times up, each rounded to T
template <typename T>
__device__ __forceinline__ float swiglu_mlx(float g, float u) {
  g = round_to<T>(g);
  u = round_to<T>(u);
  const float y = 1.0f / (1.0f + expf(fabsf(g)));
  const float sig = round_to<T>(g < 0.0f ? y : 1.0f - y);
  const float a = round_to<T>(g * sig);
  return round_to<T>(a * u);
}

// Launches the decode matvec for block type KIND (defined in matvec_impl.cuh, instantiated per type by
// matvec_kind.cu): mode MvMode, dtype SC_F32/F16/BF16, units_max an upper bound of the distinct experts,
// sg_hint the pairs a unit is expected to carry (slots decoded together).
template <int KIND>
int mv_dispatch(MvArgs a, int mode, int dtype, int units_max, int sg_hint, cudaStream_t s);

// The grouped fragment path (matvec_frag.cu): 16-bit activations, block types with fragment decoders, calls of
// gm::FROM pairs or more. Returns SC_OK or an error when it took the call, GM_DECLINED when the call is not its
// (the exact float32 kernel then takes it).
constexpr int GM_DECLINED = 1;
int gm_matvec(int kind, int mode, int dtype, const void* w, const void* w2, int experts, int rows, int cols,
              const uint32_t* idx, int pairs, int share, int glu, const void* x, const void* x2, void* out, int* err,
              cudaStream_t s);

// silu(g) * u in float32 (the Q2_0 down table's form, strata_mlx/blocks.py:709-711)
__device__ __forceinline__ float swiglu_f32(float g, float u) { return g / (1.0f + expf(-g)) * u; }

}  // namespace sc
