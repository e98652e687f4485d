// Shared declarations of the three-kernel decode block (decode_layer.cu) and its caller (moe.cu).
#pragma once

#include <algorithm>

#include "common.cuh"

namespace sc {
namespace dl {

constexpr int MAXT = 8;                // tokens in a window: the N of the m16n8k16 product
constexpr int RG = 16;                 // gate/up rows of a block (one unit's m16 tile)
constexpr int RC = 16;                 // down rows a block owns of every unit (one m16 tile)
constexpr int MAXU = 132;              // units: up to 8 x 16 routed experts + the shared one
constexpr int MAX_ROUTER_CHUNKS = 16;  // hidden sizes up to 16 x 256

// A unit is an expert the window chose (or the shared expert, unit 0) with the tokens that chose it.
struct Unit {
  int expert;        // -1 for the shared expert
  uint32_t tokmask;  // bit t: token t goes through this unit
  uint32_t kpack;    // 4 bits per token: the rank (k) of this expert among the token's choices
  int pad;
};

struct Plan {
  int units;
  int pad[3];
  Unit unit[MAXU];
};

struct LayerDev {
  const uint8_t *gate, *up, *down, *sgate, *sup, *sdown;
  const __half *router, *shared_gate;
  const void* x;
  void* out;
  int* err;
  int* ticket;
  float *logits, *gsh;
  uint32_t* idx;
  float* wts;
  Plan* plan;
  void* h;
  int T, H, I, Is, E, K, hstride;
  int rt_groups;  // route kernel: the window's tokens are split over this many groups of blocks
  int64_t rb_gu, rb_d, rb_sgu, rb_sd;
  int dn_stage, dn_stages;
  // expert parallel: this rank's experts [e0, e1) (its gate/up/down blocks hold only those, expert e at e - e0);
  // with ypairs set, the down kernel writes each pair's expert output (T, K, H), zero for pairs of other ranks'
  // experts, and the shared expert's (T, H) to sout, in place of the combine
  int e0, e1;
  void *ypairs, *sout;
  // expert parallel over peer memory (peers null: not in use): the ranks' exchange buffers (this rank's mappings),
  // G ranks, this one `rank`, `tl` tokens a rank; the layer reads window X[par] (complete when its count reaches
  // xtarget) and writes pair outputs Y[par] as words tagged with the call's step number
  const uint64_t* peers;
  int G, rank, tl, par;
  uint32_t xtarget;
  uint32_t* step;  // the layer call's step number (this rank's exchange buffer), counted up by the route kernel
  uint32_t* done;  // the down kernel's blocks, counted up once each per call (this rank's exchange buffer)
};

}  // namespace dl

struct V2Offsets {
  size_t err, ticket, logits, gsh, idx, wts, plan, h, sout;
};

// expert parallel: rank's experts [e0, e1) and where the pairs' outputs go (null: the single-GPU combine)
struct V2Ep {
  int e0 = 0, e1 = -1;
  void* ypairs = nullptr;
  const uint64_t* peers = nullptr;  // peer-memory exchange (see ep.cuh); ypairs unused then
  int G = 1, rank = 0, tl = 0, par = 0;
  uint32_t* step = nullptr;  // this rank's exchange buffer's step and down-block counts (ep.cuh)
  uint32_t* done = nullptr;
};

// h rows of the down product are padded by 32 elements so that the tokens' rows fall on different banks
inline int v2_hstride(const sc_moe_layer* L) { return std::max(L->inter, L->shared_inter) + 32; }
inline size_t v2_h_bytes(const sc_moe_layer* L, int tokens) {
  return size_t(tokens * L->top_k + 1) * size_t(tokens) * size_t(v2_hstride(L)) * 2;
}

bool v2_takes(const sc_moe_layer* L, int tokens);
// stage -1: the three kernels; 0, 1, 2: route, gate_up or down alone
int v2_run(const sc_moe_layer* L, const void* x, int tokens, void* out, uint8_t* ws, const V2Offsets& o,
           cudaStream_t s, int stage = -1, const V2Ep& ep = V2Ep{});

}  // namespace sc
