// Decode-path expert products straight from GGUF blocks:
//   sc_expert_matvec       BlockSwitchLinear.__call__   (strata_mlx/blocks.py:420-436, _MATVEC :196-220)
//   sc_expert_matvec_ptrs  matvec_separate              (blocks.py:331-346)
//   sc_window_matvec       window_matvec                (blocks.py:349-394)
//   sc_matvec_glu          matvec_glu / lookup_down_glu (blocks.py:222-259, :740-798)
//   sc_expert_gate_up      gate(x), up(x), swiglu of switch_glu (blocks.py:808-818), fused
//
// With 16-bit activations, a block type with fragment decoders and gm::FROM pairs or more, the grouped fragment
// kernel (matvec_frag.cu) takes the call. Otherwise one kernel serves all of them. A block first works out which experts its pairs name (a bitmap, so each
// expert's blocks are read once however many pairs share it), stages the activations in shared memory as
// float32, then splits the (expert, chunk of rows) list evenly over the grid. A producer warp streams each
// chunk's rows into a ring of shared-memory stages with 1-D bulk copies (TMA) completing on mbarriers; eight
// consumer warps decode the blocks from shared memory and accumulate float32 dot products, finishing each row
// with a warp-shuffle reduction.
#include <algorithm>

#include "matvec.cuh"

namespace sc {

static int pow2_hint(int v) { return v <= 1 ? 1 : v <= 2 ? 2 : v <= 4 ? 4 : 8; }

// Splits `pairs` into launches whose activations fit shared memory, keeping each launch's x rows whole
// (a multiple of `share` pairs), and calls launch(p0, n) for each.
template <typename F>
static int mv_split(int pairs, int share, int cols, int per_pair_rows, F&& launch) {
  const int64_t x_budget = 88 * 1024;
  const int64_t row_cost = int64_t(cols) * 4;
  int64_t max_xrows = std::max<int64_t>(1, x_budget / row_cost);
  int64_t step = per_pair_rows ? std::max<int64_t>(1, max_xrows) : std::max<int64_t>(share, (max_xrows) * share);
  step = std::min<int64_t>(step, MV_MAX_PAIRS - MV_MAX_PAIRS % share);
  if (step <= 0) return SC_ERR_SHAPE;
  for (int64_t p0 = 0; p0 < pairs; p0 += step) {
    const int rc = launch(int(p0), int(std::min<int64_t>(step, pairs - p0)));
    if (rc != SC_OK) return rc;
  }
  return SC_OK;
}

static int check_common(int kind, int rows, int cols, int64_t& rb) {
  if (rows <= 0 || cols <= 0) return SC_ERR_SHAPE;
  if (block_info(kind).per_block == 0) return SC_ERR_KIND;
  rb = row_bytes(kind, cols);
  if (rb < 0) return SC_ERR_SHAPE;
  return SC_OK;
}

// per-kind launchers, compiled in matvec_kind.cu
template <typename F>
static bool with_kind(int kind, F&& f) {
  return dispatch_kind(kind, [&]<int KIND>() { f([](MvArgs a, int mode, int dtype, int units, int hint, cudaStream_t s) {
    return mv_dispatch<KIND>(a, mode, dtype, units, hint, s);
  }); });
}

static bool dtype_ok(int dtype) { return dtype == SC_F32 || dtype == SC_F16 || dtype == SC_BF16; }
static int64_t dsize(int dtype) { return dtype == SC_F32 ? 4 : 2; }
static const void* offset(const void* p, int64_t elems, int dtype) {
  return static_cast<const uint8_t*>(p) + elems * dsize(dtype);
}
static void* offset(void* p, int64_t elems, int dtype) { return static_cast<uint8_t*>(p) + elems * dsize(dtype); }

}  // namespace sc

using namespace sc;

extern "C" int sc_expert_matvec(int kind, const void* blocks, int experts, int rows, int cols, const uint32_t* idx,
                                int pairs, int share, const void* x, int dtype, void* out, int* err, void* stream) {
  int64_t rb;
  if (int rc = check_common(kind, rows, cols, rb)) return rc;
  if (!blocks || !idx || !x || !out || pairs < 0 || share < 1 || experts < 1) return SC_ERR_ARG;
  if (!dtype_ok(dtype)) return SC_ERR_DTYPE;
  if (experts > MV_MAX_EXPERTS) return SC_ERR_SHAPE;
  if (pairs == 0) return SC_OK;
  if (int rc = gm_matvec(kind, MV_PLAIN, dtype, blocks, nullptr, experts, rows, cols, idx, pairs, share, 0, x,
                         nullptr, out, err, static_cast<cudaStream_t>(stream));
      rc != GM_DECLINED)
    return rc;
  int rc = SC_OK;
  with_kind(kind, [&](auto launch) {
    rc = mv_split(pairs, share, cols, 0, [&](int p0, int n) {
      MvArgs a{};
      a.w = static_cast<const uint8_t*>(blocks);
      a.idx = idx + p0;
      a.x = offset(x, int64_t(p0 / share) * cols, dtype);
      a.out = offset(out, int64_t(p0) * rows, dtype);
      a.err = err;
      a.rbytes = rb;
      a.experts = experts; a.rows = rows; a.cols = cols; a.pairs = n; a.share = share;
      const int hint = share > 1 ? pow2_hint((n + share - 1) / share) : pow2_hint(n / 10);
      return launch(a, MV_PLAIN, dtype, std::min(n, experts), hint, static_cast<cudaStream_t>(stream));
    });
  });
  return rc;
}

extern "C" int sc_expert_matvec_ptrs(int kind, const void* const* bases, int pairs, int rows, int cols, int share,
                                     const void* x, int dtype, void* out, int* err, void* stream) {
  int64_t rb;
  if (int rc = check_common(kind, rows, cols, rb)) return rc;
  if (!bases || !x || !out || pairs < 0 || share < 1) return SC_ERR_ARG;
  if (!dtype_ok(dtype)) return SC_ERR_DTYPE;
  if (pairs == 0) return SC_OK;
  int rc = SC_OK;
  with_kind(kind, [&](auto launch) {
    rc = mv_split(pairs, share, cols, 0, [&](int p0, int n) {
      MvArgs a{};
      a.bases = reinterpret_cast<const uint8_t* const*>(bases) + p0;
      a.x = offset(x, int64_t(p0 / share) * cols, dtype);
      a.out = offset(out, int64_t(p0) * rows, dtype);
      a.err = err;
      a.rbytes = rb;
      a.experts = n; a.rows = rows; a.cols = cols; a.pairs = n; a.share = share;
      return launch(a, MV_PLAIN, dtype, n, 1, static_cast<cudaStream_t>(stream));
    });
  });
  return rc;
}

extern "C" int sc_window_matvec(int kind, const void* blocks, int rows, int cols, const void* x, int dtype, int tokens,
                                void* out, int* err, void* stream) {
  int64_t rb;
  if (int rc = check_common(kind, rows, cols, rb)) return rc;
  if (!blocks || !x || !out || tokens < 0) return SC_ERR_ARG;
  if (!dtype_ok(dtype)) return SC_ERR_DTYPE;
  if (tokens == 0) return SC_OK;
  int rc = SC_OK;
  with_kind(kind, [&](auto launch) {
    rc = mv_split(tokens, 1, cols, 1, [&](int p0, int n) {
      MvArgs a{};
      a.w = static_cast<const uint8_t*>(blocks);
      a.idx = nullptr;
      a.x = offset(x, int64_t(p0) * cols, dtype);
      a.out = offset(out, int64_t(p0) * rows, dtype);
      a.err = err;
      a.rbytes = rb;
      a.experts = 1; a.rows = rows; a.cols = cols; a.pairs = n; a.share = 1;
      return launch(a, MV_PLAIN, dtype, 1, pow2_hint(n), static_cast<cudaStream_t>(stream));
    });
  });
  return rc;
}

extern "C" int sc_matvec_glu(int kind, const void* blocks, int experts, int rows, int cols, const uint32_t* idx,
                             int pairs, const void* gate, const void* up, int dtype, int glu, void* out, int* err,
                             void* stream) {
  int64_t rb;
  if (int rc = check_common(kind, rows, cols, rb)) return rc;
  if (!blocks || !idx || !gate || !up || !out || pairs < 0 || experts < 1 || (glu != 0 && glu != 1)) return SC_ERR_ARG;
  if (!dtype_ok(dtype)) return SC_ERR_DTYPE;
  if (experts > MV_MAX_EXPERTS) return SC_ERR_SHAPE;
  if (pairs == 0) return SC_OK;
  if (int rc = gm_matvec(kind, MV_GLU_IN, dtype, blocks, nullptr, experts, rows, cols, idx, pairs, 1, glu, gate, up,
                         out, err, static_cast<cudaStream_t>(stream));
      rc != GM_DECLINED)
    return rc;
  int rc = SC_OK;
  with_kind(kind, [&](auto launch) {
    rc = mv_split(pairs, 1, cols, 1, [&](int p0, int n) {
      MvArgs a{};
      a.w = static_cast<const uint8_t*>(blocks);
      a.idx = idx + p0;
      a.x = offset(gate, int64_t(p0) * cols, dtype);
      a.x2 = offset(up, int64_t(p0) * cols, dtype);
      a.out = offset(out, int64_t(p0) * rows, dtype);
      a.err = err;
      a.rbytes = rb;
      a.experts = experts; a.rows = rows; a.cols = cols; a.pairs = n; a.share = 1; a.glu = glu;
      return launch(a, MV_GLU_IN, dtype, std::min(n, experts), pow2_hint(n / 10), static_cast<cudaStream_t>(stream));
    });
  });
  return rc;
}

extern "C" int sc_expert_gate_up(int kind, const void* gate, const void* up, int experts, int rows, int cols,
                                 const uint32_t* idx, int pairs, int share, const void* x, int dtype, void* h, int* err,
                                 void* stream) {
  int64_t rb;
  if (int rc = check_common(kind, rows, cols, rb)) return rc;
  if (!gate || !up || !idx || !x || !h || pairs < 0 || share < 1 || experts < 1) return SC_ERR_ARG;
  if (!dtype_ok(dtype)) return SC_ERR_DTYPE;
  if (experts > MV_MAX_EXPERTS) return SC_ERR_SHAPE;
  if (pairs == 0) return SC_OK;
  if (int rc = gm_matvec(kind, MV_GATEUP, dtype, gate, up, experts, rows, cols, idx, pairs, share, 0, x, nullptr, h,
                         err, static_cast<cudaStream_t>(stream));
      rc != GM_DECLINED)
    return rc;
  int rc = SC_OK;
  with_kind(kind, [&](auto launch) {
    rc = mv_split(pairs, share, cols, 0, [&](int p0, int n) {
      MvArgs a{};
      a.w = static_cast<const uint8_t*>(gate);
      a.w2 = static_cast<const uint8_t*>(up);
      a.idx = idx + p0;
      a.x = offset(x, int64_t(p0 / share) * cols, dtype);
      a.out = offset(h, int64_t(p0) * rows, dtype);
      a.err = err;
      a.rbytes = rb;
      a.experts = experts; a.rows = rows; a.cols = cols; a.pairs = n; a.share = share;
      const int hint = share > 1 ? pow2_hint((n + share - 1) / share) : pow2_hint(n / 10);
      return launch(a, MV_GATEUP, dtype, std::min(n, experts), hint, static_cast<cudaStream_t>(stream));
    });
  });
  return rc;
}
