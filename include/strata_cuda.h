/*
 * strata_cuda.h -- C ABI of the B200 quantized-expert library (libstrata_cuda.so).
 *
 * The library multiplies straight from GGUF quantized blocks: the expert matvecs, the SwiGLU down product,
 * the prefill tile product on tcgen05 tensor cores, and the MoE router, top-k and combine. Every entry point
 * takes plain device pointers, sizes and a cudaStream_t passed as void*; it enqueues work on that stream and
 * returns without waiting. It never allocates: outputs and workspaces belong to the caller. Return value 0 is
 * success, a negative SC_ERR_* code a rejected call (nothing was enqueued) or a CUDA launch error.
 *
 * Kernels that find a bad expert id, or give up a bounded wait, record an SC_ERR_* code in the caller's
 * device int `err` (when not NULL) with atomicCAS(err, 0, code) and skip the work; they never trap.
 *
 * Each declaration names the interface of strata-mlx (cantrellsolutions/strata-mlx, paths inside that
 * project) that it replaces. Tensors are row-major; a stack of experts is (experts, rows, cols) weights held
 * as rows of GGUF blocks, row after row, exactly the bytes of the file (strata_mlx/gguf.py:105-115).
 */
#ifndef STRATA_CUDA_H
#define STRATA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SC_API __attribute__((visibility("default")))
#else
#define SC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SC_ABI_VERSION 1

/* block types: strata_mlx/blocks.py:35-38 (BLOCK), plus Q8_0 (strata_mlx/gguf.py:27) for dense tensors */
enum {
  SC_Q2_0 = 0, SC_IQ4_NL = 1, SC_IQ4_XS = 2, SC_IQ3_S = 3, SC_IQ3_XXS = 4,
  SC_IQ2_S = 5, SC_IQ2_XS = 6, SC_IQ2_XXS = 7, SC_IQ1_M = 8, SC_Q3_K = 9, SC_Q8_0 = 10,
  SC_NUM_KINDS = 11
};

/* activation / output types */
enum { SC_F32 = 0, SC_F16 = 1, SC_BF16 = 2 };

/* index types accepted by sc_tiles_of */
enum { SC_I32 = 0, SC_U32 = 1, SC_I64 = 2 };

/* error codes */
enum {
  SC_OK = 0,
  SC_ERR_KIND = -1,        /* unknown block type                                          */
  SC_ERR_SHAPE = -2,       /* a row does not end on a block, or a size out of range          */
  SC_ERR_DTYPE = -3,       /* activation type not taken by this entry point                  */
  SC_ERR_ALIGN = -4,       /* a pointer is not aligned as the entry point needs              */
  SC_ERR_ARG = -5,         /* a NULL or negative argument                                    */
  SC_ERR_CUDA = -6,        /* the launch failed (cudaGetLastError)                           */
  SC_ERR_WORKSPACE = -7,   /* workspace too small                                            */
  SC_ERR_UNSUPPORTED = -8, /* a combination this build does not take (caller falls back)     */
  SC_ERR_TIMEOUT = -9,     /* recorded by a kernel: a bounded wait gave up                    */
  SC_ERR_INDEX = -10,      /* recorded by a kernel: an expert id >= the number of experts    */
  SC_ERR_SCRATCH = -11     /* the call needs more scratch than SC_NOALLOC_SCRATCH_BYTES       */
};

/* library version (SC_ABI_VERSION) */
SC_API int sc_version(void);

/* a static description of an error code */
SC_API const char* sc_error_string(int code);

/* strata_mlx/blocks.py:35-38 BLOCK[kind]: weights per block and bytes per block */
SC_API int sc_block_info(int kind, int* per_block, int* block_bytes);

/* strata_mlx/blocks.py:397-404 dequantize(blocks, kind, shape, dtype): every weight of `mats` matrices of
 * rows x cols as out_dtype, out (mats, rows, cols). The float32 values are those of the reference's unpack32
 * (blocks.py:57-193) bit for bit; float16/bfloat16 outputs are those rounded to nearest even. */
SC_API int sc_dequant(int kind, const void* blocks, int64_t mats, int rows, int cols, int out_dtype, void* out,
               void* stream);

/* strata_mlx/blocks.py:420-436 BlockSwitchLinear.__call__ (the _MATVEC kernel, blocks.py:196-220):
 * out[p, r] = W[idx[p], r, :] . x[p / share, :] for p < pairs, sums in float32, out (pairs, rows) in the type of x.
 * blocks: (experts, rows, cols) stack. Pairs that name the same expert read its blocks once. */
SC_API int sc_expert_matvec(int kind, const void* blocks, int experts, int rows, int cols, const uint32_t* idx, int pairs,
                     int share, const void* x, int dtype, void* out, int* err, void* stream);

/* strata_mlx/blocks.py:331-346 matvec_separate(experts, kind, rows, cols, x, share): as sc_expert_matvec, pair p's
 * expert being its own buffer bases[p] (a device array of `pairs` device pointers, each rows x cols of blocks). */
SC_API int sc_expert_matvec_ptrs(int kind, const void* const* bases, int pairs, int rows, int cols, int share, const void* x,
                          int dtype, void* out, int* err, void* stream);

/* strata_mlx/blocks.py:383-394 window_matvec(blocks, kind, rows, cols, x): out[t] = W . x[t], one layer, tokens rows of x */
SC_API int sc_window_matvec(int kind, const void* blocks, int rows, int cols, const void* x, int dtype, int tokens, void* out,
                     int* err, void* stream);

/* strata_mlx/blocks.py:782-798 matvec_glu(lin, idx, gate, up) (the _MATVEC_GLU kernel, blocks.py:225-259):
 * out[p] = W[idx[p]] . h[p] with h = swiglu(gate[p], up[p]) worked out in shared memory.
 * glu 0: mlx-lm's rounding (sigmoid in float32 rounded to the type, then two products in the type), as _MATVEC_GLU;
 * glu 1: silu(g) * u in float32 rounded once, as the Q2_0 down table's (blocks.py:706-715, lookup_down_glu :740-760). */
SC_API int sc_matvec_glu(int kind, const void* blocks, int experts, int rows, int cols, const uint32_t* idx, int pairs,
                  const void* gate, const void* up, int dtype, int glu, void* out, int* err, void* stream);

/* strata_mlx/blocks.py:808-818 (switch_glu's per-pair branch: gate(x), up(x), swiglu) in one kernel:
 * h[p, r] = swiglu(W_gate[idx[p], r] . x[p / share], W_up[idx[p], r] . x[p / share]), mlx-lm's rounding.
 * gate and up are stacks of the same kind and shape (experts, rows, cols). */
SC_API int sc_expert_gate_up(int kind, const void* gate, const void* up, int experts, int rows, int cols, const uint32_t* idx,
                      int pairs, int share, const void* x, int dtype, void* h, int* err, void* stream);

/* mlx-lm swiglu as strata_mlx/blocks.py:230-238 restates it, elementwise over n values of dtype */
SC_API int sc_swiglu(const void* gate, const void* up, int64_t n, int dtype, void* out, void* stream);

/* strata_mlx/fused.py:357-390 WindowLinear.__call__: logits (tokens, rows) float32 = x . W^T,
 * W (rows, cols) float16, x (tokens, cols) of dtype, float32 sums. */
SC_API int sc_router(const void* w, int rows, int cols, const void* x, int dtype, int tokens, float* logits, void* stream);

/* strata_mlx/fused.py:424-436 top_k(logits, k): the k largest of each of `rows` rows of n float32 logits, largest
 * first, ties to the lower index (the order of the reference's _TOPK kernel, fused.py:400-418). idx (rows, k). */
SC_API int sc_top_k(const float* logits, int rows, int n, int k, uint32_t* idx, void* stream);

/* strata_mlx/fused.py:490-491: top_k as above, then weights (rows, k) float32 = softmax over the chosen logits */
SC_API int sc_top_k_softmax(const float* logits, int rows, int n, int k, uint32_t* idx, float* weights, void* stream);

/* strata_mlx/fused.py:467-481 moe_combine(y, w, g, s): out[t] = T(sum_k y[t,k] w[t,k]) + T(T(sigmoid(g[t])) s[t]),
 * the k terms added in MLX's col_reduce order (fused.py:448-462). y (rows, k, d), w (rows, k) float32,
 * g (rows), s (rows, d), out (rows, d); y, g, s, out of dtype. */
SC_API int sc_moe_combine(const void* y, const float* w, const void* g, const void* s, int rows, int k, int d, int dtype,
                   void* out, void* stream);

/* strata_mlx/blocks.py:539-563 tiles_of(indices, experts): the pairs of idx (pairs = tokens * k entries, of
 * idx_dtype) laid out in tiles of 16 slots, each tile one expert's, in a number of tiles that depends only on
 * the number of pairs: max_tiles = pairs / 16 + min(experts, pairs).
 * tile_expert (max_tiles): a tile's expert, or `experts` for a tile nothing fills; token (max_tiles * 16): the
 * token (pair / k) of each slot, 0 for empty slots; where (pairs): each pair's slot.
 * workspace: sc_tiles_of_workspace(experts) bytes of device memory. */
SC_API int sc_tiles_of(const void* idx, int idx_dtype, int pairs, int k, int experts, uint32_t* tile_expert, uint32_t* token,
                uint32_t* where, void* workspace, size_t workspace_bytes, void* stream);
SC_API size_t sc_tiles_of_workspace(int experts);

/* strata_mlx/blocks.py:516-536 tile_matmul(blocks, kind, shape, a, tile_expert): c (P, rows) float32 =
 * W[tile_expert[p / 16]] . a[p] for a (P, cols) of a_dtype, P a multiple of 16; the weights are rounded to
 * a_dtype before they multiply; float32 sums. Tiles naming no expert (>= experts) are left unwritten.
 * bfloat16 / float16 `a` run on the tcgen05 tensor cores; float32 `a` on the CUDA cores. err: device int that
 * records SC_ERR_TIMEOUT when one of the tensor-core kernel's bounded waits gives up (may be NULL). */
SC_API int sc_tile_matmul(int kind, const void* blocks, int experts, int rows, int cols, const void* a, int a_dtype, int P,
                   const uint32_t* tile_expert, float* c, int* err, void* stream);
/* Which kernel sc_tile_matmul runs for these arguments: 1 the tcgen05 tensor-core kernel (float16 / bfloat16 `a`,
 * rows by 128, cols by 256, at most 4096 tiles, 16-byte aligned `a` and blocks), 0 the CUDA-core kernel. No
 * counterpart in strata-mlx (its tile kernel is one Metal kernel). */
SC_API int sc_tile_matmul_path(int kind, int experts, int rows, int cols, int a_dtype, int P, const void* a,
                               const void* blocks);

/* strata_mlx/blocks.py:566-576 _tiled_glu in one call: the gate, up and down tile products of a prompt's pairs
 * laid out by sc_tiles_of (tile_expert, where): gate and up stored in a_dtype by the products' epilogues, their
 * swiglu, and the down product written straight into out (pairs, hidden) in the pairs' order, all in a_dtype
 * (float16 / bfloat16): the same bits
 * as three sc_tile_matmul calls, swiglu and the unsort. a (P, hidden) holds each slot's token (as _tiled_glu gathers
 * it). SC_ERR_UNSUPPORTED when a product is not one the tcgen05 kernel takes (the caller then composes the three).
 * workspace: sc_tile_glu_workspace(P, inter, a_dtype) bytes. */
SC_API int sc_tile_glu(int kind_gate, const void* gate, int kind_up, const void* up, int kind_down, const void* down,
                       int experts, int hidden, int inter, const void* a, int a_dtype, int P,
                       const uint32_t* tile_expert, const uint32_t* where, int pairs, void* out, void* workspace,
                       size_t workspace_bytes, int* err, void* stream);
SC_API size_t sc_tile_glu_workspace(int P, int inter, int a_dtype);

/* strata_mlx/dense.py:109-167 ScaledLinear: a dense layer held as Q6_K's three parts, a weight being
 * code * scale * d: codes int8 (rows, cols), scales int8 (rows, cols / 16), d float16 (rows, cols / d_step).
 * rows by 4 and cols by 256 (dense.py:97-99 fits), d_step a multiple of 16 dividing cols; codes and x 16-byte
 * aligned. sc_scaled_matvec: out (tokens, rows) = x (tokens, cols) . W^T in x's type, float32 sums, tokens <= 8
 * (dense.py:141-167, the window kernel). sc_scaled_floats: W (rows, cols) in out_dtype, each weight
 * float(d) * float(scale) * float(code) in float32, rounded once (dense.py:125-139, the floats of a prompt chunk).
 * err: device int in which the tensor-core window kernel records SC_ERR_TIMEOUT when one of its bounded waits for
 * a bulk copy gives up (its rows are then left unwritten); may be NULL. */
SC_API int sc_scaled_matvec(const void* codes, const void* scales, const void* d, int rows, int cols, int d_step,
                            const void* x, int dtype, int tokens, void* out, int* err, void* stream);
SC_API int sc_scaled_floats(const void* codes, const void* scales, const void* d, int rows, int cols, int d_step,
                            int out_dtype, void* out, void* stream);

/* One MoE block in decode, strata_mlx/fused.py:487-497 (_Routed.__call__): the router (fused.py:377-390), top_k
 * (:424-436), the softmax over the chosen logits (:491), the routed SwiGLU experts (blocks.py:801-829), the
 * shared expert and its gate, and moe_combine (fused.py:467-481), for a window of 1..8 tokens. */
typedef struct sc_moe_layer {
  int hidden;              /* H: x and out are (tokens, H)                                       */
  int inter;               /* I: inner size of a routed expert                                   */
  int experts;             /* E                                                                  */
  int top_k;               /* K <= 16                                                            */
  int kind_gate, kind_up, kind_down;
  const void* gate;        /* (E, I, H) blocks                                                    */
  const void* up;          /* (E, I, H) blocks                                                    */
  const void* down;        /* (E, H, I) blocks                                                    */
  const void* router;      /* (E, H) float16                                                      */
  int shared_inter;        /* inner size of the shared expert, 0 for none                         */
  int kind_sgate, kind_sup, kind_sdown;
  const void* sgate;       /* (shared_inter, H) blocks                                            */
  const void* sup;         /* (shared_inter, H) blocks                                            */
  const void* sdown;       /* (H, shared_inter) blocks                                            */
  const void* shared_gate; /* (H) float16: the shared expert's gate, a product with x               */
  int dtype;               /* activations: SC_F16 or SC_BF16                                      */
} sc_moe_layer;

/* out (tokens, H) of layer->dtype. workspace: sc_moe_decode_workspace(layer, tokens) bytes of device memory,
 * whose first int is the kernels' error word. Results a caller may read back from the workspace:
 * sc_moe_decode_routes(). */
SC_API int sc_moe_decode_layer(const sc_moe_layer* layer, const void* x, int tokens, void* out, void* workspace,
                        size_t workspace_bytes, void* stream);
SC_API size_t sc_moe_decode_workspace(const sc_moe_layer* layer, int tokens);
/* Offsets in the workspace of the last call's routes: idx (tokens, K) uint32 and weights (tokens, K) float32. */
SC_API int sc_moe_decode_routes(const sc_moe_layer* layer, int tokens, size_t* idx_offset, size_t* weight_offset);

/* A chain of decode blocks in one launch (no counterpart in strata-mlx, whose engine calls _Routed.__call__ once per
 * layer, strata_mlx/engine.py:276-279): layers[0 .. n_layers) applied in turn to a window of `tokens` (1..8) tokens,
 * each layer taking the previous one's output, except that every `refeed`-th layer (refeed > 0) takes x again; out
 * (tokens, H) is the last layer's output. Every layer has the same shape and activation type and is one that
 * sc_moe_decode_layer's fused path takes; n_layers <= 64; hidden a multiple of 128. One persistent kernel, a block
 * an SM (a cooperative launch): per layer the router, a grid-wide barrier, the routes (every block), the gate/up
 * products, a barrier, the down products, and the combine; the same bits as sc_moe_decode_layer layer by layer.
 * workspace: sc_moe_decode_chain_workspace bytes, zeroed before its first use (its first words are the error word
 * and the kernel's barrier count, which each launch leaves at zero); after a launch whose kernel recorded an error
 * in the error word, zero it again. Each layer's routes stay readable: sc_moe_decode_chain_routes gives the offsets
 * of idx (n_layers, tokens, K) uint32 and weights (n_layers, tokens, K) float32. */
SC_API int sc_moe_decode_chain(const sc_moe_layer* layers, int n_layers, const void* x, int tokens, int refeed,
                               void* out, void* workspace, size_t workspace_bytes, void* stream);
SC_API size_t sc_moe_decode_chain_workspace(const sc_moe_layer* layers, int n_layers, int tokens);
SC_API int sc_moe_decode_chain_routes(const sc_moe_layer* layers, int n_layers, int tokens, size_t* idx_offset,
                                      size_t* weight_offset);

/* One of the three kernels of sc_moe_decode_layer's fused path -- stage 0 routes (router, top-k, plan), 1 the
 * experts' gate/up, 2 the down products and the combine -- on a workspace that a previous sc_moe_decode_layer call
 * with the same layer and token count filled. For timing and profiling the kernels one at a time (no counterpart
 * in strata-mlx). SC_ERR_UNSUPPORTED when the layer does not take the fused path. */
SC_API int sc_moe_decode_stage(const sc_moe_layer* layer, const void* x, int tokens, void* out, void* workspace,
                               size_t workspace_bytes, int stage, void* stream);

/* Expert parallel decode (no counterpart in strata-mlx, which runs on one device). One rank's share of an MoE block
 * over a window of `tokens` (the window holds every rank's tokens): the router and top-k for every token, then the
 * gate/up/down of only the pairs whose expert is in [expert_begin, expert_end); layer->gate/up/down hold just those
 * experts (expert e at e - expert_begin), layer->experts is the total. Writes y_pairs (tokens, top_k, hidden) of the
 * activations' type: each pair's expert output, zero for pairs of other ranks' experts, so that a sum over ranks
 * (all-reduce) holds every pair's output exactly; the shared expert's output and the routes stay in the workspace
 * (sc_moe_decode_workspace bytes). Takes the layers the fused decode takes; SC_ERR_UNSUPPORTED otherwise. */
SC_API int sc_moe_decode_layer_ep(const sc_moe_layer* layer, const void* x, int tokens, int expert_begin,
                                  int expert_end, void* y_pairs, void* workspace, size_t workspace_bytes, void* stream);

/* After sc_moe_decode_layer_ep and the sum of y_pairs over ranks: moe_combine (strata_mlx/fused.py:467-481) of the
 * window's tokens from y_pairs and the workspace's routes and shared expert output, into out (tokens, hidden). The
 * same bits as sc_moe_decode_layer gives for those tokens on one device. */
SC_API int sc_moe_decode_combine(const sc_moe_layer* layer, const void* y_pairs, int tokens, void* out,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* Expert parallel over peer memory (no counterpart in strata-mlx): the collectives of sc_moe_decode_layer_ep's
 * exchange replaced by stores into the other ranks' memory over NVLink, with counts that mark each part complete.
 * Every rank holds an exchange buffer of sc_ep_exchange_bytes bytes (zeroed once), maps the others' buffers with
 * sc_ipc_handle / sc_ipc_open, and describes them in an sc_ep_exchange. A chain of L layers (L even) for a step:
 * sc_ep_feed (this rank's tokens into every rank's window), then per layer l sc_moe_decode_layer_ep_p2p with
 * parity l % 2 and sc_ep_combine (last = l == L - 1), which writes this rank's tokens' outputs to `out` and into
 * every rank's next window. The kernels' waits on other ranks are bounded (about a second; SC_ERR_TIMEOUT). */
typedef struct sc_ep_exchange {
  const uint64_t* peers; /* device array (ranks): each rank's exchange buffer, mapped into this process */
  uint64_t own;          /* this rank's exchange buffer (= peers[rank]), a device address */
  int ranks, rank, tokens_per_rank;
} sc_ep_exchange;

SC_API size_t sc_ep_exchange_bytes(const sc_moe_layer* layer, int ranks, int tokens_per_rank);
SC_API int sc_ipc_handle(const void* ptr, void* handle /* 64 bytes */, size_t* offset);
SC_API int sc_ipc_open(const void* handle, void** base);
SC_API int sc_ipc_close(void* base);
SC_API int sc_ep_feed(const sc_moe_layer* layer, const sc_ep_exchange* ex, const void* x, void* stream);
SC_API int sc_moe_decode_layer_ep_p2p(const sc_moe_layer* layer, const sc_ep_exchange* ex, int expert_begin,
                                      int expert_end, int parity, void* workspace, size_t workspace_bytes,
                                      void* stream);
SC_API int sc_ep_combine(const sc_moe_layer* layer, const sc_ep_exchange* ex, int parity, int last, void* out,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Paged grouped-query attention of the synthetic decoder around the MoE blocks (strata_mlx's engine runs its own
 * attention trunk, strata_mlx/engine.py:710-749; the decoder here stands in for it at BASELINE configurations 4 and
 * 5, whose MoE blocks are the hot path). One sequence: q (tokens, q_heads, head_dim) bfloat16 of the window's
 * `tokens` (1..8) new tokens; the cache k_cache, v_cache (pages, 16, kv_heads, head_dim) bfloat16, the sequence's
 * pages listed in block_table; *ctx_dev (device int, at most max_ctx, read by the kernels so that a decode step can
 * replay from a CUDA graph) tokens in all, the window's own keys already written at positions ctx - tokens ..
 * ctx - 1. Token i sees keys 0 .. ctx - tokens + i. out (tokens, q_heads, head_dim) bfloat16 = softmax(scale q k^T) v,
 * float32 sums, probabilities rounded to bfloat16 for the value product. head_dim 256, q_heads = 8 kv_heads.
 * workspace: sc_paged_attention_workspace(max_ctx, kv_heads) bytes. */
SC_API int sc_paged_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                              const int32_t* ctx_dev, int max_ctx, int tokens, int q_heads, int kv_heads, int head_dim,
                              float scale, void* out, void* workspace, size_t workspace_bytes, void* stream);
SC_API size_t sc_paged_attention_workspace(int ctx, int kv_heads);

/* The synthetic decoder's trunk (no counterpart in strata-mlx's MoE path; its engine's own trunk is out of scope):
 * sc_add_rmsnorm: x (rows, cols) += delta (rounded to the type; delta may be NULL), then out = x * rsqrt(mean(x^2) +
 * eps) * w, float32 math, cols by 8 (at most 8192), 16-byte aligned. sc_rope_cache: rotate-half RoPE on q (tokens,
 * q_heads, head_dim) in place and on k (tokens, kv_heads, head_dim), the angles' cos / sin tables (positions,
 * head_dim / 2) float32 at positions *pos .. *pos + tokens - 1 (pos a device int), and k, v written into the paged
 * cache (pages, page, kv_heads, head_dim) at those positions' slots (block_table). bfloat16 (sc_rope_cache) or
 * bfloat16 / float16 (sc_add_rmsnorm). */
SC_API int sc_add_rmsnorm(void* x, const void* delta, const void* w, int rows, int cols, float eps, int dtype, void* out,
                          void* stream);
SC_API int sc_rope_cache(void* q, const void* k, const void* v, int tokens, int q_heads, int kv_heads, int head_dim,
                         const float* cos, const float* sin, const int32_t* pos, const int32_t* block_table, int page,
                         void* k_cache, void* v_cache, int dtype, void* stream);

/* No counterpart in strata-mlx: an addition for callers that cannot allocate device memory.
 *
 * sc_moe_decode_layer without a workspace argument. Some hosts of this library own every byte of device memory
 * from start-up and hand a kernel library nothing but the inputs and outputs of each call: a serving process
 * with a fixed memory plan that forbids allocation once it runs, or a binding from a language that has no CUDA
 * allocator at all. Such a caller cannot supply the scratch sc_moe_decode_layer needs. This entry point takes
 * its scratch from a static device array inside the library instead, and calls no allocator of any kind.
 *
 * Limit: the layer's sc_moe_decode_workspace(layer, tokens) must not exceed SC_NOALLOC_SCRATCH_BYTES (4 MiB);
 * larger calls are rejected with SC_ERR_SCRATCH and enqueue nothing. Every GPU that loads the library holds this
 * array until the process exits. The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream capture begins. All calls on a
 * device share the one array and it keeps the last call's contents (the call clears what must start at zero):
 * calls whose work overlaps on the GPU (on different streams, or from several threads) race on it and must not
 * be issued. Same results as sc_moe_decode_layer, bit for bit. */
#define SC_NOALLOC_SCRATCH_BYTES (4u << 20)
SC_API int sc_moe_decode_layer_noalloc(const sc_moe_layer* layer, const void* x, int tokens, void* out, void* stream);

/* The error word of sc_moe_decode_layer_noalloc's kernels on the current device (no counterpart in strata-mlx). The
 * kernels of a call record a bad expert id or a bounded wait that gave up in the static array's first int, which no
 * caller can reach otherwise. This waits for `stream`, stores in *code the first error recorded since the last read
 * (SC_OK when none), and clears the word. Allocates nothing. */
SC_API int sc_moe_decode_noalloc_error(int* code, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* STRATA_CUDA_H */
