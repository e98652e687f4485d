// Expert parallel over peer memory: the exchange buffer every rank holds (mapped into every other rank by CUDA IPC),
// the release / acquire counters that mark a window complete, and the tagged words of the pair outputs.
//
// Layout of a rank's exchange buffer (the same on every rank):
//   [0, 512)       counters: xcount[p] at 128 p (window p complete); at 256 the step, this rank's count of layer
//                  calls on this buffer (the route kernel adds one a call: every call's pair outputs get a tag of their
//                  own, though the layers alternate two halves of Y; every rank counts alike); at 384 the down
//                  kernel's blocks of every call, each once (a combine waits for step x blocks a call)
//   X[p], p = 0, 1 the window of every rank's tokens, (T, H) of the activations' type, rank r's at rows r t ..
//   Y[p], p = 0, 1 this rank's tokens' pair outputs, (t, K, H / 2) 64-bit words, written by the ranks that own the
//                  pairs' experts: a word is two values of the activations' type (low half) and the layer call's
//                  step number (high half), stored in one single-copy-atomic 8-byte store, so that the reader knows
//                  a word is this call's by its tag, without fences or counts
// Layers alternate p, so that a rank one layer ahead writes the other half.
#pragma once

#include "common.cuh"

namespace sc {
namespace ep {

constexpr int COMBINE_BLOCKS = 8;  // blocks of the combine and feed kernels: each counts once on every rank

inline __host__ __device__ size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
inline __host__ __device__ size_t xbytes(int T, int H) { return align256(size_t(T) * H * 2); }
inline __host__ __device__ size_t ybytes(int t, int K, int H) { return align256(size_t(t) * K * H * 4); }
inline __host__ __device__ size_t xoff(int p, int T, int H) { return 512 + size_t(p) * xbytes(T, H); }
inline __host__ __device__ size_t yoff(int p, int T, int t, int K, int H) {
  return 512 + 2 * xbytes(T, H) + size_t(p) * ybytes(t, K, H);
}
inline __host__ __device__ size_t total_bytes(int T, int t, int K, int H) { return yoff(2, T, t, K, H); }
inline __host__ __device__ size_t xcount_off(int p) { return size_t(128) * p; }
constexpr size_t STEP_OFF = 256, DONE_OFF = 384;

__device__ __forceinline__ uint32_t* at_u32(uint64_t base, size_t off) {
  return reinterpret_cast<uint32_t*>(base + off);
}

// Counting once this block's writes are done: one release fence at system scope (after the block's barrier, it
// orders the writes of every thread of the block), then relaxed adds to the counts of every rank.
__device__ __forceinline__ void fence_release_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void count_relaxed(uint32_t* p) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(p) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits (about a second at most) until *p >= target; false, with SC_ERR_TIMEOUT recorded, when it gave up.
__device__ __forceinline__ bool wait_count(const uint32_t* p, uint32_t target, int* err) {
  if (load_acquire(p) >= target) return true;
  const long long start = clock64();
  while (load_acquire(p) < target) {
    if (clock64() - start > 2000000000LL) {
      record_error(err, SC_ERR_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Tagged words of Y: two 16-bit values and the step number that wrote them
__device__ __forceinline__ void store_tagged(uint64_t* p, uint32_t payload, uint32_t step) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(uint64_t(payload) | (uint64_t(step) << 32))
               : "memory");
}
__device__ __forceinline__ uint64_t load_word(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Two tagged words at once (each element of a vector access is single-copy atomic on its own)
__device__ __forceinline__ void load_words2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// The payload of *p once its tag is `step` (about a second at most; then SC_ERR_TIMEOUT is recorded and 0 returned)
__device__ __forceinline__ uint32_t wait_tagged(const uint64_t* p, uint32_t step, int* err) {
  uint64_t v = load_word(p);
  if (uint32_t(v >> 32) == step) return uint32_t(v);
  const long long start = clock64();
  while (uint32_t((v = load_word(p)) >> 32) != step) {
    if (clock64() - start > 2000000000LL) {
      record_error(err, SC_ERR_TIMEOUT);
      return 0u;
    }
    __nanosleep(32);
  }
  return uint32_t(v);
}

struct EpArgs {
  const uint64_t* peers;
  int G, rank, tl, T, H, K, Is, par, last;
  const float *wts, *gsh;  // the window's routes and shared-gate logits (this rank's workspace)
  const void* sout;        // the window's shared expert outputs (this rank's workspace)
  const void* x;           // feed: this rank's tokens
  void* out;               // combine: this rank's tokens' outputs
  int* err;
  const uint32_t* step;    // combine: the layer call's step number (this rank's exchange buffer, STEP_OFF)
  const uint32_t* done;    // combine: the down kernel's blocks count here (DONE_OFF), `dn_blocks` a call
  uint32_t dn_blocks;
};

// launchers (ep.cu); SC_OK or SC_ERR_*
int feed_launch(const EpArgs& A, int dtype, cudaStream_t s);
int combine_launch(const EpArgs& A, int dtype, cudaStream_t s);

}  // namespace ep
}  // namespace sc
