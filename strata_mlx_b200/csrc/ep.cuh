// Expert parallel over peer memory: the exchange buffer every rank holds (mapped into every other rank by CUDA IPC)
// and the release / acquire counters that mark its parts complete.
//
// Layout of a rank's exchange buffer (the same on every rank):
//   [0, 512)       counters: xcount[p] at 128 p (window p complete), ycount[p] at 256 + 128 p (pair outputs p)
//   X[p], p = 0, 1 the window of every rank's tokens, (T, H) of the activations' type, rank r's at rows r t ..
//   Y[p], p = 0, 1 this rank's tokens' pair outputs, (t, K, H), written by the ranks that own the pairs' experts
// Layers alternate p, so that a rank one layer ahead writes the other half.
#pragma once

#include "common.cuh"

namespace sc {
namespace ep {

constexpr int COMBINE_BLOCKS = 8;  // blocks of the combine and feed kernels: each counts once on every rank

inline __host__ __device__ size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
inline __host__ __device__ size_t xbytes(int T, int H) { return align256(size_t(T) * H * 2); }
inline __host__ __device__ size_t ybytes(int t, int K, int H) { return align256(size_t(t) * K * H * 2); }
inline __host__ __device__ size_t xoff(int p, int T, int H) { return 512 + size_t(p) * xbytes(T, H); }
inline __host__ __device__ size_t yoff(int p, int T, int t, int K, int H) {
  return 512 + 2 * xbytes(T, H) + size_t(p) * ybytes(t, K, H);
}
inline __host__ __device__ size_t total_bytes(int T, int t, int K, int H) { return yoff(2, T, t, K, H); }
inline __host__ __device__ size_t xcount_off(int p) { return size_t(128) * p; }
inline __host__ __device__ size_t ycount_off(int p) { return 256 + size_t(128) * p; }

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

struct EpArgs {
  const uint64_t* peers;
  int G, rank, tl, T, H, K, Is, par, last;
  const float *wts, *gsh;  // the window's routes and shared-gate logits (this rank's workspace)
  const void* sout;        // the window's shared expert outputs (this rank's workspace)
  const void* x;           // feed: this rank's tokens
  void* out;               // combine: this rank's tokens' outputs
  int* err;
  uint32_t ytarget;
};

// launchers (ep.cu); SC_OK or SC_ERR_*
int feed_launch(const EpArgs& A, int dtype, cudaStream_t s);
int combine_launch(const EpArgs& A, int dtype, cudaStream_t s);

}  // namespace ep
}  // namespace sc
