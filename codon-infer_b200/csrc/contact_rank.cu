// Ranking of predicted contacts on the device: the pair list of compute_pipeline_contacts_parallel
// (src/pipeline.rs:454-486) -- pairs (i, j) of an n x n contact-probability map with
// j >= i + min_separation, sorted by probability, the first k kept -- without copying the map to
// the host (8 x 4094^2 floats for the 3B batch).
//
// Order. The reference sorts all pairs with a stable sort on descending probability, so ties keep
// their (i, j) row-major order. Each candidate becomes one 64-bit key: the high word is the
// probability's bits mapped so that larger probabilities give smaller unsigned values, the low
// word the flat index i * n + j. Ascending key order is then exactly the reference's order, and
// keys are unique. (NaN probabilities compare Equal to everything in the reference, which has no
// consistent order; sigmoid outputs are never NaN.)
//
// Selection. Passes of one kernel: every CTA sorts a tile of kTile keys in shared memory (bitonic
// network, 1024 threads) and writes its first K (a power of two >= k), until one tile holds all
// survivors; its first k keys are the answer. n^2 = 16.8 M candidates take three passes at K = 64.
#include <atomic>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.cuh"

namespace esm {

namespace {

constexpr int kTile = 8192;         // keys sorted per CTA (64 KiB of shared memory)
constexpr int kRankThreads = 1024;
constexpr uint64_t kNoKey = ~0ull;  // sorts after every real key

__device__ __forceinline__ uint64_t pair_key(float p, uint32_t flat) {
  if (p == 0.0f) p = 0.0f;  // -0 and +0 compare Equal in the reference: one key for both
  const uint32_t u = __float_as_uint(p);
  const uint32_t asc = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // order-preserving map
  return (static_cast<uint64_t>(~asc) << 32) | flat;                 // descending probability
}

__device__ void bitonic_sort(uint64_t* s) {
  for (int size = 2; size <= kTile; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int t = threadIdx.x; t < kTile / 2; t += kRankThreads) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t a = s[lo], b = s[hi];
        if ((a > b) == up) {
          s[lo] = b;
          s[hi] = a;
        }
      }
    }
  }
  __syncthreads();
}

// Pass 0: keys straight from the map (candidates only), tile = kTile consecutive flat indices.
__global__ void __launch_bounds__(kRankThreads)
    rank_map_kernel(const float* __restrict__ map, int n, int min_sep, int keep, uint64_t* __restrict__ out) {
  extern __shared__ uint64_t s[];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile;
  const int64_t total = static_cast<int64_t>(n) * n;
  for (int t = threadIdx.x; t < kTile; t += kRankThreads) {
    const int64_t f = base + t;
    uint64_t key = kNoKey;
    if (f < total) {
      const int i = static_cast<int>(f / n), j = static_cast<int>(f - static_cast<int64_t>(i) * n);
      if (j >= i + min_sep) key = pair_key(map[f], static_cast<uint32_t>(f));
    }
    s[t] = key;
  }
  bitonic_sort(s);
  for (int t = threadIdx.x; t < keep; t += kRankThreads) out[static_cast<int64_t>(blockIdx.x) * keep + t] = s[t];
}

// Later passes: tiles of kTile keys from the previous pass's survivors.
__global__ void __launch_bounds__(kRankThreads)
    rank_keys_kernel(const uint64_t* __restrict__ in, int64_t count, int keep, uint64_t* __restrict__ out) {
  extern __shared__ uint64_t s[];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile;
  for (int t = threadIdx.x; t < kTile; t += kRankThreads) s[t] = base + t < count ? in[base + t] : kNoKey;
  bitonic_sort(s);
  for (int t = threadIdx.x; t < keep; t += kRankThreads) out[static_cast<int64_t>(blockIdx.x) * keep + t] = s[t];
}

}  // namespace

int64_t contact_rank_scratch_keys(int n, int k) {
  int keep = 1;
  while (keep < k) keep <<= 1;
  const int64_t tiles = (static_cast<int64_t>(n) * n + kTile - 1) / kTile;
  return 2 * tiles * keep;  // two ping-pong buffers of pass-0 output size
}

cudaError_t launch_contact_rank(const float* map, int n, int min_sep, int k, uint64_t* scratch, uint64_t* out_keys,
                                cudaStream_t s) {
  if (n <= 0 || k <= 0 || k > kTile / 2) return cudaErrorInvalidValue;
  int keep = 1;
  while (keep < k) keep <<= 1;
  static std::atomic<unsigned long long> configured{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = kTile * static_cast<int>(sizeof(uint64_t));
  if (dev >= 64 || !(configured.load(std::memory_order_acquire) & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(rank_map_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(rank_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured.fetch_or(1ull << dev, std::memory_order_release);
  }
  const int64_t tiles0 = (static_cast<int64_t>(n) * n + kTile - 1) / kTile;
  uint64_t* buf[2] = {scratch, scratch + tiles0 * keep};
  rank_map_kernel<<<static_cast<unsigned>(tiles0), kRankThreads, smem, s>>>(map, n, min_sep, keep, buf[0]);
  int64_t count = tiles0 * keep;
  int cur = 0;
  while (count > kTile) {
    const int64_t tiles = (count + kTile - 1) / kTile;
    rank_keys_kernel<<<static_cast<unsigned>(tiles), kRankThreads, smem, s>>>(buf[cur], count, keep, buf[cur ^ 1]);
    count = tiles * keep;
    cur ^= 1;
  }
  rank_keys_kernel<<<1, kRankThreads, smem, s>>>(buf[cur], count, keep, out_keys);
  return cudaGetLastError();
}

}  // namespace esm
