// Block-level exact top-k selection and small sorts.
#pragma once
#include "hc_common.cuh"

namespace hc {

// Shared memory needed by block_topk_flags (ints).
constexpr int kTopkSmemInts = 256 + 64;

// Marks sel[i] = 1 for the k largest x[i] (i < n) and 0 otherwise. Equal values prefer the
// lower index, so the selection is deterministic. Exact MSB radix select over the 32-bit
// order-preserving keys (4 passes of 8 bits), then one ordered pass that resolves the
// threshold ties with a block scan. `x` and `sel` may live in global or shared memory.
// All threads of the block must call; blockDim.x is a multiple of 32.
template <typename Getter>
__device__ void block_topk_flags(Getter x, int n, int k, uint8_t* sel, int* sh) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  if (k <= 0 || k >= n) {
    const uint8_t v = k > 0;
    for (int i = tid; i < n; i += nthr) sel[i] = v;
    __syncthreads();
    return;
  }
  int* hist = sh;          // 256
  int* misc = sh + 256;    // scratch for the scan and the digit search
  uint32_t prefix = 0, mask = 0;
  int kk = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += nthr) hist[b] = 0;
    __syncthreads();
    // scores cluster into few bins, so lanes of a warp that hit the same bin add once together
    for (int base = 0; base < n; base += nthr) {
      const int i = base + tid;
      const uint32_t key = i < n ? fkey(x(i)) : 0u;
      const bool live = i < n && (key & mask) == prefix;
      const unsigned act = __ballot_sync(0xffffffffu, live);
      if (live) {
        const uint32_t bin = (key >> shift) & 255u;
        const unsigned same = __match_any_sync(act, bin);
        if ((threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
      }
    }
    __syncthreads();
    if (tid < 32) {
      // lane l sums bins 255-8l .. 248-8l (descending), then a prefix scan over lanes
      int tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) tot += hist[255 - 8 * tid - j];
      int inc = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (tid >= o) inc += y;
      }
      const int excl = inc - tot;
      const unsigned hit = __ballot_sync(0xffffffffu, inc >= kk && excl < kk);
      const int owner = __ffs(hit) - 1;
      if (tid == owner) {
        int cum = excl, digit = 0;
        for (int j = 0; j < 8; ++j) {
          const int b = 255 - 8 * tid - j;
          if (cum + hist[b] >= kk) {
            digit = b;
            break;
          }
          cum += hist[b];
        }
        misc[0] = digit;
        misc[1] = kk - cum;
      }
    }
    __syncthreads();
    prefix |= (uint32_t)misc[0] << shift;
    mask |= 255u << shift;
    kk = misc[1];
    __syncthreads();
  }
  // prefix is the key of the k-th largest; kk of the elements equal to it are selected
  int running = 0;
  for (int base = 0; base < n; base += nthr) {
    const int i = base + tid;
    uint32_t key = 0;
    if (i < n) key = fkey(x(i));
    const int eq = (i < n && key == prefix) ? 1 : 0;
    int total;
    const int r = block_exclusive_scan(eq, misc, total);
    if (i < n) sel[i] = (key > prefix) || (eq && running + r < kk);
    running += total;
  }
  __syncthreads();
}

// block_topk_flags with a contiguous range of elements per thread: thread t owns
// [t * per, min(n, (t + 1) * per)), per = ceil(n / blockDim). The four radix passes read each
// thread's range; the elements equal to the threshold key are resolved in index order with a
// single block scan over the threads' counts, so the selection costs 4 + 1 block-wide steps
// instead of one scan per blockDim elements. Same result as block_topk_flags.
template <typename Getter>
__device__ void block_topk_ranges(Getter x, int n, int k, uint8_t* sel, int* sh) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int per = (n + nthr - 1) / nthr, r0 = min(n, tid * per), r1 = min(n, r0 + per);
  if (k <= 0 || k >= n) {
    const uint8_t v = k > 0;
    for (int i = r0; i < r1; ++i) sel[i] = v;
    __syncthreads();
    return;
  }
  int* hist = sh;          // 256
  int* misc = sh + 256;    // scratch for the scan and the digit search
  uint32_t prefix = 0, mask = 0;
  int kk = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += nthr) hist[b] = 0;
    __syncthreads();
    for (int i = r0; i < r1; ++i) {
      const uint32_t key = fkey(x(i));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid < 32) {
      // lane l sums bins 255-8l .. 248-8l (descending), then a prefix scan over lanes
      int tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) tot += hist[255 - 8 * tid - j];
      int inc = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (tid >= o) inc += y;
      }
      const int excl = inc - tot;
      const unsigned hit = __ballot_sync(0xffffffffu, inc >= kk && excl < kk);
      const int owner = __ffs(hit) - 1;
      if (tid == owner) {
        int cum = excl, digit = 0;
        for (int j = 0; j < 8; ++j) {
          const int b = 255 - 8 * tid - j;
          if (cum + hist[b] >= kk) {
            digit = b;
            break;
          }
          cum += hist[b];
        }
        misc[0] = digit;
        misc[1] = kk - cum;
      }
    }
    __syncthreads();
    prefix |= (uint32_t)misc[0] << shift;
    mask |= 255u << shift;
    kk = misc[1];
    __syncthreads();
  }
  // prefix is the key of the k-th largest; the first kk elements equal to it (index order) are
  // selected
  int eq = 0;
  for (int i = r0; i < r1; ++i) eq += fkey(x(i)) == prefix;
  int total;
  int before = block_exclusive_scan(eq, misc, total);
  for (int i = r0; i < r1; ++i) {
    const uint32_t key = fkey(x(i));
    bool take = key > prefix;
    if (key == prefix) take = before++ < kk;
    sel[i] = take;
  }
  __syncthreads();
}

// In-place bitonic sort of n (power of two, <= 2*blockDim) (key, id) pairs: key descending,
// id ascending among equal keys.
__device__ inline void block_sort_desc(uint32_t* key, int32_t* id, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = ((lo & size) == 0);  // this half sorts "descending" in our order
        const uint32_t ka = key[lo], kb = key[hi];
        const int32_t ia = id[lo], ib = id[hi];
        // a before b iff ka > kb or (ka == kb and ia < ib)
        const bool a_first = (ka > kb) || (ka == kb && ia < ib);
        if (a_first != up) {
          key[lo] = kb; key[hi] = ka;
          id[lo] = ib; id[hi] = ia;
        }
      }
      __syncthreads();
    }
  }
}

}  // namespace hc
