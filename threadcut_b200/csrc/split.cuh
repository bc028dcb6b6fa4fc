// Splice bookkeeping on the device: split(cached, new) of threadcut/match.py:33-48.
//
//   cached = A . B . C . (stale tail)        new = A . C . D
//   a  = min(lcp(cached, new), len(new) - 1)
//   candidates j in [a + 1, len(cached) - min_suffix] with cached[j : j + min_suffix] == new[a : a + min_suffix]
//   c_j = min(lcp(cached[j:], new[a:]), len(new) - a - 1); the first j with the largest c_j wins
//   (c_j >= min_suffix > 0 always beats the empty split (a, a, 0)).
//
// Integer work on small token arrays, so latency-bound: five small kernels on the caller's stream.
//   split_lcp_kernel:    first mismatch of cached/new (grid-stride scan, block minimum, one
//                        atomicMin per block: past the common prefix nearly every position differs)
//   split_window_kernel: positions whose min_suffix-token window matches new[a:] (appended to a list)
//   split_extend_kernel: each candidate's match range is cut into kExtendParts parts, one block per
//                        (candidate, part) finds the first mismatch in its part and atomicMins it
//                        into the candidate's slot
//   split_best_kernel:   c_j = min(first mismatch, rest - 1) per candidate, offered as (c, -j) to a
//                        64-bit atomicMax
//   split_finish_kernel: writes (a, c0, c) as three int64
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kSplitThreads = 256;
constexpr int kExtendThreads = 256;
constexpr int kExtendParts = 64;  // blocks per candidate in split_extend_kernel

struct SplitWs {
  unsigned long long best;  // (c << 32) | (0xffffffff - j), 0 = no candidate
  int64_t first_diff;       // lcp(cached, new) (min over mismatching positions, m when none)
  int64_t a;                // min(first_diff, n_new - 1)
  unsigned int ncand;       // candidates found (list below may be shorter: capped at cap)
  unsigned int pad;
  int64_t cand[1];          // candidate starts j, `cap` entries, then `cap` first-mismatch slots
};

// First-mismatch slot of candidate ci (offset from j within the new request's rest), after the list.
__device__ __forceinline__ unsigned long long* split_miss(SplitWs* ws, int64_t cap, int64_t ci) {
  return reinterpret_cast<unsigned long long*>(ws->cand + cap) + ci;
}

// Minimum of v over the block (every thread calls it; kSplitThreads-or-fewer warps).
__device__ __forceinline__ unsigned long long block_min_u64(unsigned long long v) {
  __shared__ unsigned long long s_min[32];
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w < v ? w : v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();  // s_min may still be read by a previous call
  if (lane == 0) s_min[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < nw ? s_min[lane] : ~0ull;
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
      v = w < v ? w : v;
    }
  }
  return v;  // valid in thread 0
}

struct SplitParams {
  const int32_t* cached;
  const int32_t* fresh;  // the new request's tokens
  int64_t n_cached, n_new;
  int min_suffix;
  int suffix;
  int64_t cap;      // capacity of the candidate list
  SplitWs* ws;
  int64_t* out;     // [3]: a, c0, c
};

__global__ void split_init_kernel(SplitParams p) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    p.ws->best = 0ull;
    p.ws->first_diff = p.n_cached < p.n_new ? p.n_cached : p.n_new;
    p.ws->ncand = 0u;
  }
}

__global__ void __launch_bounds__(kSplitThreads) split_lcp_kernel(SplitParams p) {
  const int64_t m = p.n_cached < p.n_new ? p.n_cached : p.n_new;
  unsigned long long first = ~0ull;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
    if (p.cached[i] != p.fresh[i]) {
      first = (unsigned long long)i;
      break;  // later mismatches of this thread are larger
    }
  first = block_min_u64(first);
  if (threadIdx.x == 0 && first != ~0ull)
    atomicMin(reinterpret_cast<unsigned long long*>(&p.ws->first_diff), first);
}

__global__ void __launch_bounds__(kSplitThreads) split_window_kernel(SplitParams p) {
  const int64_t lcp = p.ws->first_diff;
  const int64_t a = lcp < p.n_new - 1 ? lcp : p.n_new - 1;
  if (blockIdx.x == 0 && threadIdx.x == 0) p.ws->a = a;
  const int64_t rest = p.n_new - a;
  if (!p.suffix || rest <= p.min_suffix || p.n_cached - (a + 1) < p.min_suffix) return;
  const int32_t* needle = p.fresh + a;
  const int64_t last = p.n_cached - p.min_suffix;  // inclusive
  for (int64_t j = a + 1 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j <= last;
       j += (int64_t)gridDim.x * blockDim.x) {
    bool ok = true;
    for (int t = 0; t < p.min_suffix && ok; ++t) ok = p.cached[j + t] == needle[t];
    if (ok) {
      const unsigned int slot = atomicAdd(&p.ws->ncand, 1u);
      if ((int64_t)slot < p.cap) {
        p.ws->cand[slot] = j;
        *split_miss(p.ws, p.cap, slot) = ~0ull;  // no mismatch found yet
      }
    }
  }
}

__global__ void __launch_bounds__(kExtendThreads) split_extend_kernel(SplitParams p) {
  const int64_t a = p.ws->a;
  const int64_t rest = p.n_new - a;
  const int64_t nc = p.ws->ncand < (unsigned int)p.cap ? p.ws->ncand : p.cap;
  const int32_t* needle = p.fresh + a;
  for (int64_t w = blockIdx.x; w < nc * kExtendParts; w += gridDim.x) {  // uniform over the block
    const int64_t ci = w / kExtendParts;
    const int part = (int)(w - ci * kExtendParts);
    const int64_t j = p.ws->cand[ci];
    const int64_t lim = (p.n_cached - j) < rest ? (p.n_cached - j) : rest;  // lcp(cached[j:], rest) <= lim
    const int64_t span = lim - p.min_suffix;                                // the window matched already
    const int64_t len = span > 0 ? (span + kExtendParts - 1) / kExtendParts : 0;
    const int64_t lo = p.min_suffix + part * len;
    const int64_t hi = lo + len < lim ? lo + len : lim;
    unsigned long long first = ~0ull;
    for (int64_t t = lo + threadIdx.x; t < hi; t += blockDim.x)
      if (p.cached[j + t] != needle[t]) {
        first = (unsigned long long)t;
        break;
      }
    first = block_min_u64(first);
    if (threadIdx.x == 0 && first != ~0ull) atomicMin(split_miss(p.ws, p.cap, ci), first);
  }
}

__global__ void __launch_bounds__(kSplitThreads) split_best_kernel(SplitParams p) {
  const int64_t a = p.ws->a;
  const int64_t rest = p.n_new - a;
  const int64_t nc = p.ws->ncand < (unsigned int)p.cap ? p.ws->ncand : p.cap;
  for (int64_t ci = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; ci < nc; ci += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = p.ws->cand[ci];
    const int64_t lim = (p.n_cached - j) < rest ? (p.n_cached - j) : rest;
    const unsigned long long miss = *split_miss(p.ws, p.cap, ci);
    const int64_t L = miss < (unsigned long long)lim ? (int64_t)miss : lim;  // lcp(cached[j:], rest)
    const int64_t c = L < rest - 1 ? L : rest - 1;
    const unsigned long long key = ((unsigned long long)c << 32) | (0xffffffffull - (unsigned long long)j);
    atomicMax(&p.ws->best, key);
  }
}

__global__ void split_finish_kernel(SplitParams p) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int64_t a = p.ws->a;
    const unsigned long long best = p.ws->best;
    if (best == 0ull) {
      p.out[0] = a;
      p.out[1] = a;
      p.out[2] = 0;
    } else {
      p.out[0] = a;
      p.out[1] = (int64_t)(0xffffffffull - (best & 0xffffffffull));
      p.out[2] = (int64_t)(best >> 32);
    }
  }
}

}  // namespace tc
