// Splice bookkeeping on the device: split(cached, new) of threadcut/match.py:33-48.
//
//   cached = A . B . C . (stale tail)        new = A . C . D
//   a  = min(lcp(cached, new), len(new) - 1)
//   candidates j in [a + 1, len(cached) - min_suffix] with cached[j : j + min_suffix] == new[a : a + min_suffix]
//   c_j = min(lcp(cached[j:], new[a:]), len(new) - a - 1); the first j with the largest c_j wins
//   (c_j >= min_suffix > 0 always beats the empty split (a, a, 0)).
//
// Integer work, bandwidth-bound on the token arrays: four small kernels on the caller's stream.
//   split_lcp_kernel:    first mismatch of cached/new (atomicMin over a grid-stride scan)
//   split_window_kernel: positions whose min_suffix-token window matches new[a:] (appended to a list)
//   split_extend_kernel: one CTA per candidate extends the match in 8192-token chunks (first
//                        mismatch by block reduction) and offers (c, -j) to a 64-bit atomicMax
//   split_finish_kernel: writes (a, c0, c) as three int64
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kSplitThreads = 256;
constexpr int kExtendThreads = 1024;

struct SplitWs {
  unsigned long long best;  // (c << 32) | (0xffffffff - j), 0 = no candidate
  int64_t first_diff;       // lcp(cached, new) (min over mismatching positions, m when none)
  int64_t a;                // min(first_diff, n_new - 1)
  unsigned int ncand;       // candidates found (list below may be shorter: capped at cap)
  unsigned int pad;
  int64_t cand[1];          // candidate starts j, `cap` entries
};

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
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
    if (p.cached[i] != p.fresh[i]) {
      atomicMin(reinterpret_cast<unsigned long long*>(&p.ws->first_diff), (unsigned long long)i);
      break;  // later mismatches of this thread are larger
    }
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
      if ((int64_t)slot < p.cap) p.ws->cand[slot] = j;
    }
  }
}

__global__ void __launch_bounds__(kExtendThreads) split_extend_kernel(SplitParams p) {
  __shared__ int64_t s_miss;
  const int64_t a = p.ws->a;
  const int64_t rest = p.n_new - a;
  const int64_t nc = p.ws->ncand < (unsigned int)p.cap ? p.ws->ncand : p.cap;
  const int32_t* needle = p.fresh + a;
  for (int64_t ci = blockIdx.x; ci < nc; ci += gridDim.x) {
    const int64_t j = p.ws->cand[ci];
    const int64_t lim = (p.n_cached - j) < rest ? (p.n_cached - j) : rest;  // lcp(cached[j:], rest) <= lim
    int64_t L = lim;
    constexpr int kPer = 8;  // tokens per thread per chunk (coalesced: token base + k*blockDim + tid)
    for (int64_t base = p.min_suffix; base < lim; base += (int64_t)kPer * kExtendThreads) {
      if (threadIdx.x == 0) s_miss = lim;
      __syncthreads();
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int64_t t = base + (int64_t)k * kExtendThreads + threadIdx.x;
        if (t < lim && p.cached[j + t] != needle[t]) {
          atomicMin(reinterpret_cast<unsigned long long*>(&s_miss), (unsigned long long)t);
          break;  // this thread's later positions are larger
        }
      }
      __syncthreads();
      const int64_t miss = s_miss;
      __syncthreads();  // s_miss is reset by the next chunk
      if (miss < lim) {
        L = miss;
        break;
      }
    }
    if (threadIdx.x == 0) {
      const int64_t c = L < rest - 1 ? L : rest - 1;
      const unsigned long long key = ((unsigned long long)c << 32) | (0xffffffffull - (unsigned long long)j);
      atomicMax(&p.ws->best, key);
    }
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
