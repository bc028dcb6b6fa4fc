// Sums over the ranks of a tensor-parallel step without a collective library: one-shot all-reduce
// through peer memory (CUDA IPC mappings of every rank's receive region; plain loads and stores,
// no TMA, no multicast).
//
// The step's two sums per layer (after o_proj and after down_proj; threadcut_b200/tp.py) each
// follow a one-token GEMV whose rows are split over the CTAs. Here that GEMV writes its fp32 rows
// straight into every rank's receive region as 8-byte words (value, epoch): one store per row per
// rank, no flag after the data, so a row costs one NVLink trip. The next kernel of every rank then
// waits until the words of all ranks carry the current epoch, adds them in rank order (the same
// order on every rank, so every rank holds the same bits), rounds the sum to the model dtype (the
// projection's output dtype) and continues as tc_add_rmsnorm: residual add, RMSNorm.
//
// Region of each rank (zeroed at creation): [0, kArDataOffset) control (word 0: this rank's count
// of completed sums, `seq`; word 1: CTAs of the current residual sum done; at kArSsOffset the
// residual sum's per-CTA sums of squares, kArSsParts floats; all read and written only by this
// rank's kernels), then the data [kArSlots][world][rows] of uint64 words. The sum number s uses
// slot s % kArSlots and epoch s + 1. Two slots suffice: a rank writes sum s + 2 into slot s % 2 of
// rank r only after its own sum s + 1 has received r's rows of s + 1, which r sends after it
// finished reading sum s. (The residual form completes the sum inside the projection: its CTA c
// waits only for the other ranks' rows of c's own block, and the same argument holds block by
// block, every rank splitting the rows over its CTAs alike.)
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kArSlots = 2;
constexpr int kArMaxWorld = 8;
constexpr int kArCtrlBytes = 256;     // control bytes of a gather region (below)
constexpr int kArDataOffset = 2048;  // start of the words in a sum region
constexpr int kArSsOffset = 1024;    // the residual sum's per-CTA sums of squares in a sum region
constexpr int kArSsParts = 256;      // their count (CTAs of a residual sum; unused entries stay 0)
constexpr int kArRows = 16;          // GEMV rows per CTA (2 per warp)
constexpr int kArThreads = 256;
constexpr int kArNormThreads = 1024;
constexpr int kArMaxPerThread = 8;   // elements per thread of the summing kernel: hidden <= 8192

struct ArPeers {
  uint64_t* data[kArMaxWorld];  // rank p's data words as mapped in this process
  const unsigned int* seq;      // this rank's completed-sum count (its own region's control word)
  int world, rank;
  int64_t rows;                 // words per (slot, rank): the hidden size
  // residual form (h != null): the projection completes the sum itself, h[i] = T(h[i] + T(sum)),
  // writes each CTA's sum of squares of the new h to ss[blockIdx.x], and the last CTA done
  // (count in *done) advances *seq
  void* h;
  float* ss;
  unsigned int* done;
};

__device__ __forceinline__ void st_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// out rows [blockIdx.x * kArRows, +kArRows) of x [K] . w[N][K]^T, each sent to every rank as a
// (value, epoch) word. 16-bit T, K % 8 == 0, x and w 16-byte aligned. x staged in shared memory.
template <typename T, bool kSwiGLU = false>
__global__ void __launch_bounds__(kArThreads) gemv_allreduce_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                   int64_t N, int K, const __grid_constant__ ArPeers ar) {
  extern __shared__ uint4 xs[];
  __shared__ float res[kArRows];
  const int kc = K / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * kArRows;
  // this CTA's weight rows into L2 while the previous kernel finishes; x and seq only after the wait
  prefetch_rows_l2(w, row0 + warp, kArThreads / 32, row0 + kArRows < N ? row0 + kArRows : N, K, kArRows);
  pdl_launch();
  pdl_wait();
  stage_x<T, kSwiGLU>(xs, x, K);
  __syncthreads();
  constexpr int kWarps = kArThreads / 32, kRpw = kArRows / kWarps;  // rows per warp, streamed together
  float acc[kRpw];
  const uint4* wr[kRpw];
#pragma unroll
  for (int j = 0; j < kRpw; ++j) {
    const int64_t row = row0 + warp + j * kWarps;
    acc[j] = 0.f;
    wr[j] = reinterpret_cast<const uint4*>(w + (row < N ? row : 0) * (int64_t)K);
  }
#pragma unroll 4
  for (int c = lane; c < kc; c += 32) {
    const uint4 b = xs[c];
#pragma unroll
    for (int j = 0; j < kRpw; ++j) {
      const uint4 a = __ldg(wr[j] + c);
      acc[j] = dot2(a.x, b.x, acc[j], (T*)nullptr);
      acc[j] = dot2(a.y, b.y, acc[j], (T*)nullptr);
      acc[j] = dot2(a.z, b.z, acc[j], (T*)nullptr);
      acc[j] = dot2(a.w, b.w, acc[j], (T*)nullptr);
    }
  }
#pragma unroll
  for (int j = 0; j < kRpw; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    if (lane == 0) res[warp + j * kWarps] = acc[j];
  }
  __syncthreads();
  const unsigned int s = *ar.seq;
  const uint64_t ep = (uint64_t)(s + 1u) << 32;
  const int64_t slot_off = (int64_t)(s % kArSlots) * ar.world * ar.rows + (int64_t)ar.rank * ar.rows;
  const int nb = N - row0 < kArRows ? (int)(N - row0) : kArRows;
  // consecutive threads take consecutive rows of one destination: 128-byte runs per destination
  for (int idx = threadIdx.x; idx < ar.world * kArRows; idx += blockDim.x) {
    const int p = idx / kArRows, i = idx - p * kArRows;
    if (i < nb) st_sys_u64(ar.data[p] + slot_off + row0 + i, ep | __float_as_uint(res[i]));
  }
}

// After gemv_allreduce_kernel on every rank: delta = T(sum over ranks of their rows, in rank
// order), then exactly tc_add_rmsnorm: h = T(h + delta) in place, out = T(weight * T(h * rsqrt(
// mean(h^2) + eps))). One CTA; waits (bounded) for every rank's words of the current epoch and
// advances this rank's seq at the end. H <= kArNormThreads * kArMaxPerThread.
template <typename T>
__global__ void __launch_bounds__(kArNormThreads) allreduce_add_rmsnorm_kernel(
    T* __restrict__ h, const T* __restrict__ weight, T* __restrict__ out, int H, float inv_h, float eps,
    const uint64_t* __restrict__ mine, unsigned int* seq, int world, int64_t rows) {
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const unsigned int s = *seq;
  const uint32_t ep = s + 1u;
  const uint64_t* base = mine + (int64_t)(s % kArSlots) * world * rows;
  float hv[kArMaxPerThread];
  float ss = 0.f;
  bool ok = true;
#pragma unroll
  for (int j = 0; j < kArMaxPerThread; ++j) {
    const int i = threadIdx.x + j * kArNormThreads;
    hv[j] = 0.f;
    if (i < H) {
      float part[kArMaxWorld];
      uint32_t need = (1u << world) - 1u;  // ranks whose word of this epoch has not been seen
      uint32_t spin = 0;
      while (need) {
#pragma unroll
        for (int r = 0; r < kArMaxWorld; ++r) {
          if (need & (1u << r)) {
            const uint64_t wv = ld_sys_u64(base + (int64_t)r * rows + i);
            if ((uint32_t)(wv >> 32) == ep) {
              part[r] = __uint_as_float((uint32_t)wv);
              need &= ~(1u << r);
            }
          }
        }
        if (need && ++spin >= kSpinLimit / 64) {
          raise_error(TC_DEVERR_PEER_TIMEOUT);
          ok = false;
          break;
        }
        if (need) __nanosleep(64);
      }
      float sum = 0.f;
#pragma unroll
      for (int r = 0; r < kArMaxWorld; ++r)
        if (r < world) sum += (need & (1u << r)) ? 0.f : part[r];
      const T nh = from_f32<T>(to_f32(h[i]) + to_f32(from_f32<T>(sum)));
      h[i] = nh;
      hv[j] = to_f32(nh);
      ss += hv[j] * hv[j];
    }
  }
  (void)ok;
  ss = block_sum_f32(ss, red);
  const float rn = rsqrtf(ss * inv_h + eps);
#pragma unroll
  for (int j = 0; j < kArMaxPerThread; ++j) {
    const int i = threadIdx.x + j * kArNormThreads;
    if (i < H) out[i] = from_f32<T>(to_f32(weight[i]) * to_f32(from_f32<T>(hv[j] * rn)));
  }
  __syncthreads();  // every thread has read *seq and its words
  if (threadIdx.x == 0) *seq = s + 1u;
}

}  // namespace tc

namespace tc {

// ---- all-gather + log-sum-exp merge of sequence-shard partials through peer memory.
// Every rank holds, for `rows` query rows, the fp32 partial output o [rows][d] (normalised) and
// natural-log LSE [rows] of its token slice. One launch pushes them into every other rank's region
// and merges all ranks' partials into the output, in rank order, with the arithmetic of
// merge_partials_kernel (the merge of threadcut/flash_decode.py:68-69 over ranks).
//
// Region of each rank (zeroed at creation): [0, 256) control: word 0 `seq` (completed gathers of
// this rank), word 1 the count of this launch's finished CTAs, words 8 + 8*slot + src: arrivals of
// src's pusher CTAs in slot (kGmPushers per gather, never reset: gather s is complete when the count
// reaches (s / 2 + 1) * kGmPushers); then the data, [2 slots][world][gather_src_stride] fp32.
// Gather s uses slot s % 2: a rank pushes gather s + 2 into slot s % 2 of rank r only after its own
// gather s + 1 received r's data, which r pushed after it finished gather s (its reads of slot s % 2).
constexpr int kGmThreads = 256;
constexpr int kGmPushers = 8;   // CTAs pushing to one destination rank, each a slice of the data

// Floats per (slot, source) of a gather region: o [rows][d] then lse [rows], rounded up to a
// multiple of 4 floats so that every source's block starts 16-byte aligned (float4 stores).
__host__ __device__ __forceinline__ int64_t gather_src_stride(int64_t rows, int d) {
  return (rows * d + rows + 3) / 4 * 4;
}

struct GatherPeers {
  float* data[kArMaxWorld];          // rank p's data area as mapped in this process
  unsigned int* ctrl[kArMaxWorld];   // rank p's control words as mapped in this process
  int world, rank;
  int64_t src_stride;                // floats per (slot, source): gather_src_stride(rows, d)
  int64_t slot_stride;               // floats per slot: world * src_stride
};

__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add_u32(unsigned int* p, unsigned int v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// grid.x = (world - 1) * kGmPushers pushers + the mergers. Pusher CTA i copies slice i % kGmPushers
// of this rank's partials (o, then lse) to rank (rank + 1 + i / kGmPushers) % world and counts
// itself in there; each merger thread waits until every other rank's pushers have arrived in this
// rank's region, then merges one float4 of one row (its lse loads for all ranks and o loads in one
// batch). The last CTA to finish advances seq. rows * d % 4 == 0.
template <typename T>
__global__ void __launch_bounds__(kGmThreads) gather_merge_kernel(const float* __restrict__ o_local,
                                                                  const float* __restrict__ lse_local,
                                                                  T* __restrict__ out, float* __restrict__ lse_out,
                                                                  int64_t rows, int d, int64_t out_stride,
                                                                  const __grid_constant__ GatherPeers gp) {
  pdl_launch();
  pdl_wait();
  unsigned int* my_ctrl = gp.ctrl[gp.rank];
  const unsigned int s = my_ctrl[0];
  const unsigned int slot = s & 1u;
  const int pushers = (gp.world - 1) * kGmPushers;
  if ((int)blockIdx.x < pushers) {
    const int p = (gp.rank + 1 + (int)blockIdx.x / kGmPushers) % gp.world;
    const int part = (int)blockIdx.x % kGmPushers;
    float* dst = gp.data[p] + slot * gp.slot_stride + (int64_t)gp.rank * gp.src_stride;
    // the source block as float4s: o (rows * d / 4), then lse padded to the stride
    const int64_t n4 = rows * d / 4, nl = rows;
    const int64_t lo = n4 * part / kGmPushers, hi = n4 * (part + 1) / kGmPushers;
    const float4* src4 = reinterpret_cast<const float4*>(o_local);
    float4* dst4 = reinterpret_cast<float4*>(dst);
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst4[i] = src4[i];
    const int64_t l0 = nl * part / kGmPushers, l1 = nl * (part + 1) / kGmPushers;
    for (int64_t i = l0 + threadIdx.x; i < l1; i += blockDim.x) dst[rows * d + i] = lse_local[i];
    __syncthreads();  // every thread's stores precede the arrival below
    if (threadIdx.x == 0) {
      __threadfence_system();
      red_release_sys_add_u32(gp.ctrl[p] + 8 + 8 * slot + gp.rank, 1u);
    }
  } else {
    const int64_t m = (int64_t)blockIdx.x - pushers;
    const int64_t t = m * blockDim.x + threadIdx.x;  // (row, float4 column) of this thread
    const int q4 = d / 4;
    const unsigned int need = (s / 2u + 1u) * (unsigned int)kGmPushers;
    if (threadIdx.x == 0) {
      for (int r = 0; r < gp.world; ++r) {
        if (r == gp.rank) continue;
        uint32_t spin = 0;
        while (ld_acquire_sys_u32(my_ctrl + 8 + 8 * slot + r) < need) {
          if (++spin >= kSpinLimit / 64) {
            raise_error(TC_DEVERR_PEER_TIMEOUT);
            break;
          }
          __nanosleep(64);
        }
      }
    }
    __syncthreads();
    if (t < rows * q4) {
      const int64_t row = t / q4;
      const int c4 = (int)(t - row * q4);
      const float* mine = gp.data[gp.rank] + slot * gp.slot_stride;
      float l[kArMaxWorld];
      float4 x[kArMaxWorld];
#pragma unroll
      for (int r = 0; r < kArMaxWorld; ++r) {
        if (r < gp.world) {
          const bool own = r == gp.rank;
          const float* src = mine + (int64_t)r * gp.src_stride;
          l[r] = own ? lse_local[row] : __ldcg(src + rows * d + row);
          x[r] = own ? reinterpret_cast<const float4*>(o_local)[row * q4 + c4]
                     : __ldcg(reinterpret_cast<const float4*>(src) + row * q4 + c4);
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < kArMaxWorld; ++r)
        if (r < gp.world) M = fmaxf(M, l[r]);
      float L = 0.f;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      if (M != -INFINITY) {
#pragma unroll
        for (int r = 0; r < kArMaxWorld; ++r)
          if (r < gp.world) L += __expf(l[r] - M);
#pragma unroll
        for (int r = 0; r < kArMaxWorld; ++r) {
          if (r < gp.world) {
            const float wgt = __expf(l[r] - M);
            o.x += wgt * x[r].x;
            o.y += wgt * x[r].y;
            o.z += wgt * x[r].z;
            o.w += wgt * x[r].w;
          }
        }
      }
      T* orow = out + row * out_stride + 4 * c4;
      orow[0] = from_f32<T>(L > 0.f ? o.x / L : 0.f);
      orow[1] = from_f32<T>(L > 0.f ? o.y / L : 0.f);
      orow[2] = from_f32<T>(L > 0.f ? o.z / L : 0.f);
      orow[3] = from_f32<T>(L > 0.f ? o.w / L : 0.f);
      if (lse_out != nullptr && c4 == 0) lse_out[row] = L > 0.f ? M + __logf(L) : -INFINITY;
    }
  }
  // the last CTA of this launch advances seq (every CTA read it above)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(my_ctrl + 1, 1u) == gridDim.x - 1) {
      my_ctrl[1] = 0u;
      my_ctrl[0] = s + 1u;
    }
  }
}

}  // namespace tc

namespace tc {

// ---- split-K GEMV for long input rows (K >= kSplitKMin): a CTA owns kSkRows output rows and its 8
// warps split K into 8 contiguous slices, so every lane keeps kSkRows loads per column step in
// flight however few rows the matrix has. Measured (bf16, graph-timed, 4 distinct weights): the
// 2560 x 9728 down projection 21.8 -> 12.7 us, 2560 x 4096 6.12 -> 5.92 us; at K = 2560 the rows
// per warp of gemv_kernel are faster (19456 x 2560: 22.4 vs 37.0 us), hence the threshold. Per row: each lane sums its columns in order, the lanes by xor
// shuffles, the warps' sums in warp order through shared memory; fp32 throughout, one rounding.
// kAR: the rows go to every rank's region as (value, epoch) words instead of `out` (as
// gemv_allreduce_kernel). kSwiGLU: x is gate|up [2K], as stage_x.
constexpr int kSplitKMin = 4096;
constexpr int kSkRows = 8;

template <typename T, bool kSwiGLU, bool kAR>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_splitk_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                      T* __restrict__ out, int64_t N, int K,
                                                                      const __grid_constant__ ArPeers ar) {
  extern __shared__ uint4 xs[];
  __shared__ float part[kGemvWarps][kSkRows];
  __shared__ float res[kSkRows];
  const int kc = K / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * kSkRows;
  pdl_launch();
  pdl_wait();
  stage_x<T, kSwiGLU>(xs, x, K);
  __syncthreads();
  const int c0 = kc * warp / kGemvWarps, c1 = kc * (warp + 1) / kGemvWarps;
  const uint4* wr[kSkRows];
  float acc[kSkRows];
#pragma unroll
  for (int j = 0; j < kSkRows; ++j) {
    const int64_t row = row0 + j;
    wr[j] = reinterpret_cast<const uint4*>(w + (row < N ? row : N - 1) * (int64_t)K);
    acc[j] = 0.f;
  }
#pragma unroll 2
  for (int c = c0 + lane; c < c1; c += 32) {
    const uint4 b = xs[c];
#pragma unroll
    for (int j = 0; j < kSkRows; ++j) {
      const uint4 a = __ldg(wr[j] + c);
      acc[j] = dot2(a.x, b.x, acc[j], (T*)nullptr);
      acc[j] = dot2(a.y, b.y, acc[j], (T*)nullptr);
      acc[j] = dot2(a.z, b.z, acc[j], (T*)nullptr);
      acc[j] = dot2(a.w, b.w, acc[j], (T*)nullptr);
    }
  }
#pragma unroll
  for (int j = 0; j < kSkRows; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    if (lane == 0) part[warp][j] = acc[j];
  }
  __syncthreads();
  const int nb = N - row0 < kSkRows ? (int)(N - row0) : kSkRows;
  if (threadIdx.x < kSkRows) {
    float sum = 0.f;
#pragma unroll
    for (int ww = 0; ww < kGemvWarps; ++ww) sum += part[ww][threadIdx.x];
    if (!kAR && (int)threadIdx.x < nb) out[row0 + threadIdx.x] = from_f32<T>(sum);
    res[threadIdx.x] = sum;
  }
  if constexpr (kAR) {
    __syncthreads();
    const unsigned int s = *ar.seq;
    const uint64_t ep = (uint64_t)(s + 1u) << 32;
    const int64_t slot_off = (int64_t)(s % kArSlots) * ar.world * ar.rows + (int64_t)ar.rank * ar.rows;
    for (int idx = threadIdx.x; idx < ar.world * kSkRows; idx += blockDim.x) {
      const int p = idx / kSkRows, i = idx - p * kSkRows;
      if (i < nb) st_sys_u64(ar.data[p] + slot_off + row0 + i, ep | __float_as_uint(res[i]));
    }
  }
}

}  // namespace tc
