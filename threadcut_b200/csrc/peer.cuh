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
// Region of each rank (zeroed at creation): [0, 256) control (word 0: this rank's count of
// completed sums, `seq`; read and advanced only by its own kernels), then the data
// [kArSlots][world][rows] of uint64 words. The sum number s uses slot s % kArSlots and epoch s + 1.
// Two slots suffice: a rank writes sum s + 2 into slot s % 2 of rank r only after its own sum s + 1
// has received r's rows of s + 1, which r sends after it finished reading sum s.
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kArSlots = 2;
constexpr int kArMaxWorld = 8;
constexpr int kArCtrlBytes = 256;
constexpr int kArRows = 16;          // GEMV rows per CTA (2 per warp)
constexpr int kArThreads = 256;
constexpr int kArNormThreads = 1024;
constexpr int kArMaxPerThread = 8;   // elements per thread of the summing kernel: hidden <= 8192

struct ArPeers {
  uint64_t* data[kArMaxWorld];  // rank p's data words as mapped in this process
  const unsigned int* seq;      // this rank's completed-sum count (its own region's control word)
  int world, rank;
  int64_t rows;                 // words per (slot, rank): the hidden size
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
// this rank), word 1 the count of this launch's finished CTAs, words 8 + 8*slot + src: the epoch
// (gather number + 1) of src's data in slot; then the data, [2 slots][world][gather_src_stride] fp32.
// Gather s uses slot s % 2: a rank pushes gather s + 2 into slot s % 2 of rank r only after its own
// gather s + 1 received r's data, which r pushed after it finished gather s (its reads of slot s % 2).
constexpr int kGmThreads = 256;
constexpr int kGmMergers = 64;

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

__device__ __forceinline__ void st_release_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid.x = (world - 1) pushers + kGmMergers mergers. Pusher i copies this rank's partials to rank
// (rank + 1 + i) % world and then raises that rank's flag for this rank; merger m waits for every
// other rank's flag in this rank's region and merges its share of the rows. The last CTA to finish
// advances seq. rows * d % 4 == 0.
template <typename T>
__global__ void __launch_bounds__(kGmThreads) gather_merge_kernel(const float* __restrict__ o_local,
                                                                  const float* __restrict__ lse_local,
                                                                  T* __restrict__ out, float* __restrict__ lse_out,
                                                                  int64_t rows, int d, int64_t out_stride,
                                                                  const __grid_constant__ GatherPeers gp) {
  __shared__ int s_ok;
  pdl_launch();
  pdl_wait();
  unsigned int* my_ctrl = gp.ctrl[gp.rank];
  const unsigned int s = my_ctrl[0];
  const unsigned int slot = s & 1u, ep = s + 1u;
  const int pushers = gp.world - 1;
  if ((int)blockIdx.x < pushers) {
    const int p = (gp.rank + 1 + (int)blockIdx.x) % gp.world;
    float* dst = gp.data[p] + slot * gp.slot_stride + (int64_t)gp.rank * gp.src_stride;
    const int64_t n4 = rows * d / 4;
    const float4* src4 = reinterpret_cast<const float4*>(o_local);
    float4* dst4 = reinterpret_cast<float4*>(dst);
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) dst4[i] = src4[i];
    for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) dst[rows * d + i] = lse_local[i];
    __syncthreads();  // every thread's stores precede the flag below
    if (threadIdx.x == 0) {
      __threadfence_system();
      st_release_sys_u32(gp.ctrl[p] + 8 + 8 * slot + gp.rank, ep);
    }
  } else {
    const int m = (int)blockIdx.x - pushers, nm = (int)gridDim.x - pushers;
    if (threadIdx.x == 0) {
      int ok = 1;
      for (int r = 0; r < gp.world; ++r) {
        if (r == gp.rank) continue;
        uint32_t spin = 0;
        while (ld_acquire_sys_u32(my_ctrl + 8 + 8 * slot + r) != ep) {
          if (++spin >= kSpinLimit / 64) {
            raise_error(TC_DEVERR_PEER_TIMEOUT);
            ok = 0;
            break;
          }
          __nanosleep(64);
        }
      }
      s_ok = ok;
    }
    __syncthreads();
    const float* mine = gp.data[gp.rank] + slot * gp.slot_stride;
    const int64_t r0 = rows * m / nm, r1 = rows * (m + 1) / nm;
    for (int64_t row = r0; row < r1; ++row) {
      // part r: this rank's own partial from its inputs, the others' from its region
      float M = -INFINITY;
      for (int r = 0; r < gp.world; ++r) {
        const float l = r == gp.rank ? lse_local[row] : __ldcg(mine + (int64_t)r * gp.src_stride + rows * d + row);
        M = fmaxf(M, l);
      }
      float L = 0.f;
      if (M != -INFINITY)
        for (int r = 0; r < gp.world; ++r) {
          const float l = r == gp.rank ? lse_local[row] : __ldcg(mine + (int64_t)r * gp.src_stride + rows * d + row);
          L += __expf(l - M);
        }
      for (int dd = threadIdx.x; dd < d; dd += blockDim.x) {
        float o = 0.f;
        if (M != -INFINITY)
          for (int r = 0; r < gp.world; ++r) {
            const bool own = r == gp.rank;
            const float l = own ? lse_local[row] : __ldcg(mine + (int64_t)r * gp.src_stride + rows * d + row);
            const float x = own ? o_local[row * d + dd] : __ldcg(mine + (int64_t)r * gp.src_stride + row * d + dd);
            o += __expf(l - M) * x;
          }
        out[row * out_stride + dd] = from_f32<T>(L > 0.f ? o / L : 0.f);
      }
      if (lse_out != nullptr && threadIdx.x == 0) lse_out[row] = L > 0.f ? M + __logf(L) : -INFINITY;
    }
    (void)s_ok;
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
