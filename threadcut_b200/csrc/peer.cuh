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
