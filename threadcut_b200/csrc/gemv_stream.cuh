// Streaming GEMV of the one-token projections: out[row] = x . w[row] for 16-bit w [N][K], one
// persistent CTA per SM, the CTA's contiguous block of weight rows streamed through a shared-memory
// ring by 1-D bulk copies (cp.async.bulk, mbarrier completion).
//
// The weights do not depend on the previous kernel, so the producer lane fills the whole ring
// BEFORE griddepcontrol.wait: with programmatic dependent launch the first ~190 KB per SM (the
// whole matrix for the tensor-parallel shards at 8 GPUs) are in shared memory by the time the
// previous kernel finishes; x (the previous kernel's output) is read after the wait.
//
// Rows: each stage holds rs = max(1, 16 KB / row bytes) whole rows. With at least 8 stage chunks per
// CTA, consumer warp j % 8 takes chunk j (8 stages consumed at once); with fewer, every consumer warp
// waits for every chunk and takes its rows whose index in the CTA's block is its warp number modulo
// 8, so a small block still spreads over all warps (measured: spreading the rows of large blocks
// too made the 19456 x 2560 projection 31 % slower, 24.5 vs 18.8 us). Each lane sums the row's
// 16-byte columns lane, lane + 32, ... in order and the lanes reduce by xor shuffles: the same order as gemv_kernel with one row per warp, so the result
// bits are those of tc_gemv's single-row pass. Epilogues: the row rounded to T into `out`, or (kAR)
// the fp32 row as a (value, epoch) word into every rank's region (as gemv_allreduce_kernel).
// kSwiGLU: x is gate|up [2K] and the staged input is the SwiGLU activation (stage_x).
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kGsConsumers = 8;                    // consumer warps (+1 producer warp)
constexpr int kGsThreads = 32 * (kGsConsumers + 1);
constexpr int kGsMaxStages = 16;
constexpr int kGsSmemBudget = 200 * 1024;          // x + ring, of the 227 KB a CTA may use
constexpr int kGsMaxRowsPerCta = 64;               // kAR: rows whose results are kept for the stores
constexpr int kGsStageBatch = 6;                   // x chunks per thread loaded before use (one batch: K <= 12288)

struct GsPlan {
  int rs;          // rows per stage
  int stage_bytes; // rs * K * 2
  int nstages;
  int x_bytes;     // K * 2 rounded up to 128
};

// budget: bytes of shared memory for x and the ring (at most kGsSmemBudget); a smaller budget lets
// two CTAs of consecutive projections share an SM, the next one loading while this one runs.
__host__ __device__ __forceinline__ GsPlan gs_plan(int K, int budget = kGsSmemBudget) {
  GsPlan g;
  const int row = K * 2;
  g.rs = row >= 16384 ? 1 : 16384 / row;
  g.stage_bytes = g.rs * row;
  g.x_bytes = (row + 127) / 128 * 128;
  int ns = (budget - g.x_bytes - 1024) / g.stage_bytes;
  if (ns < 1) ns = 1;
  g.nstages = ns > kGsMaxStages ? kGsMaxStages : ns;
  return g;
}

__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kGsConsumers) : "memory");
}

// The rows [r0, r1) of CTA c: an even split of N rows over gridDim.x CTAs.
template <typename T, bool kSwiGLU, bool kAR>
__global__ void __launch_bounds__(kGsThreads, 1) gemv_stream_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                    T* __restrict__ out, int64_t N, int K,
                                                                    const __grid_constant__ ArPeers ar,
                                                                    const GsPlan g) {
  extern __shared__ __align__(128) uint8_t gs_smem[];
  __shared__ uint64_t full[kGsMaxStages], empty[kGsMaxStages];
  __shared__ float res[kAR ? kGsMaxRowsPerCta : 1];
  uint4* xs = reinterpret_cast<uint4*>(gs_smem);
  uint8_t* ring = gs_smem + g.x_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = N * blockIdx.x / gridDim.x, r1 = N * (blockIdx.x + 1) / gridDim.x;
  const int nrows = (int)(r1 - r0);
  const int nchunks = (nrows + g.rs - 1) / g.rs;
  const int64_t row_bytes = (int64_t)K * 2;
  const bool spread = nchunks < kGsConsumers;  // rows of every chunk spread over all consumer warps
  if (threadIdx.x == 0) {
    for (int s = 0; s < g.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], spread ? kGsConsumers : 1);  // the warps that read the stage release it
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kGsConsumers) {
    // producer: the whole ring is filled before waiting for the previous kernel (weights are
    // constant), the rest as consumers free stages
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const char* base = reinterpret_cast<const char*>(w) + r0 * row_bytes;
      const int pre = nchunks < g.nstages ? nchunks : g.nstages;
      for (int j = 0; j < pre; ++j) {
        const int rows = nrows - j * g.rs < g.rs ? nrows - j * g.rs : g.rs;
        mbar_arrive_expect_tx(&full[j], (uint32_t)(rows * row_bytes));
        bulk_g2s(ring + j * g.stage_bytes, base + (int64_t)j * g.rs * row_bytes, (uint32_t)(rows * row_bytes),
                 &full[j], pol);
      }
      pdl_launch();
      for (int j = pre; j < nchunks; ++j) {
        const int s = j % g.nstages;
        if (!mbar_wait(&empty[s], ((j / g.nstages) - 1) & 1, TC_DEVERR_PIPE_TIMEOUT)) break;
        const int rows = nrows - j * g.rs < g.rs ? nrows - j * g.rs : g.rs;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(rows * row_bytes));
        bulk_g2s(ring + s * g.stage_bytes, base + (int64_t)j * g.rs * row_bytes, (uint32_t)(rows * row_bytes),
                 &full[s], pol);
      }
    } else {
      pdl_launch();
    }
    pdl_wait();  // every thread of the block waits before the kernel may end (nothing read here)
  } else {
    pdl_launch();
    pdl_wait();  // x is the previous kernel's output
    {
      // each thread issues the loads of up to kGsStageBatch of its 16-byte chunks before using any,
      // so staging x costs one L2 round trip per batch instead of one per chunk
      const int kc = K / 8;
      const uint4* xg = reinterpret_cast<const uint4*>(x);
      for (int base = threadIdx.x; base < kc; base += 32 * kGsConsumers * kGsStageBatch) {
        uint4 gv[kGsStageBatch], uv[kSwiGLU ? kGsStageBatch : 1];
#pragma unroll
        for (int u = 0; u < kGsStageBatch; ++u) {
          const int i = base + u * 32 * kGsConsumers;
          if (i < kc) {
            gv[u] = xg[i];
            if constexpr (kSwiGLU) uv[u] = reinterpret_cast<const uint4*>(x + K)[i];
          }
        }
#pragma unroll
        for (int u = 0; u < kGsStageBatch; ++u) {
          const int i = base + u * 32 * kGsConsumers;
          if (i < kc) {
            if constexpr (kSwiGLU) {
              const T* ge = reinterpret_cast<const T*>(&gv[u]);
              const T* ue = reinterpret_cast<const T*>(&uv[u]);
              uint4 o;
              T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
              for (int t = 0; t < 8; ++t) {
                const float gf = to_f32(ge[t]);
                const float act = to_f32(from_f32<T>(gf / (1.0f + expf(-gf))));
                oe[t] = from_f32<T>(act * to_f32(ue[t]));
              }
              xs[i] = o;
            } else {
              xs[i] = gv[u];
            }
          }
        }
      }
    }
    consumer_bar();
    const int kc = K / 8;
    for (int j = spread ? 0 : warp; j < nchunks; j += spread ? 1 : kGsConsumers) {
      const int s = j % g.nstages;
      if (!mbar_wait(&full[s], (j / g.nstages) & 1, TC_DEVERR_PIPE_TIMEOUT)) break;
      const uint4* st = reinterpret_cast<const uint4*>(ring + s * g.stage_bytes);
      const int rows = nrows - j * g.rs < g.rs ? nrows - j * g.rs : g.rs;
      // spread: this warp's rows of the chunk are block rows j * rs + rr with (j * rs + rr) % 8 ==
      // warp; otherwise all rows of its chunk
      const int first = spread ? ((warp - (j * g.rs) % kGsConsumers) + kGsConsumers) % kGsConsumers : 0;
      for (int rr = first; rr < rows; rr += spread ? kGsConsumers : 1) {
        const uint4* wr = st + (int64_t)rr * kc;
        float acc = 0.f;
#pragma unroll 8
        for (int c = lane; c < kc; c += 32) {
          const uint4 a = wr[c];
          const uint4 b = xs[c];
          acc = dot2(a.x, b.x, acc, (T*)nullptr);
          acc = dot2(a.y, b.y, acc, (T*)nullptr);
          acc = dot2(a.z, b.z, acc, (T*)nullptr);
          acc = dot2(a.w, b.w, acc, (T*)nullptr);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        const int local = j * g.rs + rr;
        if (lane == 0) {
          if constexpr (kAR)
            res[local] = acc;
          else
            out[r0 + local] = from_f32<T>(acc);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if constexpr (kAR) {
      consumer_bar();  // every row's result is in res
      const unsigned int sq = *ar.seq;
      const uint64_t ep = (uint64_t)(sq + 1u) << 32;
      const int64_t slot_off = (int64_t)(sq % kArSlots) * ar.world * ar.rows + (int64_t)ar.rank * ar.rows;
      for (int idx = threadIdx.x; idx < ar.world * nrows; idx += 32 * kGsConsumers) {
        const int p = idx / nrows, i = idx - p * nrows;
        st_sys_u64(ar.data[p] + slot_off + r0 + i, ep | __float_as_uint(res[i]));
      }
    }
  }
}

}  // namespace tc
