// Streaming GEMV of the one-token projections: out[row] = x . w[row] for 16-bit w [N][K], one
// persistent CTA per SM, the CTA's contiguous block of weight rows streamed through a shared-memory
// ring by 1-D bulk copies (cp.async.bulk, mbarrier completion).
//
// The weights do not depend on the previous kernel, so the producer lane starts the first
// kGsPreWait stages BEFORE griddepcontrol.wait (with programmatic dependent launch they arrive while
// the previous kernel finishes) and the rest of the ring after it; x (the previous kernel's output)
// is read after the wait.
//
// Rows: each stage holds rs = max(1, 16 KB / row bytes) whole rows. With at least 8 stage chunks per
// CTA, consumer warp j % 8 takes chunk j (8 stages consumed at once); with fewer, every consumer warp
// waits for every chunk and takes its rows whose index in the CTA's block is its warp number modulo
// 8, so a small block still spreads over all warps (measured: spreading the rows of large blocks
// too made the 19456 x 2560 projection 31 % slower, 24.5 vs 18.8 us). Each lane sums the row's
// 16-byte columns lane, lane + 32, ... in order and the lanes reduce by xor shuffles: the same order as gemv_kernel with one row per warp, so the result
// bits are those of tc_gemv's single-row pass. Epilogues: the row rounded to T into `out`, or (kAR)
// the fp32 row as a (value, epoch) word into every rank's region (as gemv_allreduce_kernel); in
// the residual form (ar.h set) the CTA then waits for the other ranks' words of its own rows, adds
// them in rank order into the residual h (h = T(h + T(sum)), the arithmetic of
// tc_allreduce_add_rmsnorm) and records its rows' sum of squares of the new h, so that no separate
// summing kernel runs.
// Inputs: x [K]; kSwiGLU: x is gate|up [2K] and the staged input is the SwiGLU activation
// (stage_x); kNormIn: the staged input is RMSNorm(h) * weight, its 1/rms computed from the sums of
// squares a residual-form projection recorded (ni.ss; every CTA adds them in the same order).
// kActOut (the gate/up projection of the MLP, its rows interleaved: row 2i the gate row of
// intermediate i, row 2i + 1 its up row): each CTA holds whole pairs, keeps its rows rounded to T
// in shared memory and writes out[i] = T(T(silu(gate_i)) * up_i), silu_mul_kernel's arithmetic, so
// that the down projection stages a plain input: the activation is computed once per element
// instead of by every CTA of the down projection.
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kGsConsumers = 8;                    // consumer warps (+1 producer warp)
constexpr int kGsThreads = 32 * (kGsConsumers + 1);
constexpr int kGsMaxStages = 16;
constexpr int kGsSmemBudget = 200 * 1024;          // x + ring, of the 227 KB a CTA may use
constexpr int kGsMaxRowsPerCta = 64;               // kAR: rows whose results are kept for the stores
constexpr int kGsMaxActRows = 256;                 // kActOut: rows (gate/up pairs x 2) per CTA
constexpr int kGsStageBatch = 6;                   // x chunks per thread loaded before use (one batch: K <= 12288)
// Stages the producer fills before griddepcontrol.wait. Filling the whole ring early (up to
// ~190 KB per SM as soon as the CTA is resident) competes with the previous kernel's last CTAs for
// HBM and delays its end: measured over the tensor-parallel step's projection chain (36 layers,
// graph-timed) whole ring 54.6 us/layer at 1 GPU and 21.0 at the 8-GPU shapes, 4 stages 51.4 /
// 20.7, none 50.7 / 20.0, 2 stages 49.4 / 19.8; the same 2 stages as L2 prefetches instead 52.3 / 20.2.
constexpr int kGsPreWait = 2;

// kNormIn: x = T(weight * T(h * rsqrt(sum(ss) * inv_h + eps))), ss the kArSsParts partial sums of
// squares of h written by the residual-form projection before (unused entries 0).
struct NormIn {
  const void* h;
  const void* weight;
  const float* ss;
  float inv_h, eps;
};

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
template <typename T, bool kSwiGLU, bool kAR, bool kNormIn, bool kActOut = false>
__global__ void __launch_bounds__(kGsThreads, 1) gemv_stream_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                    T* __restrict__ out, int64_t N, int K,
                                                                    const __grid_constant__ ArPeers ar,
                                                                    const GsPlan g,
                                                                    const __grid_constant__ NormIn ni) {
  extern __shared__ __align__(128) uint8_t gs_smem[];
  __shared__ uint64_t full[kGsMaxStages], empty[kGsMaxStages];
  __shared__ float res[kAR ? kGsMaxRowsPerCta : (kActOut ? kGsMaxActRows : 1)];
  __shared__ float red[kGsConsumers];
  uint4* xs = reinterpret_cast<uint4*>(gs_smem);
  uint8_t* ring = gs_smem + g.x_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // kActOut: an even split of the N / 2 row pairs
  const int64_t r0 = kActOut ? 2 * ((N / 2) * blockIdx.x / gridDim.x) : N * blockIdx.x / gridDim.x;
  const int64_t r1 = kActOut ? 2 * ((N / 2) * (blockIdx.x + 1) / gridDim.x) : N * (blockIdx.x + 1) / gridDim.x;
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
    // producer: kGsPreWait stages before waiting for the previous kernel (weights are constant),
    // the rest of the ring after it, then each stage again as the consumers free it
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const char* base = reinterpret_cast<const char*>(w) + r0 * row_bytes;
      int pre = nchunks < g.nstages ? nchunks : g.nstages;
      if (pre > kGsPreWait) pre = kGsPreWait;
      for (int j = 0; j < pre; ++j) {
        const int rows = nrows - j * g.rs < g.rs ? nrows - j * g.rs : g.rs;
        mbar_arrive_expect_tx(&full[j], (uint32_t)(rows * row_bytes));
        bulk_g2s(ring + j * g.stage_bytes, base + (int64_t)j * g.rs * row_bytes, (uint32_t)(rows * row_bytes),
                 &full[j], pol);
      }
      pdl_launch();
      pdl_wait();  // the rest of the ring only once the previous kernel is done (see kGsPreWait)
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
    // residual form: this sum's number and this thread's residual element, loaded now so that the
    // epilogue does not wait for them
    unsigned int sq_pre = 0u;
    float h_pre = 0.f;
    if constexpr (kAR) {
      sq_pre = *ar.seq;
      if (ar.h != nullptr && (int)threadIdx.x < nrows) h_pre = to_f32(static_cast<const T*>(ar.h)[r0 + threadIdx.x]);
    }
    {
      // each thread issues the loads of up to kGsStageBatch of its 16-byte chunks before using any,
      // so staging x costs one L2 round trip per batch instead of one per chunk
      const int kc = K / 8;
      float rn = 0.f;
      float sv[kNormIn ? kArSsParts / 32 : 1];
      if constexpr (kNormIn) {
#pragma unroll
        for (int q = 0; q < kArSsParts / 32; ++q) sv[q] = ni.ss[lane + 32 * q];
      }
      const uint4* xg = reinterpret_cast<const uint4*>(kNormIn ? ni.h : static_cast<const void*>(x));
      const uint4* nw = reinterpret_cast<const uint4*>(ni.weight);
      constexpr int kStride = 32 * kGsConsumers * kGsStageBatch;
      // every consumer thread runs the first pass (the 1/rms reduction below needs whole warps)
      for (int base = threadIdx.x;; base += kStride) {
        uint4 gv[kGsStageBatch], uv[(kSwiGLU || kNormIn) ? kGsStageBatch : 1];
#pragma unroll
        for (int u = 0; u < kGsStageBatch; ++u) {
          const int i = base + u * 32 * kGsConsumers;
          if (i < kc) {
            gv[u] = xg[i];
            if constexpr (kSwiGLU) uv[u] = reinterpret_cast<const uint4*>(x + K)[i];
            if constexpr (kNormIn) uv[u] = nw[i];
          }
        }
        if constexpr (kNormIn) {
          if (base == (int)threadIdx.x) {
            // 1/rms of h: lane l adds parts l, l + 32, ... in order, then a xor butterfly (every
            // warp of every CTA computes the same value)
            float t = 0.f;
#pragma unroll
            for (int q = 0; q < kArSsParts / 32; ++q) t += sv[q];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            rn = rsqrtf(t * ni.inv_h + ni.eps);
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
            } else if constexpr (kNormIn) {
              // the arithmetic of add_rmsnorm_kernel's output: T(weight * T(h * rn))
              const T* he = reinterpret_cast<const T*>(&gv[u]);
              const T* we = reinterpret_cast<const T*>(&uv[u]);
              uint4 o;
              T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
              for (int t = 0; t < 8; ++t) oe[t] = from_f32<T>(to_f32(we[t]) * to_f32(from_f32<T>(to_f32(he[t]) * rn)));
              xs[i] = o;
            } else {
              xs[i] = gv[u];
            }
          }
        }
        if (base + kStride >= kc) break;
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
          else if constexpr (kActOut)
            res[local] = to_f32(from_f32<T>(acc));  // the projection's output, rounded as stored
          else
            out[r0 + local] = from_f32<T>(acc);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if constexpr (kActOut) {
      consumer_bar();  // every row's result is in res
      for (int i = threadIdx.x; 2 * i < nrows; i += 32 * kGsConsumers) {
        const float gf = res[2 * i];
        const float act = to_f32(from_f32<T>(gf / (1.0f + expf(-gf))));
        out[r0 / 2 + i] = from_f32<T>(act * res[2 * i + 1]);
      }
    }
    if constexpr (kAR) {
      consumer_bar();  // every row's result is in res
      const unsigned int sq = sq_pre;
      const uint64_t ep = (uint64_t)(sq + 1u) << 32;
      const int64_t slot = (int64_t)(sq % kArSlots) * ar.world * ar.rows;
      const int64_t slot_off = slot + (int64_t)ar.rank * ar.rows;
      if (ar.world > 1 || ar.h == nullptr) {
        for (int idx = threadIdx.x; idx < ar.world * nrows; idx += 32 * kGsConsumers) {
          const int p = idx / nrows, i = idx - p * nrows;
          st_sys_u64(ar.data[p] + slot_off + r0 + i, ep | __float_as_uint(res[i]));
        }
      }
      if (ar.h != nullptr) {
        // residual form: the sum of this CTA's rows over the ranks (rank order), into h
        T* hh = static_cast<T*>(ar.h);
        float sq2 = 0.f;
        const int i = threadIdx.x;  // at most kGsMaxRowsPerCta rows: one per consumer thread
        if (i < nrows) {
          const uint64_t* mine = ar.data[ar.rank] + slot + r0 + i;
          uint64_t wv[kArMaxWorld];
#pragma unroll
          for (int r = 0; r < kArMaxWorld; ++r)
            if (r < ar.world && r != ar.rank) wv[r] = ld_sys_u64(mine + (int64_t)r * ar.rows);
          float sum = 0.f;
#pragma unroll
          for (int r = 0; r < kArMaxWorld; ++r) {
            if (r >= ar.world) continue;
            float v = res[i];
            if (r != ar.rank) {
              uint32_t spin = 0;
              while ((uint32_t)(wv[r] >> 32) != (uint32_t)(sq + 1u)) {
                if (++spin >= kSpinLimit / 64) {
                  raise_error(TC_DEVERR_PEER_TIMEOUT);
                  wv[r] = ep;  // value 0
                  break;
                }
                __nanosleep(64);
                wv[r] = ld_sys_u64(mine + (int64_t)r * ar.rows);
              }
              v = __uint_as_float((uint32_t)wv[r]);
            }
            sum += v;
          }
          const T nh = from_f32<T>(h_pre + to_f32(from_f32<T>(sum)));
          hh[r0 + i] = nh;
          sq2 = to_f32(nh) * to_f32(nh);
        }
        // the CTA's sum of squares, in a fixed order: each warp's xor butterfly, then the warps in order
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq2 += __shfl_xor_sync(0xffffffffu, sq2, o);
        if (lane == 0) red[warp] = sq2;
        consumer_bar();  // also: every consumer thread has read *ar.seq and its words
        if (threadIdx.x == 0) {
          float t = 0.f;
#pragma unroll
          for (int q = 0; q < kGsConsumers; ++q) t += red[q];
          ar.ss[blockIdx.x] = t;
          if (ar.world > 1) {
            __threadfence();
            const unsigned int prev = atomicAdd(ar.done, 1u);
            if (prev == gridDim.x - 1) {  // the last CTA: every CTA has read seq; the sum is complete
              *ar.done = 0u;
              *const_cast<unsigned int*>(ar.seq) = sq + 1u;
            }
          }
        }
      }
    }
  }
}

}  // namespace tc
