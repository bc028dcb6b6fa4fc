// Small per-token ops of the tensor-parallel decode step (threadcut_b200/tp.py), one launch each,
// in place of the chains of torch ops of transformers' Qwen3 layer (modeling_qwen3.py):
//   add_rmsnorm_kernel:  h = h + delta (rounded to T), x = Qwen3RMSNorm(h): fp32 mean of squares
//                        (sum times the host-computed 1/H, as torch's mean), rsqrt, cast to T, times
//                        the weight (rounded to T). One CTA per row.
//   qk_norm_rope_kernel: per head (q_norm / k_norm, then apply_rotary_pos_emb): RMSNorm over d, then
//                        x*cos + rotate_half(x)*sin with each product and the sum rounded to T, as
//                        the torch ops round. In place; one CTA per head, one thread per element.
//   silu_mul_kernel:     act(gate) * up for Qwen3MLP, with gate and up side by side in one row
//                        (the output of the fused gate/up projection); silu rounded to T first.
//   gemv_kernel:         the step's projections (one token: x [K] times w [N][K]^T), HBM-bound.
// They move a few KB per token: launch latency, not bandwidth, is what they save.
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kNormThreads = 256;

// Sum of v over the block (blockDim.x a multiple of 32, at most 1024); red holds 32 floats.
__device__ __forceinline__ float block_sum_f32(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // red may still be read by an earlier call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(T* __restrict__ h, const T* __restrict__ delta,
                                                                   const T* __restrict__ w, T* __restrict__ x,
                                                                   int H, float inv_h, float eps) {
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const int64_t off = (int64_t)blockIdx.x * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = to_f32(h[off + i]);
    if (delta != nullptr) {
      const T s = from_f32<T>(v + to_f32(delta[off + i]));
      h[off + i] = s;
      v = to_f32(s);
    }
    ss += v * v;
  }
  ss = block_sum_f32(ss, red);
  const float r = rsqrtf(ss * inv_h + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const T y = from_f32<T>(to_f32(h[off + i]) * r);
    x[off + i] = from_f32<T>(to_f32(w[i]) * to_f32(y));
  }
}

// 16-bit T only: H % 8 == 0 and H / 8 <= kNormThreads * MAXC. Same arithmetic as add_rmsnorm_kernel,
// with 16-byte loads and the row kept in registers between the two passes.
template <typename T, int MAXC>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_vec_kernel(T* __restrict__ h,
                                                                       const T* __restrict__ delta,
                                                                       const T* __restrict__ w, T* __restrict__ x,
                                                                       int H, float inv_h, float eps) {
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const int64_t off = (int64_t)blockIdx.x * (H / 8);
  uint4* hr = reinterpret_cast<uint4*>(h) + off;
  const uint4* dr = delta != nullptr ? reinterpret_cast<const uint4*>(delta) + off : nullptr;
  const int hc = H / 8;
  uint4 hv[MAXC];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < MAXC; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < hc) {
      hv[j] = hr[c];
      T* e = reinterpret_cast<T*>(&hv[j]);
      if (dr != nullptr) {
        const uint4 dv = dr[c];
        const T* de = reinterpret_cast<const T*>(&dv);
#pragma unroll
        for (int t = 0; t < 8; ++t) e[t] = from_f32<T>(to_f32(e[t]) + to_f32(de[t]));
        hr[c] = hv[j];
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float v = to_f32(e[t]);
        ss += v * v;
      }
    }
  }
  ss = block_sum_f32(ss, red);
  const float r = rsqrtf(ss * inv_h + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* xr = reinterpret_cast<uint4*>(x) + off;
#pragma unroll
  for (int j = 0; j < MAXC; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < hc) {
      const uint4 wv = wr[c];
      const T* we = reinterpret_cast<const T*>(&wv);
      const T* e = reinterpret_cast<const T*>(&hv[j]);
      uint4 ov;
      T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
      for (int t = 0; t < 8; ++t) oe[t] = from_f32<T>(to_f32(we[t]) * to_f32(from_f32<T>(to_f32(e[t]) * r)));
      xr[c] = ov;
    }
  }
}

// out[row] = sum_k x[k] * w[row][k] for a one-row x (the decode step's projections): 16-bit T,
// K % 8 == 0, x and w 16-byte aligned. x is staged in shared memory; each warp streams whole weight
// rows with 16-byte non-coherent loads (the weights are read once per step) and reduces across
// lanes; fp32 accumulation, one rounding to T, as a library GEMM does.
constexpr int kGemvWarps = 8;

__device__ __forceinline__ float dot2(uint32_t a, uint32_t b, float acc, __nv_bfloat16*) {
  const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a));
  const float2 fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b));
  return fmaf(fa.y, fb.y, fmaf(fa.x, fb.x, acc));
}
__device__ __forceinline__ float dot2(uint32_t a, uint32_t b, float acc, __half*) {
  const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&a));
  const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&b));
  return fmaf(fa.y, fb.y, fmaf(fa.x, fb.x, acc));
}

// L2 prefetch of weight rows (the constant operand of a GEMV) before the wait for the previous
// kernel: at most `count` rows row0, row0 + stride, ... below N, one bulk prefetch of K * 2 bytes per
// row, issued by lane 0 of the calling warp. K * 2 is a multiple of 16 and the rows are 16-byte
// aligned. Only the first rows of a warp are worth it: the wait is short, and prefetching a whole
// large projection would only evict what the step reads next.
__device__ __forceinline__ void prefetch_rows_l2(const void* w, int64_t row0, int64_t stride, int64_t N, int K,
                                                 int count) {
  if ((threadIdx.x & 31) != 0) return;
  for (int64_t row = row0; row < N && count > 0; row += stride, --count) {
    const char* r = static_cast<const char*>(w) + row * (int64_t)K * 2;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(r), "r"((uint32_t)K * 2) : "memory");
  }
}

// The GEMV's x staged in shared memory as K/8 16-byte chunks. kSwiGLU: x is Qwen3MLP's activation
// computed on the fly from gate|up [2K] (the fused gate/up projection's output): chunk i holds
// T(T(silu(gate)) * up) for its 8 elements, exactly silu_mul_kernel's rounding.
template <typename T, bool kSwiGLU>
__device__ __forceinline__ void stage_x(uint4* xs, const T* __restrict__ x, int K) {
  const int kc = K / 8;
  for (int i = threadIdx.x; i < kc; i += blockDim.x) {
    if constexpr (kSwiGLU) {
      const uint4 gv = reinterpret_cast<const uint4*>(x)[i];
      const uint4 uv = reinterpret_cast<const uint4*>(x + K)[i];
      const T* ge = reinterpret_cast<const T*>(&gv);
      const T* ue = reinterpret_cast<const T*>(&uv);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float g = to_f32(ge[t]);
        const float act = to_f32(from_f32<T>(g / (1.0f + expf(-g))));
        oe[t] = from_f32<T>(act * to_f32(ue[t]));
      }
      xs[i] = o;
    } else {
      xs[i] = reinterpret_cast<const uint4*>(x)[i];
    }
  }
}

// RPW rows per warp streamed together (their loads in flight at once; each row keeps the per-lane
// order of a single-row pass, so the result bits do not depend on RPW); rows of warp-group u are
// u * RPW .. u * RPW + RPW - 1, warp-groups strided over the grid.
template <typename T, bool kSwiGLU = false, int RPW = 1>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                               T* __restrict__ out, int64_t N, int K) {
  extern __shared__ uint4 xs[];
  const int kc = K / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t g0 = (int64_t)blockIdx.x * kGemvWarps + warp, gstride = (int64_t)gridDim.x * kGemvWarps;
  // the weights do not depend on the previous kernel: start pulling this warp's first rows into L2
  prefetch_rows_l2(w, g0 * RPW, 1, g0 * RPW + RPW < N ? g0 * RPW + RPW : N, K, RPW);
  pdl_launch();
  pdl_wait();
  stage_x<T, kSwiGLU>(xs, x, K);
  __syncthreads();
  for (int64_t grp = g0; grp * RPW < N; grp += gstride) {
    const uint4* wr[RPW];
    float acc[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int64_t row = grp * RPW + j;
      wr[j] = reinterpret_cast<const uint4*>(w + (row < N ? row : N - 1) * (int64_t)K);
      acc[j] = 0.f;
    }
#pragma unroll 8
    for (int c = lane; c < kc; c += 32) {
      const uint4 b = xs[c];
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const uint4 a = __ldg(wr[j] + c);
        acc[j] = dot2(a.x, b.x, acc[j], (T*)nullptr);
        acc[j] = dot2(a.y, b.y, acc[j], (T*)nullptr);
        acc[j] = dot2(a.z, b.z, acc[j], (T*)nullptr);
        acc[j] = dot2(a.w, b.w, acc[j], (T*)nullptr);
      }
    }
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
      const int64_t row = grp * RPW + j;
      if (lane == 0 && row < N) out[row] = from_f32<T>(acc[j]);
    }
  }
}

template <typename T>
__global__ void qk_norm_rope_kernel(T* __restrict__ q, T* __restrict__ k, const T* __restrict__ wq,
                                    const T* __restrict__ wk, const T* __restrict__ cosv,
                                    const T* __restrict__ sinv, int q_heads, int d, float inv_d, float eps) {
  __shared__ float red[32];
  extern __shared__ float z[];  // the normed head, for rotate_half
  pdl_launch();
  pdl_wait();
  const int head = blockIdx.x;
  const bool is_q = head < q_heads;
  T* row = is_q ? q + (int64_t)head * d : k + (int64_t)(head - q_heads) * d;
  const T* w = is_q ? wq : wk;
  const int i = threadIdx.x;  // blockDim.x = d rounded up to a warp multiple
  const float xi = i < d ? to_f32(row[i]) : 0.f;
  const float ss = block_sum_f32(xi * xi, red);
  const float r = rsqrtf(ss * inv_d + eps);
  float zi = 0.f;
  if (i < d) {
    const T y = from_f32<T>(xi * r);
    zi = to_f32(from_f32<T>(to_f32(w[i]) * to_f32(y)));
    z[i] = zi;
  }
  __syncthreads();
  if (i < d) {
    const int half = d >> 1;
    const float rot = i < half ? -z[i + half] : z[i - half];
    const float t1 = to_f32(from_f32<T>(zi * to_f32(cosv[i])));
    const float t2 = to_f32(from_f32<T>(rot * to_f32(sinv[i])));
    row[i] = from_f32<T>(t1 + t2);
  }
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ out,
                                                                int64_t rows, int inter) {
  pdl_launch();
  pdl_wait();
  const int64_t total = rows * inter;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rr = t / inter;
    const int c = (int)(t - rr * inter);
    const float g = to_f32(gu[rr * 2 * inter + c]);
    const float act = to_f32(from_f32<T>(g / (1.0f + expf(-g))));
    out[t] = from_f32<T>(act * to_f32(gu[rr * 2 * inter + inter + c]));
  }
}

}  // namespace tc
