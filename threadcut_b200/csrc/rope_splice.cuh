// RoPE key shift and KV splice for sm_100a.
//
// Reference semantics (threadcut/kv.py):
//   shift_keys (kv.py:20-25): angle = delta * inv_freq (fp32), emb = cat(angle, angle),
//     out = k*cos(emb) + rotate_half(k)*sin(emb) in fp32, cast to the cache dtype. For a half
//     index i < d/2 with x = k[i], y = k[i + d/2], c = cos(angle_i), s = sin(angle_i):
//       out[i]       = x*c + (-y)*s        out[i + d/2] = y*c + x*s
//     torch evaluates the two products and the sum as separate fp32 roundings; the kernels do the
//     same with __fmul_rn/__fadd_rn, so the result is bit-identical to the fp32 torch expression
//     for the same cos/sin table.
//   GrowingLayer.splice (kv.py:83-92): rows [c0, c0+c) of K (re-rotated by -(c0-a)) and V move
//     to [a, a+c) of the same buffer; splice() (kv.py:28-33) does it for every layer.
//
// The splice is pure bandwidth: 16-byte vector loads/stores, each thread owns matching 16-byte
// chunks of both halves of a row (the rotation pairs i and i + d/2). In-place with overlap
// (c0 - a < c) is done in ONE launch: a persistent grid takes units (chunk i of layer-head lh) from
// an atomic ticket in chunk-major order, reads the unit into registers, publishes a per-unit
// "read" flag, and writes only after the units whose source rows it overwrites have published
// theirs (at most two earlier units; bounded wait). Writers never precede the readers they could
// clobber, and no unit waits on one that has not been handed out, so the grid cannot deadlock.
#pragma once

#include "tc_common.cuh"

namespace tc {

constexpr int kMaxLayers = 128;
constexpr int kMaxRopeDim = 512;
constexpr int kSpliceThreads = 256;
constexpr int kSpliceTasksPerThread = 2;  // (row, chunk-pair) tasks per thread per unit

// 16-byte vector of T (VEC = 16 / sizeof(T)) or a single element (VEC = 1).
template <typename T, int VEC>
struct Chunk {
  T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ Chunk<T, VEC> ld_chunk(const T* p) {
  Chunk<T, VEC> c;
  if constexpr (VEC * sizeof(T) == 16) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    memcpy(&c, &u, 16);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) c.v[i] = p[i];
  }
  return c;
}
template <typename T, int VEC>
__device__ __forceinline__ void st_chunk(T* p, const Chunk<T, VEC>& c) {
  if constexpr (VEC * sizeof(T) == 16) {
    uint4 u;
    memcpy(&u, &c, 16);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = c.v[i];
  }
}

// Rotate the pair of chunks (x from the first half, y from the second half) in place.
// cs: cos at [0, d/2), sin at [d/2, d); i0 = index of the chunk's first element within the half.
template <typename T, int VEC>
__device__ __forceinline__ void rotate_pair(Chunk<T, VEC>& x, Chunk<T, VEC>& y, const float* cs, int half, int i0) {
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    const float xf = to_f32<T>(x.v[e]), yf = to_f32<T>(y.v[e]);
    const float c = cs[i0 + e], s = cs[half + i0 + e];
    const float o0 = __fadd_rn(__fmul_rn(xf, c), __fmul_rn(-yf, s));
    const float o1 = __fadd_rn(__fmul_rn(yf, c), __fmul_rn(xf, s));
    x.v[e] = from_f32<T>(o0);
    y.v[e] = from_f32<T>(o1);
  }
}

struct ShiftParams {
  const void* in;
  void* out;
  int64_t outer, n;
  int64_t in_so, in_sn, out_so, out_sn;
  int d;
  float cs[kMaxRopeDim];
};

// Out-of-place shift of [outer, n, d] keys.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) shift_keys_kernel(const __grid_constant__ ShiftParams p) {
  __shared__ float s_cs[kMaxRopeDim];
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) s_cs[i] = p.cs[i];
  __syncthreads();
  const int half = p.d / 2, cph = half / VEC;
  const int64_t tasks = p.outer * p.n * cph;
  const T* in = static_cast<const T*>(p.in);
  T* out = static_cast<T*>(p.out);
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < tasks; t += (int64_t)gridDim.x * blockDim.x) {
    const int ch = (int)(t % cph);
    const int64_t row = t / cph;
    const int64_t o = row / p.n, r = row - o * p.n;
    const T* src = in + o * p.in_so + r * p.in_sn + ch * VEC;
    T* dst = out + o * p.out_so + r * p.out_sn + ch * VEC;
    Chunk<T, VEC> x = ld_chunk<T, VEC>(src), y = ld_chunk<T, VEC>(src + half);
    rotate_pair<T, VEC>(x, y, s_cs, half, ch * VEC);
    st_chunk<T, VEC>(dst, x);
    st_chunk<T, VEC>(dst + half, y);
  }
}

struct SpliceCopyParams {
  const void* kin;
  const void* vin;
  void* kout;
  void* vout;
  int64_t hkv, a, c0, c;
  int64_t in_sh, in_sn, out_sh, out_sn;
  int d;
  int rotate;
  float cs[kMaxRopeDim];
};

// Copy splice: out rows [0, a) <- in rows [0, a); out rows [a, a+c) <- in rows [c0, c0+c)
// (keys rotated when `rotate`).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) splice_copy_kernel(const __grid_constant__ SpliceCopyParams p) {
  __shared__ float s_cs[kMaxRopeDim];
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) s_cs[i] = p.cs[i];
  __syncthreads();
  const int half = p.d / 2, cph = half / VEC;
  const int64_t rows = p.a + p.c;
  const int64_t tasks = p.hkv * rows * cph;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < tasks; t += (int64_t)gridDim.x * blockDim.x) {
    const int ch = (int)(t % cph);
    const int64_t hr = t / cph;
    const int64_t h = hr / rows, r = hr - h * rows;
    const int64_t sr = r < p.a ? r : p.c0 + (r - p.a);
    const int64_t so = h * p.in_sh + sr * p.in_sn + ch * VEC;
    const int64_t dof = h * p.out_sh + r * p.out_sn + ch * VEC;
    const T* kin = static_cast<const T*>(p.kin) + so;
    const T* vin = static_cast<const T*>(p.vin) + so;
    T* kout = static_cast<T*>(p.kout) + dof;
    T* vout = static_cast<T*>(p.vout) + dof;
    Chunk<T, VEC> kx = ld_chunk<T, VEC>(kin), ky = ld_chunk<T, VEC>(kin + half);
    const Chunk<T, VEC> vx = ld_chunk<T, VEC>(vin), vy = ld_chunk<T, VEC>(vin + half);
    if (p.rotate && r >= p.a) rotate_pair<T, VEC>(kx, ky, s_cs, half, ch * VEC);
    st_chunk<T, VEC>(kout, kx);
    st_chunk<T, VEC>(kout + half, ky);
    st_chunk<T, VEC>(vout, vx);
    st_chunk<T, VEC>(vout + half, vy);
  }
}

// Workspace of the in-place splice: two counters, then one uint32 "read" flag per unit.
struct SpliceWs {
  unsigned int ticket;
  unsigned int exits;
  unsigned int pad[2];
  unsigned int flags[1];  // [layers*hkv][nchunks]
};

struct SpliceParams {
  void* kb[kMaxLayers];
  void* vb[kMaxLayers];
  int layers, hkv, d;
  int rows_per_unit;  // tokens of C per unit
  int64_t a, c0, c, gap, nchunks;
  int64_t sh, sn;
  SpliceWs* ws;
  unsigned int epoch;
  float cs[kMaxRopeDim];
};

template <typename T, int VEC>
__global__ void __launch_bounds__(kSpliceThreads) splice_inplace_kernel(const __grid_constant__ SpliceParams p) {
  __shared__ float s_cs[kMaxRopeDim];
  __shared__ unsigned int s_unit;
  __shared__ int s_ok;
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) s_cs[i] = p.cs[i];
  const int half = p.d / 2, cph = half / VEC;
  const int64_t lh_count = (int64_t)p.layers * p.hkv;
  const int64_t units = lh_count * p.nchunks;
  const int tid = threadIdx.x;

  for (;;) {
    if (tid == 0) s_unit = atomicAdd(&p.ws->ticket, 1u);
    __syncthreads();  // also publishes s_cs on the first pass
    const int64_t u = s_unit;
    if (u >= units) break;
    const int64_t i = u / lh_count, lh = u - i * lh_count;
    const int layer = (int)(lh / p.hkv), h = (int)(lh - (int64_t)layer * p.hkv);
    const int64_t r0 = i * p.rows_per_unit;
    const int64_t r1 = (r0 + p.rows_per_unit < p.c) ? r0 + p.rows_per_unit : p.c;
    T* kb = static_cast<T*>(p.kb[layer]) + h * p.sh;
    T* vb = static_cast<T*>(p.vb[layer]) + h * p.sh;

    // read phase: up to kSpliceTasksPerThread (row, chunk) tasks per thread, rotated in registers
    Chunk<T, VEC> kx[kSpliceTasksPerThread], ky[kSpliceTasksPerThread];
    Chunk<T, VEC> vx[kSpliceTasksPerThread], vy[kSpliceTasksPerThread];
    const int64_t ntask = (r1 - r0) * cph;
#pragma unroll
    for (int k = 0; k < kSpliceTasksPerThread; ++k) {
      const int64_t t = tid + (int64_t)k * kSpliceThreads;
      if (t < ntask) {
        const int64_t r = r0 + t / cph;
        const int ch = (int)(t % cph);
        const int64_t off = (p.c0 + r) * p.sn + ch * VEC;
        kx[k] = ld_chunk<T, VEC>(kb + off);
        ky[k] = ld_chunk<T, VEC>(kb + off + half);
        vx[k] = ld_chunk<T, VEC>(vb + off);
        vy[k] = ld_chunk<T, VEC>(vb + off + half);
        rotate_pair<T, VEC>(kx[k], ky[k], s_cs, half, ch * VEC);
      }
    }
    __threadfence();  // this thread's reads are performed before the unit is published
    __syncthreads();
    if (tid == 0) {
      st_release_u32(&p.ws->flags[lh * p.nchunks + i], p.epoch);
      // wait for the earlier units whose source rows this unit's destination rows overlap
      int ok = 1;
      const int64_t lo_t = r0 - p.gap, hi_t = r1 - 1 - p.gap;  // C-index range of overwritten sources
      if (hi_t >= 0) {
        const int64_t j_lo = (lo_t > 0 ? lo_t : 0) / p.rows_per_unit;
        int64_t j_hi = hi_t / p.rows_per_unit;
        if (j_hi > i - 1) j_hi = i - 1;
        for (int64_t j = j_lo; j <= j_hi && ok; ++j) {
          const unsigned int* f = &p.ws->flags[lh * p.nchunks + j];
          uint32_t spin = 0;
          while (ld_acquire_u32(f) != p.epoch) {
            if (++spin >= kSpinLimit) {
              raise_error(TC_DEVERR_FLAG_TIMEOUT);
              ok = 0;
              break;
            }
            __nanosleep(64);
          }
        }
      }
      s_ok = ok;
    }
    __syncthreads();
    if (s_ok) {
#pragma unroll
      for (int k = 0; k < kSpliceTasksPerThread; ++k) {
        const int64_t t = tid + (int64_t)k * kSpliceThreads;
        if (t < ntask) {
          const int64_t r = r0 + t / cph;
          const int ch = (int)(t % cph);
          const int64_t off = (p.a + r) * p.sn + ch * VEC;
          st_chunk<T, VEC>(kb + off, kx[k]);
          st_chunk<T, VEC>(kb + off + half, ky[k]);
          st_chunk<T, VEC>(vb + off, vx[k]);
          st_chunk<T, VEC>(vb + off + half, vy[k]);
        }
      }
    }
    __syncthreads();  // s_unit / s_ok are rewritten by the next pass
  }
  // the last CTA to leave resets the ticket for the next call on this workspace
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&p.ws->exits, 1u) == gridDim.x - 1) {
      p.ws->ticket = 0;
      p.ws->exits = 0;
      __threadfence();
    }
  }
}

}  // namespace tc
