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
// When the rows are contiguous and 16-byte aligned (every GrowingLayer buffer), splice_bulk_kernel
// runs the same protocol with the unit moved by bulk copies through a shared-memory ring.
#pragma once

#include <type_traits>

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

// ------------------------------------------------------------------------------------------------
// Rotation of one 16-byte chunk pair held as raw words (x from the first half of a row, y from the
// second), element e of the pair at half-index i0 + e; the same separately rounded fp32 products and
// sum as rotate_pair. cs is 16-byte aligned with i0 and half multiples of 4.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  else
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  uint32_t w;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    memcpy(&w, &v, 4);
  } else {
    const __half2 v = __floats2half2_rn(a, b);
    memcpy(&w, &v, 4);
  }
  return w;
}
__device__ __forceinline__ void rot1(float x, float y, float c, float s, float& o0, float& o1) {
  o0 = __fadd_rn(__fmul_rn(x, c), __fmul_rn(-y, s));
  o1 = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, s));
}
template <typename T>
__device__ __forceinline__ void rotate_words(uint4& x, uint4& y, const float* cs, int half, int i0) {
  uint32_t* xw = reinterpret_cast<uint32_t*>(&x);
  uint32_t* yw = reinterpret_cast<uint32_t*>(&y);
  if constexpr (std::is_same<T, float>::value) {
    const float4 c = *reinterpret_cast<const float4*>(cs + i0);
    const float4 sn = *reinterpret_cast<const float4*>(cs + half + i0);
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float o0, o1;
      rot1(__uint_as_float(xw[e]), __uint_as_float(yw[e]), cc[e], ss[e], o0, o1);
      xw[e] = __float_as_uint(o0);
      yw[e] = __float_as_uint(o1);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 2; ++q) {  // 4 elements per float4 of the table
      const float4 c = *reinterpret_cast<const float4*>(cs + i0 + 4 * q);
      const float4 sn = *reinterpret_cast<const float4*>(cs + half + i0 + 4 * q);
      const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const float2 a = unpack2<T>(xw[2 * q + w]), b = unpack2<T>(yw[2 * q + w]);
        float o0a, o1a, o0b, o1b;
        rot1(a.x, b.x, cc[2 * w], ss[2 * w], o0a, o1a);
        rot1(a.y, b.y, cc[2 * w + 1], ss[2 * w + 1], o0b, o1b);
        xw[2 * q + w] = pack2<T>(o0a, o0b);
        yw[2 * q + w] = pack2<T>(o1a, o1b);
      }
    }
  }
}

// In-place splice through shared memory (rows contiguous, 16-byte aligned). Same units, ticket
// order and read flags as splice_inplace_kernel; a unit's K rows and V rows (16 KB each at most)
// arrive by two bulk copies into one stage of a kBulkStages ring, the K rows are rotated in shared
// memory, and two bulk stores write them to the destination. Thread 0 drives the ring with no
// memory round trip on a unit's path: the next ticket is always taken one fetch ahead, a unit's read
// flag is stored as soon as its bulk loads have completed, and the flags a unit must wait for are
// read one iteration ahead and only polled again if they were not yet set.
//   Ordering: a read flag is written after the mbarrier reported the unit's loads complete, and
//   the bulk stores that overwrite those rows are issued only after another thread has seen the
//   flag, so the overwrite cannot reach the rows before they were read; relaxed accesses suffice.
//   Progress: a unit's flag is written only when this CTA reaches it, but the CTA's earlier units
//   hold smaller tickets and wait only on smaller ones, so the smallest unwritten flag always
//   progresses: no deadlock, with or without co-resident CTAs.
// Same rotation with this chunk's cos (c) and sin (sn) already in registers: VEC values each.
template <typename T>
__device__ __forceinline__ void rotate_words_reg(uint4& x, uint4& y, const float* c, const float* sn) {
  uint32_t* xw = reinterpret_cast<uint32_t*>(&x);
  uint32_t* yw = reinterpret_cast<uint32_t*>(&y);
  if constexpr (std::is_same<T, float>::value) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float o0, o1;
      rot1(__uint_as_float(xw[e]), __uint_as_float(yw[e]), c[e], sn[e], o0, o1);
      xw[e] = __float_as_uint(o0);
      yw[e] = __float_as_uint(o1);
    }
  } else {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float2 a = unpack2<T>(xw[w]), b = unpack2<T>(yw[w]);
      float o0a, o1a, o0b, o1b;
      rot1(a.x, b.x, c[2 * w], sn[2 * w], o0a, o1a);
      rot1(a.y, b.y, c[2 * w + 1], sn[2 * w + 1], o0b, o1b);
      xw[w] = pack2<T>(o0a, o0b);
      yw[w] = pack2<T>(o1a, o1b);
    }
  }
}

constexpr int kBulkStages = 3;
constexpr int kBulkCtasPerSm = 2;
constexpr int kBulkUnitBytes = 16384;  // K (or V) bytes of one unit, upper bound
constexpr int kBulkThreads = 256;
constexpr unsigned int kNoUnit = 0xffffffffu;

// Flags unit (lh, chunk i) waits for: chunks [j_lo, j_hi] of the same layer-head (none if j_lo > j_hi).
__device__ __forceinline__ void splice_deps(const SpliceParams& p, int64_t i, int64_t& j_lo, int64_t& j_hi) {
  const int64_t r0 = i * p.rows_per_unit;
  const int64_t r1 = (r0 + p.rows_per_unit < p.c) ? r0 + p.rows_per_unit : p.c;
  const int64_t lo_t = r0 - p.gap, hi_t = r1 - 1 - p.gap;  // C-index range of overwritten sources
  j_lo = 1;
  j_hi = 0;
  if (hi_t < 0) return;
  j_lo = (lo_t > 0 ? lo_t : 0) / p.rows_per_unit;
  j_hi = hi_t / p.rows_per_unit;
  if (j_hi > i - 1) j_hi = i - 1;
}

template <typename T>
__global__ void __launch_bounds__(kBulkThreads) splice_bulk_kernel(const __grid_constant__ SpliceParams p) {
  constexpr int VEC = 16 / (int)sizeof(T);
  extern __shared__ __align__(128) uint8_t smem[];  // kBulkStages x (K rows, V rows)
  __shared__ __align__(8) uint64_t full[kBulkStages];
  __shared__ __align__(16) float s_cs[kMaxRopeDim];
  __shared__ unsigned int s_unit[kBulkStages];
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int half = p.d / 2, cph = half / VEC;
  const int64_t lh_count = (int64_t)p.layers * p.hkv;
  const int64_t units = lh_count * p.nchunks;
  const int64_t row_elems = p.d;  // rows are contiguous: token stride == d
  for (int i = tid; i < p.d; i += blockDim.x) s_cs[i] = p.cs[i];
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kBulkStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- thread 0 state
  // every task of a thread has the same chunk index when the stride divides by the chunks per
  // half-row: then its cos/sin live in registers (no shared-memory table reads in the loop)
  const bool fixed_ch = kBulkThreads % cph == 0;
  const int my_ch = tid % cph;
  float my_c[VEC], my_s[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    my_c[e] = fixed_ch ? s_cs[my_ch * VEC + e] : 0.f;
    my_s[e] = fixed_ch ? s_cs[half + my_ch * VEC + e] : 0.f;
  }

  int fetched = 0;             // iterations whose stage has been filled (or marked as the end)
  unsigned int next_ticket = 0;  // taken one fetch ahead
  uint64_t pol = 0;
  unsigned int dep_seen = 0;   // the next unit's dependency flags were all set when read ahead
  auto fetch = [&](int it) {   // start the loads of iteration `it` (or mark it as the end)
    const int s = it % kBulkStages;
    const unsigned int u = next_ticket;
    next_ticket = atomicAdd(&p.ws->ticket, 1u);  // consumed by the next fetch
    ++fetched;
    if ((int64_t)u >= units) {
      s_unit[s] = kNoUnit;
      mbar_arrive(&full[s]);
      return;
    }
    s_unit[s] = u;
    const int64_t i = u / lh_count, lh = u - i * lh_count;
    const int layer = (int)(lh / p.hkv), h = (int)(lh - (int64_t)layer * p.hkv);
    const int64_t r0 = i * p.rows_per_unit;
    const int64_t r1 = (r0 + p.rows_per_unit < p.c) ? r0 + p.rows_per_unit : p.c;
    const uint32_t bytes = (uint32_t)((r1 - r0) * row_elems * (int64_t)sizeof(T));
    const T* ks = static_cast<const T*>(p.kb[layer]) + h * p.sh + (p.c0 + r0) * row_elems;
    const T* vs = static_cast<const T*>(p.vb[layer]) + h * p.sh + (p.c0 + r0) * row_elems;
    uint8_t* st = smem + (size_t)s * 2 * kBulkUnitBytes;
    mbar_arrive_expect_tx(&full[s], 2 * bytes);
    bulk_g2s(st, ks, bytes, &full[s], pol);
    bulk_g2s(st + kBulkUnitBytes, vs, bytes, &full[s], pol);
  };
  auto read_deps_ahead = [&](int it) {  // read the dependency flags of iteration `it`'s unit
    dep_seen = 0;
    if (it >= fetched) return;
    const unsigned int u = s_unit[it % kBulkStages];
    if (u == kNoUnit) return;
    const int64_t i = u / lh_count, lh = u - i * lh_count;
    int64_t j_lo, j_hi;
    splice_deps(p, i, j_lo, j_hi);
    unsigned int all = 1;
    for (int64_t j = j_lo; j <= j_hi; ++j) all &= ld_relaxed_u32(&p.ws->flags[lh * p.nchunks + j]) == p.epoch;
    dep_seen = all;
  };
  if (tid == 0) {
    pol = policy_evict_first();
    next_ticket = atomicAdd(&p.ws->ticket, 1u);
    for (int it = 0; it < kBulkStages; ++it) fetch(it);
    read_deps_ahead(0);
  }

  int it = 0;
  for (;; ++it) {
    const int s = it % kBulkStages;
    if (tid == 0) {
      const bool ok = mbar_wait(&full[s], (uint32_t)((it / kBulkStages) & 1), TC_DEVERR_PIPE_TIMEOUT);
      s_ok = ok;
      // the unit's source rows are in shared memory: later units may overwrite them
      if (ok && s_unit[s] != kNoUnit) {
        const int64_t u = s_unit[s];
        const int64_t i = u / lh_count, lh = u - i * lh_count;
        st_relaxed_u32(&p.ws->flags[lh * p.nchunks + i], p.epoch);
      }
    }
    __syncthreads();
    if (!s_ok || s_unit[s] == kNoUnit) break;  // uniform
    const int64_t u = s_unit[s];
    const int64_t i = u / lh_count, lh = u - i * lh_count;
    const int layer = (int)(lh / p.hkv), h = (int)(lh - (int64_t)layer * p.hkv);
    const int64_t r0 = i * p.rows_per_unit;
    const int64_t r1 = (r0 + p.rows_per_unit < p.c) ? r0 + p.rows_per_unit : p.c;
    uint8_t* st = smem + (size_t)s * 2 * kBulkUnitBytes;

    // rotate the K rows in place in shared memory (a quarter warp covers 128 contiguous bytes)
    const int ntask = (int)(r1 - r0) * cph;
    if (fixed_ch) {
      for (int t = tid; t < ntask; t += kBulkThreads) {
        T* row = reinterpret_cast<T*>(st) + (int64_t)(t / cph) * row_elems;
        uint4* xp = reinterpret_cast<uint4*>(row + my_ch * VEC);
        uint4* yp = reinterpret_cast<uint4*>(row + half + my_ch * VEC);
        uint4 x = *xp, y = *yp;
        rotate_words_reg<T>(x, y, my_c, my_s);
        *xp = x;
        *yp = y;
      }
    } else {
      for (int t = tid; t < ntask; t += kBulkThreads) {
        const int r = t / cph, ch = t - (t / cph) * cph;
        T* row = reinterpret_cast<T*>(st) + (int64_t)r * row_elems;
        uint4* xp = reinterpret_cast<uint4*>(row + ch * VEC);
        uint4* yp = reinterpret_cast<uint4*>(row + half + ch * VEC);
        uint4 x = *xp, y = *yp;
        rotate_words<T>(x, y, s_cs, half, ch * VEC);
        *xp = x;
        *yp = y;
      }
    }
    fence_proxy_async_smem();  // the rotated rows are read next by the bulk store (async proxy)

    int ok = 1;
    if (tid == 0 && !dep_seen) {
      // some flag this unit waits for was not set when read ahead: poll it now (bounded)
      int64_t j_lo, j_hi;
      splice_deps(p, i, j_lo, j_hi);
      for (int64_t j = j_lo; j <= j_hi && ok; ++j) {
        const unsigned int* f = &p.ws->flags[lh * p.nchunks + j];
        uint32_t spin = 0;
        while (ld_relaxed_u32(f) != p.epoch) {
          if (++spin >= kSpinLimit) {
            raise_error(TC_DEVERR_FLAG_TIMEOUT);
            ok = 0;
            break;
          }
          __nanosleep(64);
        }
      }
    }
    __syncthreads();  // every thread's rotation is written and fenced
    if (tid == 0) {
      if (ok) {
        const uint32_t bytes = (uint32_t)((r1 - r0) * row_elems * (int64_t)sizeof(T));
        T* kd = static_cast<T*>(p.kb[layer]) + h * p.sh + (p.a + r0) * row_elems;
        T* vd = static_cast<T*>(p.vb[layer]) + h * p.sh + (p.a + r0) * row_elems;
        bulk_s2g(kd, st, bytes);
        bulk_s2g(vd, st + kBulkUnitBytes, bytes);
      }
      bulk_commit();
      // refill the previous iteration's stage once its stores have read it
      if (it > 0) {
        bulk_wait_read<1>();
        fetch(it - 1 + kBulkStages);
      }
      read_deps_ahead(it + 1);
    }
  }
  if (tid == 0) {
    // drain: stages filled for iterations this CTA never reached (end markers, or loads still in
    // flight after a timeout), then this thread's stores
    for (int j = s_ok ? it + 1 : it; j < fetched; ++j)
      mbar_wait(&full[j % kBulkStages], (uint32_t)((j / kBulkStages) & 1), TC_DEVERR_PIPE_TIMEOUT);
    bulk_wait<0>();
    // the last CTA to leave resets the ticket for the next call on this workspace
    __threadfence();
    if (atomicAdd(&p.ws->exits, 1u) == gridDim.x - 1) {
      p.ws->ticket = 0;
      p.ws->exits = 0;
      __threadfence();
    }
  }
}

}  // namespace tc
