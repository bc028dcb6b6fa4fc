// Split-KV GQA decode attention for sm_100a.
//
// Reference semantics: threadcut/flash_decode.py:21-69 (_partial + softmax(lse) merge) and the
// folded decode branch of threadcut/attention.py:35-42: for each KV head h the g query heads that
// share it form a g-row query; out = softmax(scale * q k^T) v over the n cached tokens, fp32 math,
// result cast to the input dtype.
//
// B200 design (16-bit K/V, the hot path):
//   * grid (split, kv_head, sequence), one CTA per SM (about 192 KB of K/V in flight per CTA); each
//     CTA owns one contiguous KV slice of one head, so every K/V byte is read exactly once per step
//     and the folded g heads share it.
//   * warp 6 is the producer: for every 32-token tile one elected lane issues tensor-map TMA copies
//     (cp.async.bulk.tensor, one per 64-column box of K and of V: 4 copies per 16 KB stage at
//     d = 128) with the 128-byte swizzle, which makes the ldmatrix reads below bank-conflict free;
//     each stage completes on its mbarrier. The 4-D maps (d, tokens, heads, batch) carry the real
//     strides of the cache views, and rows past the end of the tensor arrive as zeros.
//   * warps 0-5 are consumers; tile j goes to warp j % 6 and stage j % 12. Per tile:
//       S^T[32 tok x 8 heads] = K . q^T     mma.m16n8k16 (K from ldmatrix, q^T fragments in regs)
//       online softmax in the exp2 domain    (max via 3 xor-shuffles over the 8 token lanes)
//       O^T[d x 8 heads] += V^T . P^T        mma.m16n8k16 (V^T from ldmatrix.trans, P^T from the
//                                            score fragments by movmatrix.trans; P is split into a
//                                            hi and lo 16-bit part so the product keeps ~16 more
//                                            bits than a single bf16 P would)
//     Only 4 of the 8 head columns are real for Qwen3 (g = 4); the tensor core has throughput to
//     spare, the point is to take the per-token FMA/shuffle work off the issue slots so the CTA
//     stays a pure HBM stream.
//   * epilogue: the warps' (m, l, o) are combined in shared memory; with one split the CTA writes
//     the output, otherwise it publishes an unnormalised partial to the workspace. Heads with few
//     splits (<= 3 per warp) are merged by the CTA that arrives last on the head's acq_rel count;
//     heads with more splits by up to 16 CTAs chosen by start ticket, each owning a slice of the
//     output columns, after a bounded wait on the head's release count (see finish_cta).
//   * launched with programmatic dependent launch: the prologue (barrier init, tensor-map and L2
//     prefetches, and the TMA loads of rows the caller declared stable) overlaps the previous
//     kernel's tail; q, lengths, the workspace and everything else that kernel may write are read
//     after griddepcontrol.wait.
//   * fused append (k_app/v_app): the consumer whose tile holds row n-1 patches that row into the
//     staged tile from k_app/v_app and stores it to the cache.
// fp32, d < 64, or K/V whose strides break the 16-byte TMA rule use decode_generic_kernel: the same
// partition and epilogue with plain loads and FMA math.
#pragma once

#include <math.h>

#include "tc_common.cuh"

namespace tc {

constexpr int kTile = 32;        // tokens per staged tile (the TMA box height)
constexpr int kCWarps = 6;       // consumer warps per CTA of the tensor-core kernel (+1 producer warp)
constexpr int kGenWarps = 4;     // warps per CTA of the generic kernel
constexpr int kMaxSplits = 128;  // KV slices per (sequence, head)
// Per (sequence, head) control words at the start of the workspace, all zero between calls:
// [0] start ticket, [1] published partials, [2] mergers done waiting, [3] spare.
constexpr int kCtrWords = 4;
constexpr int kMergeLoads = 8;   // partials one merger thread loads per L2 round trip
constexpr int kLastSplitsPerWarp = 3;  // last-arrival merge: partials per warp (one round trip)
constexpr int kMaxMergers = 16;        // start-ticket mergers per (sequence, head), column slices
constexpr int kMmaCtasPerSm = 1; // resident CTAs per SM of the tensor-core kernel
constexpr int kTabTiles = 256;   // paged mode: tile-table entries of a slice staged in shared memory
constexpr int kGenCtasPerSm = 4; // same for the generic kernel
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct DecodeParams {
  CUtensorMap tmk;               // 4-D maps (d, tokens, heads, batch) of K and V for the tensor-core
  CUtensorMap tmv;               // kernel; unused in ragged mode and by the generic kernel
  const CUtensorMap* tm_ragged;  // ragged mode: device array, maps of sequence b at [2b] (K), [2b+1] (V)
  const void* q;
  void* out;
  float* lse;                 // optional natural-log LSE out, [batch][hkv][g] (stride lse_b per b)
  const void* k;
  const void* v;
  const void* const* k_ptrs;  // ragged: per-sequence K/V bases (device arrays) or null
  const void* const* v_ptrs;
  const int64_t* head_strides;  // ragged: per-sequence head stride (elements) or null
  const int32_t* lengths;       // per-sequence valid length (device) or null (= n)
  int64_t n;
  int64_t sq_b, sq_h, sq_g, so_b, so_h, so_g;
  int64_t sk_b, sk_h, sk_n, sv_b, sv_h, sv_n;
  int64_t lse_b;
  int hkv, g, batch;
  int tiles_per_split;  // KV slice = tiles_per_split * kTile tokens
  int max_splits;       // grid.x and the workspace stride between (sequence, head) rows
  float c;              // scale * log2(e)
  float* ws_o;          // [batch*hkv][max_splits][g][d]  unnormalised partial outputs
  float2* ws_ml;        // [batch*hkv][max_splits][g]  (running max (log2 domain), sum)
  unsigned int* counters;  // [batch*hkv][kCtrWords] (zero between calls)
  int out_f32;             // 1: `out` is fp32 (unrounded partial for a cross-GPU merge), else T
  int64_t stable_rows;     // uniform lengths only: rows [0, stable_rows) of K/V are written by no
                           // kernel that can still be running when this one starts (0: none)
  // fused append (single sequence, tensor-core kernel): row n-1 of K/V is k_app/v_app ([hkv][d],
  // head strides sa_k/sa_v); the CTA whose tile holds that row takes it from there and writes it to
  // the cache. Null: no append.
  const void* k_app;
  const void* v_app;
  int64_t sa_k, sa_v;
  // q/k norm + RoPE fused in front of the attention (tensor-core kernel, with the fused append):
  // q and k_app are the raw projections; each CTA normalises and rotates its head's g query rows
  // and its head's k_app row as qk_norm_rope_kernel does (Qwen3 RMSNorm with weights nq_w / nk_w,
  // then x*cos + rotate_half(x)*sin with cos/sin [d]) into shared memory, and the rotated k_app is
  // the row written to the cache. Null nq_w: q and k_app are used as given.
  const void* nq_w;
  const void* nk_w;
  const void* rope_cos;
  const void* rope_sin;
  float norm_eps, norm_inv_d;
  // paged mode (single sequence, tensor-core kernel): K and V live in pages of a pool and the
  // sequence is n_tiles tiles, tile t being rows [tiles[3t+1], tiles[3t+1] + tiles[3t+2]) of page
  // tiles[3t] (at most kTile rows, inside the page); tmk/tmv are (d, page rows, heads, pages) maps,
  // k/v the pool bases and sk_b/sk_h/sk_n (sv_*) the page, head and row strides. A fused append
  // (k_app) is the last row of the last tile. Null: contiguous rows.
  const int32_t* tiles;
  int64_t n_tiles;
  int64_t stable_tiles;  // paged: tiles [0, stable_tiles) and their rows are written by no kernel
                         // that can still be running when this one starts (0: none)
};

// Stores one output element at element offset `off` of p.out, in T or (partial mode) fp32.
template <typename T>
__device__ __forceinline__ void put_out(const DecodeParams& p, int64_t off, float v) {
  if (p.out_f32)
    static_cast<float*>(p.out)[off] = v;
  else
    static_cast<T*>(p.out)[off] = from_f32<T>(v);
}

// Tiles [t0, t1) of split `split` out of `nsplit` over a sequence of `tiles` tiles: as even as
// integer division allows (no split is more than one tile longer than another).
__device__ __forceinline__ void split_range(int64_t tiles, int split, int nsplit, int64_t& t0, int64_t& t1) {
  t0 = tiles * split / nsplit;
  t1 = tiles * (split + 1) / nsplit;
}

template <typename T>
__device__ __forceinline__ void resolve_seq(const DecodeParams& p, int b, int h, const T*& kh, const T*& vh,
                                            int64_t& n) {
  n = p.lengths ? (int64_t)p.lengths[b] : p.n;
  if (p.k_ptrs) {
    const int64_t hs = p.head_strides ? p.head_strides[b] : p.sk_h;
    kh = static_cast<const T*>(p.k_ptrs[b]) + h * hs;
    vh = static_cast<const T*>(p.v_ptrs[b]) + h * hs;
  } else {
    kh = static_cast<const T*>(p.k) + b * p.sk_b + h * p.sk_h;
    vh = static_cast<const T*>(p.v) + b * p.sv_b + h * p.sv_h;
  }
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float lse_nat(float m2, float l) {
  return l > 0.f ? (m2 + __log2f(l)) * kLn2 : -INFINITY;
}

// Per-warp softmax state in shared memory: m[HP], l[HP], then acc[HP][D + 4] (the +4 keeps the
// fragment-ordered stores bank-conflict free).
template <int D, int HP>
struct Region {
  static constexpr int kAccStride = D + 4;
  static constexpr int kFloats = 2 * HP + HP * kAccStride;
  __device__ static float* m(float* r) { return r; }
  __device__ static float* l(float* r) { return r + HP; }
  __device__ static float* acc(float* r, int i) { return r + 2 * HP + i * kAccStride; }
};

// Heads with at most kLastSplitsPerWarp splits per warp of the CTA are merged by the CTA that
// publishes last (one atomic round trip after the last partial); heads with more splits by
// min(g, nsplit) mergers chosen by start ticket.
__host__ __device__ __forceinline__ bool last_arrival_merge(int nsplit, int nthreads) {
  return nsplit <= (nthreads >> 5) * kLastSplitsPerWarp;
}

// Takes this CTA's start ticket for (sequence b, head h) and returns its merger index: ticket -
// (nsplit - nm) for the last nm = merger_count() tickets, -1 before them.
// Number of start-ticket mergers of a head: one per slice of the g*D/4 float4 output columns, at
// most kMaxMergers and at most one per split.
__device__ __forceinline__ int merger_count(int nsplit, int ncols) {
  int nm = nsplit < kMaxMergers ? nsplit : kMaxMergers;
  return nm < ncols ? nm : ncols;
}

__device__ __forceinline__ int merger_index(const DecodeParams& p, int b, int h, int nsplit, int ncols) {
  const unsigned int t = atomicAdd(p.counters + ((int64_t)b * p.hkv + h) * kCtrWords, 1u);
  const int nm = merger_count(nsplit, ncols);
  const int mi = (int)t - (nsplit - nm);
  return mi >= 0 ? mi : -1;
}

// Last-arrival merge of all nsplit partials of (sequence b, head h), every one visible to the calling
// CTA: warp w folds splits w, w + nwarps, ... (at most kLastSplitsPerWarp), lane l the float4 columns
// c0 + l + 32k of each 128-column pass, and the warps' states are combined through `scratch`
// (merge_scratch_bytes(blockDim.x) bytes). Called by all threads of the CTA.
template <typename T, int D>
__device__ void merge_last(const DecodeParams& p, uint8_t* scratch, int b, int h, int nsplit) {
  constexpr int Q = D / 4;   // float4 columns per query head
  constexpr int C = 128;     // columns per pass, 4 per lane
  const int g = p.g;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int nwarps = nthr >> 5, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = (int64_t)b * p.hkv + h;
  const int64_t out0 = b * p.so_b + h * p.so_h;
  const int ncols = g * Q;
  float* sM = reinterpret_cast<float*>(scratch);  // [nwarps][C]
  float* sL = sM + nwarps * C;
  float4* sA = reinterpret_cast<float4*>(sL + nwarps * C);
  const float2* mlb = p.ws_ml + bh * p.max_splits * g;
  const float4* ob = reinterpret_cast<const float4*>(p.ws_o + bh * p.max_splits * g * D);
  for (int c0 = 0; c0 < ncols; c0 += C) {
    float M[4], L[4];
    float4 A[4];
    int hd[4];
    float2 ml[kLastSplitsPerWarp][4];
    float4 x[kLastSplitsPerWarp][4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + lane + 32 * k;
      hd[k] = c < ncols ? c / Q : -1;
    }
#pragma unroll
    for (int j = 0; j < kLastSplitsPerWarp; ++j) {
      const int s = warp + j * nwarps;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const bool use = s < nsplit && hd[k] >= 0;
        ml[j][k] = use ? __ldcg(mlb + (int64_t)s * g + hd[k]) : make_float2(-INFINITY, 0.f);
        x[j][k] = use ? __ldcg(ob + (int64_t)s * ncols + c0 + lane + 32 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float mc = -INFINITY;
#pragma unroll
      for (int j = 0; j < kLastSplitsPerWarp; ++j) mc = fmaxf(mc, ml[j][k].x);
      L[k] = 0.f;
      A[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kLastSplitsPerWarp; ++j) {
        const float w = ml[j][k].x == -INFINITY ? 0.f : fast_exp2(ml[j][k].x - mc);
        L[k] += w * ml[j][k].y;
        A[k].x += w * x[j][k].x;
        A[k].y += w * x[j][k].y;
        A[k].z += w * x[j][k].z;
        A[k].w += w * x[j][k].w;
      }
      M[k] = mc;
      sM[warp * C + lane + 32 * k] = M[k];
      sL[warp * C + lane + 32 * k] = L[k];
      sA[warp * C + lane + 32 * k] = A[k];
    }
    __syncthreads();
    const int cn = ncols - c0 < C ? ncols - c0 : C;
    for (int c = tid; c < cn; c += nthr) {
      const int i = (c0 + c) / Q;
      float Mt = -INFINITY;
      for (int w = 0; w < nwarps; ++w) Mt = fmaxf(Mt, sM[w * C + c]);
      float Lt = 0.f;
      float4 At = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int w = 0; w < nwarps; ++w) {
        const float mw = sM[w * C + c];
        const float wt = mw == -INFINITY ? 0.f : fast_exp2(mw - Mt);
        const float4 v = sA[w * C + c];
        Lt += wt * sL[w * C + c];
        At.x += wt * v.x;
        At.y += wt * v.y;
        At.z += wt * v.z;
        At.w += wt * v.w;
      }
      const float inv = Lt > 0.f ? 1.f / Lt : 0.f;
      const int64_t o = out0 + i * p.so_g + (c0 + c - i * Q) * 4;
      put_out<T>(p, o, At.x * inv);
      put_out<T>(p, o + 1, At.y * inv);
      put_out<T>(p, o + 2, At.z * inv);
      put_out<T>(p, o + 3, At.w * inv);
      if (p.lse != nullptr && c0 + c == i * Q) p.lse[b * p.lse_b + (int64_t)h * g + i] = lse_nat(Mt, Lt);
    }
    __syncthreads();  // the scratch is rewritten by the next pass
  }
}

// Combine the per-warp states of this CTA, then write the output (one split) or publish a partial;
// in a merger CTA of this (sequence, head), then merge the partials.
//
// Few splits (last_arrival_merge): each CTA publishes its partial and bumps the head's counter with
// an acq_rel atomic; the CTA that sees nsplit - 1 published last, so every partial is visible to it,
// and it merges all query heads at once: warp w folds splits w, w + nwarps, w + 2*nwarps (one L2
// round trip), lane l columns l, l+32, l+64, l+96, and the warps are combined in shared memory. It
// clears the counter. No start ticket and no waiting.
//
// Many splits: every CTA publishes its unnormalised partial and bumps the head's published counter
// with a release. The CTAs that took the last nm = merger_count() START tickets are the head's
// mergers (`mi` = ticket - (nsplit - nm), -1 for the others): every other CTA of the head took its
// ticket earlier, so it is already running (or done) and publishes without waiting on anything,
// and the mergers' bounded waits need no co-residency guarantee. Merger mi owns the mi-th of nm
// equal slices of the g*D/4 float4 output columns: thread t folds one column of the splits
// t / w, t / w + nsg, ... (w = slice width, nsg = blockDim.x / w split groups), loading up to
// kMergeLoads of them per L2 round trip, and the split groups are combined through shared memory.
// The last merger past the wait clears the published count; the merger with the last ticket clears
// the ticket.
// Preconditions: every thread calls this after a __syncthreads() that follows the region writes;
// the region area holds at least merge_scratch_bytes(blockDim.x) bytes.
template <typename T, int D, int HP>
__device__ void finish_cta(const DecodeParams& p, uint8_t* regions, int region_stride_bytes, int nregions,
                           int b, int h, int split, int nsplit, int mi) {
  __shared__ float s_M[16], s_L[16];
  __shared__ int s_ok;
  using R = Region<D, HP>;
  const int g = p.g;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int64_t bh = (int64_t)b * p.hkv + h;
  const int64_t out0 = b * p.so_b + h * p.so_h;
  auto region = [&](int w) { return reinterpret_cast<float*>(regions + (size_t)w * region_stride_bytes); };

  if (tid < g) {
    float M = -INFINITY;
    for (int w = 0; w < nregions; ++w) M = fmaxf(M, R::m(region(w))[tid]);
    float L = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < nregions; ++w) L += R::l(region(w))[tid] * fast_exp2(R::m(region(w))[tid] - M);
    s_M[tid] = M;
    s_L[tid] = L;
    if (nsplit > 1) p.ws_ml[(bh * p.max_splits + split) * g + tid] = make_float2(M, L);
  }
  __syncthreads();
  float* wo = p.ws_o + (bh * p.max_splits + split) * g * D;
  for (int idx = tid; idx < g * D; idx += nthr) {
    const int i = idx / D, d = idx - i * D;
    const float M = s_M[i];
    float o = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < nregions; ++w) o += R::acc(region(w), i)[d] * fast_exp2(R::m(region(w))[i] - M);
    if (nsplit == 1) {
      const float L = s_L[i];
      put_out<T>(p, out0 + i * p.so_g + d, L > 0.f ? o / L : 0.f);
    } else {
      wo[idx] = o;
    }
  }
  if (nsplit == 1) {
    if (p.lse != nullptr && tid < g) p.lse[b * p.lse_b + (int64_t)h * g + tid] = lse_nat(s_M[tid], s_L[tid]);
    return;
  }
  unsigned int* ctr = p.counters + bh * kCtrWords;
  __syncthreads();  // every thread's partial writes precede the release below
  if (last_arrival_merge(nsplit, nthr)) {
    if (tid == 0) s_ok = atom_add_acq_rel_u32(ctr + 1, 1u) == (unsigned int)(nsplit - 1);
    __syncthreads();  // also: the regions are free for the merge scratch
    if (!s_ok) return;
    merge_last<T, D>(p, regions, b, h, nsplit);
    if (tid == 0) ctr[1] = 0u;
    return;
  }
  if (tid == 0) red_release_add_u32(ctr + 1, 1u);
  if (mi < 0) return;

  // ---- merger mi: wait (bounded) until all nsplit partials are published
  constexpr int Q = D / 4;  // float4 columns per query head
  const int ncols = g * Q;
  const int nm = merger_count(nsplit, ncols);
  if (tid == 0) {
    int ok = 1;
    uint32_t spin = 0;
    while (ld_acquire_u32(ctr + 1) < (unsigned int)nsplit) {
      if (++spin >= kSpinLimit) {
        raise_error(TC_DEVERR_PIPE_TIMEOUT);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    s_ok = ok;
    // the last merger past the wait clears the published count (the result is needed only at the end)
    if (ok && atomicAdd(ctr + 2, 1u) == (unsigned int)(nm - 1)) {
      ctr[1] = 0u;
      ctr[2] = 0u;
    }
    if (mi == nm - 1) ctr[0] = 0u;  // every CTA of this head has taken its ticket
  }
  __syncthreads();  // also: the regions are free for the merge scratch
  if (!s_ok) return;

  // this merger's float4 columns [c_lo, c_hi) of the g*Q, in chunks of at most nthr columns: thread
  // t folds column t % w of the splits t / w, t / w + nsg, ... (nsg = nthr / w split groups)
  const int c_lo = (int)((int64_t)ncols * mi / nm), c_hi = (int)((int64_t)ncols * (mi + 1) / nm);
  const float2* mlb = p.ws_ml + bh * p.max_splits * g;
  const float4* ob = reinterpret_cast<const float4*>(p.ws_o + bh * p.max_splits * g * D);
  for (int cc = c_lo; cc < c_hi; cc += nthr) {
    const int w = c_hi - cc < nthr ? c_hi - cc : nthr;
    const int nsg = nthr / w;
    const int sg = tid / w, col = cc + (tid - (tid / w) * w);
    const int hd = col / Q;
    float* sM = reinterpret_cast<float*>(regions);  // [nsg][w] per-thread states
    float* sL = sM + nsg * w;
    float4* sA = reinterpret_cast<float4*>(sL + nsg * w);
    float M = -INFINITY, L = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    if (sg < nsg) {
      for (int s0 = sg; s0 < nsplit; s0 += nsg * kMergeLoads) {
        float2 ml[kMergeLoads];
        float4 x[kMergeLoads];
#pragma unroll
        for (int k = 0; k < kMergeLoads; ++k) {
          const int s = s0 + k * nsg;
          const bool use = s < nsplit;
          ml[k] = use ? __ldcg(mlb + (int64_t)s * g + hd) : make_float2(-INFINITY, 0.f);
          x[k] = use ? __ldcg(ob + (int64_t)s * ncols + col) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float mc = M;
#pragma unroll
        for (int k = 0; k < kMergeLoads; ++k) mc = fmaxf(mc, ml[k].x);
        const float a = M == -INFINITY ? 0.f : fast_exp2(M - mc);
        L *= a;
        A.x *= a;
        A.y *= a;
        A.z *= a;
        A.w *= a;
#pragma unroll
        for (int k = 0; k < kMergeLoads; ++k) {
          const float wk = ml[k].x == -INFINITY ? 0.f : fast_exp2(ml[k].x - mc);
          L += wk * ml[k].y;
          A.x += wk * x[k].x;
          A.y += wk * x[k].y;
          A.z += wk * x[k].z;
          A.w += wk * x[k].w;
        }
        M = mc;
      }
      sM[sg * w + (col - cc)] = M;
      sL[sg * w + (col - cc)] = L;
      sA[sg * w + (col - cc)] = A;
    }
    __syncthreads();
    if (tid < w) {
      const int c = cc + tid, i = c / Q;
      float Mt = -INFINITY;
      for (int j = 0; j < nsg; ++j) Mt = fmaxf(Mt, sM[j * w + tid]);
      float Lt = 0.f;
      float4 At = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < nsg; ++j) {
        const float mw = sM[j * w + tid];
        const float wt = mw == -INFINITY ? 0.f : fast_exp2(mw - Mt);
        const float4 v = sA[j * w + tid];
        Lt += wt * sL[j * w + tid];
        At.x += wt * v.x;
        At.y += wt * v.y;
        At.z += wt * v.z;
        At.w += wt * v.w;
      }
      const float inv = Lt > 0.f ? 1.f / Lt : 0.f;
      const int64_t o = out0 + i * p.so_g + (c - i * Q) * 4;
      put_out<T>(p, o, At.x * inv);
      put_out<T>(p, o + 1, At.y * inv);
      put_out<T>(p, o + 2, At.z * inv);
      put_out<T>(p, o + 3, At.w * inv);
      if (p.lse != nullptr && c == i * Q) p.lse[b * p.lse_b + (int64_t)h * g + i] = lse_nat(Mt, Lt);
    }
    __syncthreads();  // the scratch is rewritten by the next chunk
  }
}

// Shared-memory scratch of a merger: (m, l, float4 o) states, 128 per warp (last-arrival merge)
// or one per thread (start-ticket mergers).
__host__ __device__ constexpr int merge_scratch_bytes(int nthreads) { return (nthreads >> 5) * 128 * 24; }


template <typename T>
__device__ __forceinline__ uint32_t pack_raw(T lo, T hi) {
  uint16_t a, b;
  memcpy(&a, &lo, 2);
  memcpy(&b, &hi, 2);
  return (uint32_t)a | ((uint32_t)b << 16);
}

// One d-vector through Qwen3's q_norm/k_norm and the rotate-half RoPE, by one warp, into dst: the
// arithmetic of qk_norm_rope_kernel, including its sum order (lane l holds elements l + 32 t; the
// squares of each group of 32 are summed by a xor butterfly, then the group sums, placed in lanes
// 0..D/32-1, by another), so the result has the same bits.
template <typename T, int D>
__device__ __forceinline__ void norm_rope_row(const T* __restrict__ src, const T* __restrict__ w,
                                              const T* __restrict__ cosv, const T* __restrict__ sinv,
                                              float inv_d, float eps, T* dst, int lane) {
  constexpr int E = D / 32;
  float x[E], z[E];
#pragma unroll
  for (int t = 0; t < E; ++t) x[t] = to_f32(src[lane + 32 * t]);
  float tot = 0.f;
#pragma unroll
  for (int t = 0; t < E; ++t) {
    float s = x[t] * x[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == t) tot = s;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  const float r = rsqrtf(tot * inv_d + eps);
#pragma unroll
  for (int t = 0; t < E; ++t) {
    const T y = from_f32<T>(x[t] * r);
    z[t] = to_f32(from_f32<T>(to_f32(w[lane + 32 * t]) * to_f32(y)));
  }
#pragma unroll
  for (int t = 0; t < E; ++t) {
    const int i = lane + 32 * t;
    const float rot = t < E / 2 ? -z[t + E / 2] : z[t - E / 2];
    const float t1 = to_f32(from_f32<T>(z[t] * to_f32(cosv[i])));
    const float t2 = to_f32(from_f32<T>(rot * to_f32(sinv[i])));
    dst[i] = from_f32<T>(t1 + t2);
  }
}

template <int D>
struct MmaGeom {
  static_assert(D % 64 == 0, "the tensor-core kernel stages 64-column (128-byte) swizzled boxes");
  static constexpr int kBoxBytes = kTile * 128;      // one TMA box: 32 rows x 64 columns of 16-bit data
  static constexpr int kTileBytes = kTile * D * 2;   // D/64 boxes side by side
  static constexpr int kStageBytes = 2 * kTileBytes; // K tile then V tile
  // ~192 KB of K/V in flight per CTA (one CTA per SM): 12 stages at d <= 128, 6 at d = 256.
  // A multiple of kCWarps, so tile j always goes to consumer warp j % kCWarps and stage j % kStages.
  static constexpr int kStages = D <= 128 ? 12 : 6;
  static_assert(kStages % kCWarps == 0, "stages must divide evenly among the consumer warps");
  static constexpr int kPipeBytes = kStages * kStageBytes;
  static constexpr int kSmem = 1024 + kPipeBytes + 2 * kStages * 8;  // + 1 KB base alignment slack
};

// Byte offset of element (row, col) of a staged tile: 64-column boxes of 32 rows x 128 bytes, each
// written by TMA with the 128-byte swizzle (16-byte chunk c of row r lands at chunk c ^ (r & 7)), so
// the 8 rows an ldmatrix phase reads fall in 8 different bank groups.
__device__ __forceinline__ uint32_t swz(int row, int col) {
  const int box = col >> 6, chunk = (col & 63) >> 3;
  return (uint32_t)(box * (kTile * 128) + row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------------------------------------------
// Tensor-core path: T in {bf16, f16}, D in {64, 128, 256}, NG = number of 8-head column tiles
// (g <= 8*NG). K/V tiles arrive by tensor-map TMA: one cp.async.bulk.tensor per 64-column box.
// kPaged: K/V rows come through the tile table (p.tiles); a separate instantiation, so the
// contiguous kernel carries none of it.
template <typename T, int D, int NG, bool kPaged>
__global__ void __launch_bounds__(32 * (kCWarps + 1), 1)
    decode_mma_kernel(const __grid_constant__ DecodeParams p) {
  using G = MmaGeom<D>;
  constexpr int HP = 8 * NG;
  constexpr int KS = D / 16;
  constexpr int NBOX = D / 64;
  constexpr int kStages = G::kStages;
  static_assert(Region<D, HP>::kFloats * 4 <= G::kStageBytes, "combine region must fit in a stage");
  static_assert(merge_scratch_bytes(32 * (kCWarps + 1)) <= G::kPipeBytes, "merge scratch must fit in the pipeline");
  extern __shared__ uint8_t smem_raw[];
  // TMA 128-byte swizzle is defined on absolute shared addresses: align the pipeline to 1 KB
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kPipeBytes);
  uint64_t* empty = full + kStages;
  __shared__ int s_mi;  // merger index of this CTA (-1: not a merger)
  __shared__ int4 s_tab[kPaged ? kTabTiles : 1];  // paged: this CTA's first kTabTiles table entries
  // fused q/k norm + RoPE (p.nq_w): the head's g rotated query rows, then its rotated k_app row
  __shared__ uint4 s_qk[(HP + 1) * D / 8];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised before the producer may arm them below
  int staged = 0;   // producer lane: leading tiles already issued before pdl_wait()
  if (!kPaged && warp == kCWarps && lane == 0) {
    // Before waiting for the previous kernel (it may still be running):
    //  * tiles whose rows the caller declared stable (p.stable_rows, uniform lengths, where n and
    //    the partition come from kernel parameters) are loaded into the pipeline right away;
    //  * the rest of the first pipeline-depth is only prefetched into L2: a length read here may
    //    be stale and the rows may still be being written, both harmless for a prefetch.
    // q, the workspace and everything else used for the result are read after pdl_wait().
    const CUtensorMap* mk = p.tm_ragged ? p.tm_ragged + 2 * b : &p.tmk;
    const CUtensorMap* mv = p.tm_ragged ? p.tm_ragged + 2 * b + 1 : &p.tmv;
    const int cb = p.tm_ragged ? 0 : b;
    prefetch_tensormap(mk);
    prefetch_tensormap(mv);
    const int64_t n_hint = p.lengths ? (int64_t)p.lengths[b] : p.n;
    const int64_t tiles_hint = (n_hint + kTile - 1) / kTile;
    const int ns_hint = n_hint > 0 ? (int)((tiles_hint + p.tiles_per_split - 1) / p.tiles_per_split) : 1;
    if (n_hint > 0 && split < ns_hint) {
      int64_t a0, a1;
      split_range(tiles_hint, split, ns_hint, a0, a1);
      const int64_t pre = a1 - a0 < kStages ? a1 - a0 : kStages;
      if (p.lengths == nullptr && p.stable_rows > 0) {
        const uint64_t pol = policy_evict_first();
        while (staged < pre && (a0 + staged + 1) * kTile <= p.stable_rows) {
          const int s = staged;  // round 0 of stage s: no empty wait
          mbar_arrive_expect_tx(&full[s], (uint32_t)G::kStageBytes);
          uint8_t* st = smem + s * G::kStageBytes;
          const int tok = (int)((a0 + staged) * kTile);
#pragma unroll
          for (int bx = 0; bx < NBOX; ++bx) {
            tma_load_4d(st + bx * G::kBoxBytes, mk, bx * 64, tok, h, cb, &full[s], pol);
            tma_load_4d(st + G::kTileBytes + bx * G::kBoxBytes, mv, bx * 64, tok, h, cb, &full[s], pol);
          }
          ++staged;
        }
      }
      for (int64_t j = staged; j < pre; ++j)
#pragma unroll
        for (int bx = 0; bx < NBOX; ++bx) {
          tma_prefetch_4d(mk, bx * 64, (int)((a0 + j) * kTile), h, cb);
          tma_prefetch_4d(mv, bx * 64, (int)((a0 + j) * kTile), h, cb);
        }
    }
  }
  int tab_pre = 0;  // paged: leading slice entries already in s_tab before pdl_wait()
  if constexpr (kPaged) {
    // paged: the split comes from kernel parameters, so the slice's leading entries that the caller
    // declared stable (p.stable_tiles) are loaded into s_tab by the whole CTA before waiting for the
    // previous kernel. (Starting their K/V copies here too, as the contiguous path does for its
    // stable rows, measured slower for paged decode, so the copies wait for the producer loop.)
    const int64_t nt = p.n_tiles;
    const int ns = nt > 0 ? (int)((nt + p.tiles_per_split - 1) / p.tiles_per_split) : 1;
    if (nt > 0 && split < ns && p.stable_tiles > 0) {
      int64_t a0, a1;
      split_range(nt, split, ns, a0, a1);
      const int64_t lim = (a1 < p.stable_tiles ? a1 : p.stable_tiles) - a0;
      tab_pre = lim <= 0 ? 0 : (lim < kTabTiles ? (int)lim : kTabTiles);
      for (int i = threadIdx.x; i < tab_pre; i += blockDim.x) {
        const int32_t* tt = p.tiles + 3 * (a0 + i);
        s_tab[i] = make_int4(tt[0], tt[1], tt[2], 0);
      }
    }
  }
  pdl_launch();
  pdl_wait();  // everything below may read what the previous kernel in the stream wrote
  const int64_t n = p.lengths ? (int64_t)p.lengths[b] : p.n;
  const int64_t seq_tiles = kPaged ? p.n_tiles : (n + kTile - 1) / kTile;
  const int nsplit = (kPaged ? seq_tiles > 0 : n > 0) ? (int)((seq_tiles + p.tiles_per_split - 1) / p.tiles_per_split) : 1;
  if (split >= nsplit) return;  // whole CTA leaves together; the barriers are never used
  int64_t tt0, tt1;
  split_range(seq_tiles, split, nsplit, tt0, tt1);
  const int64_t t0 = tt0 * kTile;
  const int64_t t1 = n < tt1 * kTile ? n : tt1 * kTile;
  const int ntiles = (int)(tt1 - tt0);
  if (threadIdx.x == 0) s_mi = -1;
  const bool rope = p.nq_w != nullptr;
  if (rope) {
    // warps 0..g-1: the query rows of head h; warp g: the head's k_app row (the producer warp
    // included, before it starts issuing: its leading tiles are already in flight)
    T* sq = reinterpret_cast<T*>(s_qk);
    const T* cs = static_cast<const T*>(p.rope_cos);
    const T* sn = static_cast<const T*>(p.rope_sin);
    for (int r = warp; r <= p.g; r += kCWarps + 1) {
      const bool isq = r < p.g;
      const T* src = isq ? static_cast<const T*>(p.q) + b * p.sq_b + h * p.sq_h + r * p.sq_g
                         : static_cast<const T*>(p.k_app) + h * p.sa_k;
      norm_rope_row<T, D>(src, static_cast<const T*>(isq ? p.nq_w : p.nk_w), cs, sn, p.norm_inv_d, p.norm_eps,
                          sq + (isq ? r : HP) * D, lane);
    }
  }
  if constexpr (kPaged) {
    // the slice's table entries, loaded once by the whole CTA instead of a dependent global load
    // in front of every TMA issue and every consumer tile
    const int nt = ntiles < kTabTiles ? ntiles : kTabTiles;
    for (int i = tab_pre + threadIdx.x; i < nt; i += blockDim.x) {
      const int32_t* tt = p.tiles + 3 * (tt0 + i);
      s_tab[i] = make_int4(tt[0], tt[1], tt[2], 0);
    }
  }
  __syncthreads();
  // (page, first row, rows) of tile j of this slice in paged mode
  auto tab_entry = [&](int j) -> int4 {
    if (j < kTabTiles) return s_tab[j];
    const int32_t* tt = p.tiles + 3 * (tt0 + j);
    return make_int4(tt[0], tt[1], tt[2], 0);
  };

  if (warp == kCWarps) {
    // the start ticket (which CTA merges) is taken by an idle producer lane, off the pipeline's path;
    // the result is read only after the final __syncthreads
    if (lane == 1 && nsplit > 1 && !last_arrival_merge(nsplit, blockDim.x))
      s_mi = merger_index(p, b, h, nsplit, p.g * (D / 4));
    // ---------------- producer: one elected lane issues 2*D/64 tensor copies per tile
    if (lane == 0 && ntiles > 0) {
      const CUtensorMap* mk = p.tm_ragged ? p.tm_ragged + 2 * b : &p.tmk;
      const CUtensorMap* mv = p.tm_ragged ? p.tm_ragged + 2 * b + 1 : &p.tmv;
      const int cb = p.tm_ragged ? 0 : b;
      const uint64_t pol = policy_evict_first();
      for (int j = staged; j < ntiles; ++j) {
        const int s = j % kStages;
        const int r = j / kStages;
        if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, TC_DEVERR_PIPE_TIMEOUT)) break;
        mbar_arrive_expect_tx(&full[s], (uint32_t)G::kStageBytes);
        uint8_t* st = smem + s * G::kStageBytes;
        // rows past the tensor end (or, paged, past the page end) arrive as zeros
        int tok = (int)(t0 + (int64_t)j * kTile), cbj = cb;
        if constexpr (kPaged) {
          const int4 te = tab_entry(j);
          cbj = te.x;
          tok = te.y;
        }
#pragma unroll
        for (int bx = 0; bx < NBOX; ++bx) {
          tma_load_4d(st + bx * G::kBoxBytes, mk, bx * 64, tok, h, cbj, &full[s], pol);
          tma_load_4d(st + G::kTileBytes + bx * G::kBoxBytes, mv, bx * 64, tok, h, cbj, &full[s], pol);
        }
      }
    }
  } else {
    // ---------------- consumers
    const int gid = lane >> 2, qd = lane & 3;
    const float c = p.c;
    uint32_t bq[NG][KS][2];
    {
      const T* qb = rope ? reinterpret_cast<const T*>(s_qk) : static_cast<const T*>(p.q) + b * p.sq_b + h * p.sq_h;
      const int64_t qg = rope ? (int64_t)D : p.sq_g;
      const T zero = from_f32<T>(0.f);
#pragma unroll
      for (int nt = 0; nt < NG; ++nt) {
        const int i = nt * 8 + gid;
        const bool ok = i < p.g;
        const T* qr = qb + (ok ? i : 0) * qg;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int d0 = ks * 16 + 2 * qd;
          bq[nt][ks][0] = pack_raw<T>(ok ? qr[d0] : zero, ok ? qr[d0 + 1] : zero);
          bq[nt][ks][1] = pack_raw<T>(ok ? qr[d0 + 8] : zero, ok ? qr[d0 + 9] : zero);
        }
      }
    }
    float m_run[NG][2], l_run[NG][2];
    float oacc[KS][NG][4];
#pragma unroll
    for (int nt = 0; nt < NG; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        m_run[nt][e] = -INFINITY;
        l_run[nt][e] = 0.f;
      }
#pragma unroll
    for (int md = 0; md < KS; ++md)
#pragma unroll
      for (int nt = 0; nt < NG; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) oacc[md][nt][r] = 0.f;

    for (int j = warp; j < ntiles; j += kCWarps) {
      const int s = j % kStages;
      if (!mbar_wait(&full[s], (j / kStages) & 1, TC_DEVERR_PIPE_TIMEOUT)) break;
      uint8_t* stage = smem + s * G::kStageBytes;
      const uint32_t kst = smem_u32(stage);
      const uint32_t vst = kst + G::kTileBytes;
      int valid;
      if constexpr (kPaged) {
        const int vt = tab_entry(j).z;  // device table: clamp into [0, kTile]
        valid = vt < 0 ? 0 : (vt > kTile ? kTile : vt);
      } else {
        const int64_t rem = t1 - (t0 + (int64_t)j * kTile);
        valid = rem < kTile ? (int)rem : kTile;
      }
      int64_t app_r = -1, app_row = n - 1, app_pg = 0;  // row in the tile, row and page in the cache
      if (p.k_app != nullptr) {
        if constexpr (kPaged) {
          if (tt0 + j == p.n_tiles - 1 && valid > 0) {
            app_r = valid - 1;
            const int4 te = tab_entry(j);
            app_pg = te.x;
            app_row = te.y + app_r;
          }
        } else {
          app_r = (n - 1) - (t0 + (int64_t)j * kTile);
        }
      }
      const bool patch = app_r >= 0 && app_r < kTile;
      if (patch) {
        // the appended row: the cache still holds stale data there, so replace the staged copy with
        // k_app/v_app (16-byte chunks into the swizzled row) and write the row to the cache
        const int r = (int)app_r;
        constexpr int CH = D / 8;  // 16-byte chunks per row
        const uint4* ka = rope ? s_qk + HP * D / 8
                               : reinterpret_cast<const uint4*>(static_cast<const T*>(p.k_app) + h * p.sa_k);
        const uint4* va = reinterpret_cast<const uint4*>(static_cast<const T*>(p.v_app) + h * p.sa_v);
        uint4* kc = reinterpret_cast<uint4*>(const_cast<T*>(static_cast<const T*>(p.k)) + app_pg * p.sk_b + h * p.sk_h +
                                             app_row * p.sk_n);
        uint4* vc = reinterpret_cast<uint4*>(const_cast<T*>(static_cast<const T*>(p.v)) + app_pg * p.sv_b + h * p.sv_h +
                                             app_row * p.sv_n);
        for (int idx = lane; idx < 2 * CH; idx += 32) {
          const bool isv = idx >= CH;
          const int c = isv ? idx - CH : idx;
          const uint4 x = isv ? va[c] : ka[c];
          *reinterpret_cast<uint4*>(stage + (isv ? G::kTileBytes : 0) + (c >> 3) * G::kBoxBytes + r * 128 +
                                    (((c & 7) ^ (r & 7)) << 4)) = x;
          (isv ? vc : kc)[c] = x;
        }
        __syncwarp();
      }
      if (valid < kTile) {
        // rows past this slice may hold another sequence's or uninitialised data (ragged caches
        // are mapped to their capacity): zero those V rows so a masked p = 0 never meets a NaN
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        for (int idx = lane; idx < (kTile - valid) * (D / 8); idx += 32) {
          const int row = valid + idx / (D / 8), cc = idx % (D / 8);
          *reinterpret_cast<uint4*>(stage + G::kTileBytes + (cc >> 3) * G::kBoxBytes + row * 128 + (cc & 7) * 16) = z;
        }
        __syncwarp();
      }

      // S^T = K q^T over two 16-token m-tiles
      float sacc[2][NG][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NG; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) sacc[mt][nt][r] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t a[4];
          const int row = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int col = ks * 16 + (lane >> 4) * 8;
          ldsm_x4(kst + swz(row, col), a);
#pragma unroll
          for (int nt = 0; nt < NG; ++nt) Mma<T>::run(sacc[mt][nt], a, bq[nt][ks][0], bq[nt][ks][1]);
        }
      }

      // online softmax; this lane holds tokens {gid, gid+8, gid+16, gid+24} x heads {2qd, 2qd+1}
      float alpha[NG][2];
#pragma unroll
      for (int nt = 0; nt < NG; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float x0 = sacc[0][nt][e] * c, x1 = sacc[0][nt][2 + e] * c;
          float x2 = sacc[1][nt][e] * c, x3 = sacc[1][nt][2 + e] * c;
          if (gid >= valid) x0 = -INFINITY;
          if (gid + 8 >= valid) x1 = -INFINITY;
          if (gid + 16 >= valid) x2 = -INFINITY;
          if (gid + 24 >= valid) x3 = -INFINITY;
          float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float mnew = fmaxf(m_run[nt][e], mx);
          alpha[nt][e] = fast_exp2(m_run[nt][e] - mnew);
          m_run[nt][e] = mnew;
          const float p0 = fast_exp2(x0 - mnew), p1 = fast_exp2(x1 - mnew);
          const float p2 = fast_exp2(x2 - mnew), p3 = fast_exp2(x3 - mnew);
          l_run[nt][e] = l_run[nt][e] * alpha[nt][e] + ((p0 + p1) + (p2 + p3));
          sacc[0][nt][e] = p0;
          sacc[0][nt][2 + e] = p1;
          sacc[1][nt][e] = p2;
          sacc[1][nt][2 + e] = p3;
        }
      }
#pragma unroll
      for (int md = 0; md < KS; ++md)
#pragma unroll
        for (int nt = 0; nt < NG; ++nt) {
          oacc[md][nt][0] *= alpha[nt][0];
          oacc[md][nt][1] *= alpha[nt][1];
          oacc[md][nt][2] *= alpha[nt][0];
          oacc[md][nt][3] *= alpha[nt][1];
        }

      // P^T fragments: pack (hi, lo) 16-bit parts, transpose 8x8 blocks with movmatrix
      uint32_t bhi[2][NG][2], blo[2][NG][2];
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
#pragma unroll
        for (int nt = 0; nt < NG; ++nt) {
          const float* sp = sacc[kk][nt];
          const uint32_t x0 = Mma<T>::pack(sp[0], sp[1]);
          const uint32_t x1 = Mma<T>::pack(sp[2], sp[3]);
          const uint32_t y0 = Mma<T>::pack(sp[0] - Mma<T>::lo(x0), sp[1] - Mma<T>::hi(x0));
          const uint32_t y1 = Mma<T>::pack(sp[2] - Mma<T>::lo(x1), sp[3] - Mma<T>::hi(x1));
          bhi[kk][nt][0] = movm_t(x0);
          bhi[kk][nt][1] = movm_t(x1);
          blo[kk][nt][0] = movm_t(y0);
          blo[kk][nt][1] = movm_t(y1);
        }

      // O^T += V^T P^T
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
        for (int md = 0; md < KS; ++md) {
          uint32_t a[4];
          const int mi = lane >> 3;
          const int tok = kk * 16 + (mi >> 1) * 8 + (lane & 7);
          const int dim = md * 16 + (mi & 1) * 8;
          ldsm_x4_t(vst + swz(tok, dim), a);
#pragma unroll
          for (int nt = 0; nt < NG; ++nt) {
            Mma<T>::run(oacc[md][nt], a, bhi[kk][nt][0], bhi[kk][nt][1]);
            Mma<T>::run(oacc[md][nt], a, blo[kk][nt][0], blo[kk][nt][1]);
          }
        }
      }
      if (valid < kTile || patch) fence_proxy_async_smem();  // generic writes above precede the next TMA write
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // this warp's state -> its own (now idle) stage buffer
#pragma unroll
    for (int nt = 0; nt < NG; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float l = l_run[nt][e];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_run[nt][e] = l;
      }
    using R = Region<D, HP>;
    float* reg = reinterpret_cast<float*>(smem + warp * G::kStageBytes);
    if (gid == 0) {
#pragma unroll
      for (int nt = 0; nt < NG; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int i = nt * 8 + 2 * qd + e;
          R::m(reg)[i] = m_run[nt][e];
          R::l(reg)[i] = l_run[nt][e];
        }
    }
#pragma unroll
    for (int md = 0; md < KS; ++md)
#pragma unroll
      for (int nt = 0; nt < NG; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int dim = md * 16 + gid + (r >> 1) * 8;
          const int i = nt * 8 + 2 * qd + (r & 1);
          R::acc(reg, i)[dim] = oacc[md][nt][r];
        }
  }
  __syncthreads();
  finish_cta<T, D, HP>(p, smem, G::kStageBytes, kCWarps, b, h, split, nsplit, s_mi);
}

// ------------------------------------------------------------------------------------------------
// Generic path (fp32, or 16-bit K/V that break the bulk-copy alignment rule): 4 warps, warp w takes
// tokens t0+w, t0+w+4, ...; lane owns dims lane, lane+32, ...; scores by warp reduction.
template <int D>
struct GenGeom {
  static constexpr int HP = 16;
  static constexpr int kRegionBytes = ((Region<D, HP>::kFloats * 4 + 127) / 128) * 128;
  static constexpr int kSmem = kGenWarps * kRegionBytes > merge_scratch_bytes(32 * kGenWarps)
                                   ? kGenWarps * kRegionBytes
                                   : merge_scratch_bytes(32 * kGenWarps);
};

template <typename T, int D>
__global__ void __launch_bounds__(32 * kGenWarps) decode_generic_kernel(const __grid_constant__ DecodeParams p) {
  using G = GenGeom<D>;
  constexpr int HP = G::HP;
  constexpr int DPL = D >= 32 ? D / 32 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_launch();
  pdl_wait();
  __shared__ int s_mi;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const T* kh;
  const T* vh;
  int64_t n;
  resolve_seq<T>(p, b, h, kh, vh, n);
  const int64_t seq_tiles = (n + kTile - 1) / kTile;
  const int nsplit = n > 0 ? (int)((seq_tiles + p.tiles_per_split - 1) / p.tiles_per_split) : 1;
  if (split >= nsplit) return;
  int64_t tt0, tt1;
  split_range(seq_tiles, split, nsplit, tt0, tt1);
  const int64_t t0 = tt0 * kTile;
  const int64_t t1 = n < tt1 * kTile ? n : tt1 * kTile;
  if (threadIdx.x == 0)
    s_mi = nsplit > 1 && !last_arrival_merge(nsplit, blockDim.x) ? merger_index(p, b, h, nsplit, p.g * (D / 4)) : -1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = p.g;

  float qv[HP][DPL], acc[HP][DPL], m[HP], l[HP];
  const T* qb = static_cast<const T*>(p.q) + b * p.sq_b + h * p.sq_h;
#pragma unroll
  for (int i = 0; i < HP; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int d = lane + 32 * j;
      qv[i][j] = (i < g && d < D) ? to_f32<T>(qb[i * p.sq_g + d]) : 0.f;
      acc[i][j] = 0.f;
    }
  }
  for (int64_t t = t0 + warp; t < t1; t += kGenWarps) {
    float kv[DPL], vv[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int d = lane + 32 * j;
      kv[j] = d < D ? to_f32<T>(kh[t * p.sk_n + d]) : 0.f;
      vv[j] = d < D ? to_f32<T>(vh[t * p.sv_n + d]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < HP; ++i) {
      if (i < g) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) s = fmaf(qv[i][j], kv[j], s);
        s = warp_sum(s) * p.c;
        const float mn = fmaxf(m[i], s);
        const float al = fast_exp2(m[i] - mn);
        const float pp = fast_exp2(s - mn);
        l[i] = l[i] * al + pp;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[i][j] = fmaf(pp, vv[j], acc[i][j] * al);
        m[i] = mn;
      }
    }
  }
  using R = Region<D, HP>;
  float* reg = reinterpret_cast<float*>(smem + warp * G::kRegionBytes);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < HP; ++i) {
      R::m(reg)[i] = m[i];
      R::l(reg)[i] = l[i];
    }
  }
#pragma unroll
  for (int i = 0; i < HP; ++i)
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int d = lane + 32 * j;
      if (d < D) R::acc(reg, i)[d] = acc[i][j];
    }
  __syncthreads();
  finish_cta<T, D, HP>(p, smem, G::kRegionBytes, kGenWarps, b, h, split, nsplit, s_mi);
}

// ------------------------------------------------------------------------------------------------
// LSE merge of normalised partials (cross-GPU combine and the merge of flash_decode.py:68-69).
template <typename T>
__global__ void merge_partials_kernel(const float* __restrict__ o_parts, const float* __restrict__ lse_parts,
                                      T* __restrict__ out, float* __restrict__ lse_out, int parts, int64_t rows,
                                      int d, int64_t out_stride_row) {
  const int64_t row = blockIdx.x;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int pi = 0; pi < parts; ++pi) M = fmaxf(M, lse_parts[(int64_t)pi * rows + row]);
  float L = 0.f;
  if (M != -INFINITY)
    for (int pi = 0; pi < parts; ++pi) L += __expf(lse_parts[(int64_t)pi * rows + row] - M);
  for (int dd = threadIdx.x; dd < d; dd += blockDim.x) {
    float o = 0.f;
    if (M != -INFINITY)
      for (int pi = 0; pi < parts; ++pi) {
        const float w = __expf(lse_parts[(int64_t)pi * rows + row] - M);
        o += w * o_parts[((int64_t)pi * rows + row) * d + dd];
      }
    out[row * out_stride_row + dd] = from_f32<T>(L > 0.f ? o / L : 0.f);
  }
  if (lse_out != nullptr && threadIdx.x == 0) lse_out[row] = L > 0.f ? M + __logf(L) : -INFINITY;
}

}  // namespace tc
