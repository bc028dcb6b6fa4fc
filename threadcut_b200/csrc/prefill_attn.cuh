// GQA prefill attention on the 5th-generation tensor cores (tcgen05), for sm_100a.
//
// Reference semantics: the prefill branch of threadcut/attention.py:43-46 — softmax(scale q k^T) v
// with the query heads of each KV head sharing it (repeat_kv), causal with the cache offset: query
// position p of lq new tokens sees keys [0, lk - lq + p] of the lk-token cache (the HF mask of a
// prefill over a cache). fp32 accumulation, output in the input dtype.
//
// One CTA per (64 query positions, KV head): two Q tiles, each the group's 4 query heads x 32
// positions = the 128 rows of its MMAs, so each K/V tile is read once for 8 query rows per head
// group and never expanded.
//   warp 8 (one lane): TMA — the two Q tiles once (64-column boxes, 128-byte swizzle), then K and V
//                      tiles of 128 keys through a 2-stage ring (64 KB per stage).
//   warp 9 (one lane): tcgen05.mma issue, per K/V tile: S_0 and S_1 = Q_x K^T (M 128 x N 128 keys x
//                      K 128, A and B K-major from shared memory, fp32 in TMEM), then O_x += P_x V
//                      with P_x read from TMEM (it overwrites the first 64 columns of S_x, 16-bit
//                      pairs) and V MN-major straight from its TMA tile. Order per K/V tile j:
//                      P V_0(j), S_0(j+1), P V_1(j), S_1(j+1) — the ops run in issue order, so S_x(j+1)
//                      overwrites P_x(j) only after P V_x(j) read it, and S_x(j+1)'s commit also
//                      means O_x is current for the softmax's rescale. The tensor core works on one
//                      Q tile while the softmax of the other runs (ping-pong).
//   warps 10-11:       idle (they complete the third warpgroup, which gives its registers to the
//                      softmax warpgroups through setmaxnreg)
//   warps 0-3 / 4-7:   softmax of Q tile 0 / 1 — thread = TMEM lane = one row: tcgen05.ld of the
//                      row's 128 scores, causal mask with the cache offset, exp2, P packed to 16 bits
//                      and tcgen05.st back over S; the row max is kept stale until a tile's max
//                      exceeds it by 2^8, so O_x is rescaled in TMEM (tcgen05.ld/st) only on jumps.
//                      The epilogue divides by l and stores (or, with KV splits, writes fp32
//                      partials and the natural-log LSE for a merge).
// TMEM: 512 columns — S_0 | S_1 | O_0 | O_1. mbarriers order the roles (q_full, kv_full/kv_empty per
// stage, s_full/p_full/o_full per Q tile); every wait is bounded, a failed wait makes all roles
// skip to the end, and the MMA lane's final commit is waited for before TMEM is freed.
#pragma once

#include <type_traits>

#include "tc_common.cuh"

namespace tc {

constexpr int kPfQ = 32;          // query positions per Q tile (x 4 heads = 128 MMA rows)
constexpr int kPfTiles = 2;       // Q tiles per CTA (ping-pong softmax warpgroups)
constexpr int kPfKeys = 128;      // keys per K/V tile
constexpr int kPfThreads = 384;   // warps 0-3 / 4-7 softmax of Q tile 0 / 1, 8 TMA, 9 MMA, 10-11 idle
// Registers per thread after the warpgroup split (setmaxnreg): the launch gives 384 x 168 = 64512,
// softmax warpgroups 2 x 128 x 232 + the TMA/MMA warpgroup 128 x 40 = 64512.
constexpr int kPfRegsSoftmax = 232;
constexpr int kPfRegsOther = 40;
constexpr int kPfGroup = 4;       // query heads per KV head handled by the kernel
constexpr int kPfSmem = 1024 + kPfTiles * 32768 + 2 * 65536;  // alignment slack, Q tiles, 2 K/V stages
constexpr uint32_t kPfSpin = 1u << 20;  // mbarrier polls before a wait gives up (about a second)
// A row keeps its running max until a tile's max exceeds it by more than this (log2 units): P stays
// below 2^8 (exact enough in 16 bits) and O is rescaled in TMEM only on such jumps.
constexpr float kPfLazyMax = 8.f;

struct PrefillParams {
  CUtensorMap tmq;  // (d, lq, hq, 1), box (64, 32, 4, 1)
  CUtensorMap tmk;  // (d, lk, hkv, 1), box (64, 128, 1, 1)
  CUtensorMap tmv;
  void* out;        // element (p, head, dim) at p*so_p + head*so_h + dim
  int64_t so_p, so_h;
  int lq, lk, hq, hkv;
  float c;          // scale * log2(e)
  int nsplit;       // KV splits (grid.z); > 1: fp32 partials + LSE per split, merged afterwards
  float* o_part;    // [nsplit][lq*hq][128] normalised partial outputs (row = position*hq + head)
  float* lse_part;  // [nsplit][lq*hq] natural-log LSE of each partial
  // paged (prefill_kernel<T, true>): K and V live in pages; key tile j is the 32-row sub-tiles
  // [4j, 4j + 4) of ktab (page, first row, rows <= 32, logical position of the first row), loaded
  // as four boxes (64, 32) of (d, page rows, heads, pages) maps; a sub-tile past n_sub is loaded
  // from page oob_page (past the pool: zeros) and masked. qb_tiles[qb] = key tiles visible to
  // query block qb (host-computed from the logical positions).
  const int4* ktab;
  int n_sub;
  int oob_page;
  const int32_t* qb_tiles;
};

// TMEM columns (fp32 words) of Q tile x: S (and P over its first 64 columns), then O.
__device__ __forceinline__ uint32_t pf_col_s(int x) { return (uint32_t)(x * 128); }
__device__ __forceinline__ uint32_t pf_col_o(int x) { return (uint32_t)(256 + x * 128); }

template <typename T, bool kPaged>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                        // Q tile x at +32768*x: 2 boxes x 128 rows x 128 B
  uint8_t* sKV = smem + kPfTiles * 32768;    // stage s: K at +65536*s, V at +65536*s + 32768
  __shared__ __align__(8) uint64_t q_full, kv_full[2], kv_empty[2], s_full[kPfTiles], p_full[kPfTiles],
      o_full[kPfTiles], fin;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heaviest causal Q blocks first (blocks are dispatched in blockIdx.x order): longest-first
  // scheduling shortens the tail when the grid is more than one wave
  const int qb = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int p0 = qb * kPfQ * kPfTiles;  // first position of Q tile 0; tile x starts at p0 + 32x
  const int off = p.lk - p.lq;          // key j is visible to position pos iff j <= off + pos
  const int kend = p.lk < off + p0 + kPfQ * kPfTiles ? p.lk : off + p0 + kPfQ * kPfTiles;
  // >= 1: key 0 is visible to every position
  const int ntot = kPaged ? p.qb_tiles[qb] : (kend + kPfKeys - 1) / kPfKeys;
  const int t_lo = (int)((int64_t)ntot * split / p.nsplit);
  const int ntile = (int)((int64_t)ntot * (split + 1) / p.nsplit) - t_lo;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < kPfTiles; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);
      mbar_init(&o_full[x], 1);
    }
    mbar_init(&fin, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 0) tmem_alloc(&s_tmem, 512);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp >= 8) {
    reg_dealloc<kPfRegsOther>();
  }
  if (warp == 8) {
    // ---------------- TMA producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      prefetch_tensormap(&p.tmq);
      prefetch_tensormap(&p.tmk);
      prefetch_tensormap(&p.tmv);
      mbar_arrive_expect_tx(&q_full, (uint32_t)(kPfTiles * 32768));
      for (int x = 0; x < kPfTiles; ++x)
        for (int bx = 0; bx < 2; ++bx)
          tma_load_4d(sQ + x * 32768 + bx * 16384, &p.tmq, bx * 64, p0 + kPfQ * x, h * kPfGroup, 0, &q_full, pol);
      int armed = 0;  // K/V tiles whose copies were issued
      int4 nxt[4];      // paged: the next tile's sub-tile entries, read one tile ahead
      auto fetch = [&](int j) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int si = 4 * (t_lo + j) + c;
          nxt[c] = si < p.n_sub ? p.ktab[si] : make_int4(p.oob_page, 0, 0, 0);
        }
      };
      if (kPaged && ntile > 0) fetch(0);
      for (int j = 0; j < ntile; ++j) {
        const int s = j & 1;
        int4 cur[4];
        if constexpr (kPaged) {
#pragma unroll
          for (int c = 0; c < 4; ++c) cur[c] = nxt[c];
          if (j + 1 < ntile) fetch(j + 1);
        }
        if (s_abort) break;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin)) {
          s_abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 65536u);
        uint8_t* st = sKV + s * 65536;
        if constexpr (kPaged) {
          // four 32-row boxes per 64 columns, at row offsets 0/32/64/96 of the 128-row swizzled tile
          // (the 128-byte swizzle repeats every 8 rows, so the tile image is the contiguous one)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            for (int bx = 0; bx < 2; ++bx) {
              tma_load_4d(st + bx * 16384 + c * 4096, &p.tmk, bx * 64, cur[c].y, h, cur[c].x, &kv_full[s], pol);
              tma_load_4d(st + 32768 + bx * 16384 + c * 4096, &p.tmv, bx * 64, cur[c].y, h, cur[c].x, &kv_full[s],
                          pol);
            }
        } else {
          for (int bx = 0; bx < 2; ++bx) {
            tma_load_4d(st + bx * 16384, &p.tmk, bx * 64, (t_lo + j) * kPfKeys, h, 0, &kv_full[s], pol);
            tma_load_4d(st + 32768 + bx * 16384, &p.tmv, bx * 64, (t_lo + j) * kPfKeys, h, 0, &kv_full[s], pol);
          }
        }
        armed = j + 1;
      }
      // copies still in flight after an abort must land before the CTA leaves (normally these
      // phases completed long ago and the waits return at once)
      for (int j = armed - 2 > 0 ? armed - 2 : 0; j < armed; ++j)
        mbar_wait(&kv_full[j & 1], (j >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
      mbar_wait(&q_full, 0, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
    }
  } else if (warp == 9) {
    // ---------------- tcgen05.mma issue: per K/V tile S_0, S_1, P V_0, P V_1
    if (lane == 0) {
      const uint32_t idS = umma_idesc_f16(kBf16, false, 128, 128);
      const uint32_t idO = umma_idesc_f16(kBf16, true, 128, 128);
      auto issue_s = [&](int x, int j) {  // S_x = Q_x K_j^T over d in 8 steps of 16
        const uint32_t q0 = smem_u32(sQ + x * 32768), k0 = smem_u32(sKV + (j & 1) * 65536);
        for (int kd = 0; kd < 8; ++kd) {
          const uint32_t o = (uint32_t)((kd >> 2) * 16384 + (kd & 3) * 32);
          umma_f16(tmem + pf_col_s(x), umma_desc_sw128(q0 + o, 16, 1024), umma_desc_sw128(k0 + o, 16, 1024), idS,
                   kd > 0);
        }
      };
      auto issue_pv = [&](int x, int j) {  // O_x (+)= P_x V_j, P_x from TMEM (8 columns per 16 keys)
        const uint32_t v0 = smem_u32(sKV + (j & 1) * 65536 + 32768);
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_tmem_a(tmem + pf_col_o(x), tmem + pf_col_s(x) + (uint32_t)(kk * 8),
                          umma_desc_sw128(v0 + kk * 2048, 16384, 1024), idO, j > 0 || kk > 0);
      };
      // tcgen05.mma ops of one thread run in issue order, so S_x(j+1) may be issued straight after
      // the P V_x(j) that reads P_x(j) from the same columns.
      bool ok = ntile > 0 && mbar_wait(&q_full, 0, TC_DEVERR_PIPE_TIMEOUT, kPfSpin) &&
                mbar_wait(&kv_full[0], 0, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
      if (ok) {
        tmem_fence_after();
        for (int x = 0; x < kPfTiles; ++x) {
          issue_s(x, 0);
          umma_commit(&s_full[x]);
        }
      }
      for (int j = 0; ok && j < ntile; ++j) {
        for (int x = 0; x < kPfTiles; ++x) {
          ok = !s_abort && mbar_wait(&p_full[x], j & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
          if (!ok) break;
          tmem_fence_after();
          issue_pv(x, j);
          umma_commit(&o_full[x]);
          if (x == kPfTiles - 1) umma_commit(&kv_empty[j & 1]);
          if (j + 1 < ntile) {
            if (x == 0) ok = !s_abort && mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
            if (!ok) break;
            issue_s(x, j + 1);
            umma_commit(&s_full[x]);
          }
        }
      }
      if (!ok && ntile > 0) s_abort = 1;
      umma_commit(&fin);  // completes once every MMA issued above has
    }
  } else if (warp < 8) {
    // ---------------- softmax: Q tile x = warp / 4; thread = TMEM lane (warp % 4)*32 + lane = row
    // (query head h*4 + warp % 4, position p0 + 32x + lane)
    reg_alloc<kPfRegsSoftmax>();
    const int x = warp >> 2, wq = warp & 3;
    const int pos = p0 + kPfQ * x + lane;
    const int limit = off + pos;                 // last visible key of this row
    const int limit_min = off + p0 + kPfQ * x;   // smallest limit in this Q tile
    const uint32_t lb = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + pf_col_s(x), tO = tmem + pf_col_o(x);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntile; ++j) {
      int4 te[4];  // paged: this tile's sub-tile entries (read before the wait, which hides the load)
      if constexpr (kPaged) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int si = 4 * (t_lo + j) + c;
          te[c] = si < p.n_sub ? p.ktab[si] : make_int4(0, 0, 0, 0);
        }
      }
      // warp-uniform: tcgen05.ld/st and the votes below are warp-collective
      ok = __all_sync(0xffffffffu, !s_abort && mbar_wait(&s_full[x], j & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin));
      if (!ok) break;
      tmem_fence_after();
      uint32_t v[4][32];
#pragma unroll
      for (int cch = 0; cch < 4; ++cch) tmem_ld32(tS + lb + cch * 32, v[cch]);
      tmem_wait_ld();
      // raw scores, masked (-inf) past this row's last visible key; row max over 8 partial chains
      const int ja = t_lo + j;
      float mx[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) mx[r] = -INFINITY;
      if constexpr (kPaged) {
        // chunk c of the row is sub-tile c: slot e holds logical key te[c].w + e if e < te[c].z
        const bool full = te[0].z == 32 && te[1].z == 32 && te[2].z == 32 && te[3].z == 32 &&
                          te[3].w + 31 <= limit_min;
        if (!full) {
#pragma unroll
          for (int cch = 0; cch < 4; ++cch)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (e >= te[cch].z || te[cch].w + e > limit) v[cch][e] = __float_as_uint(-INFINITY);
        }
      } else {
        const bool masked_tile = (ja + 1) * kPfKeys - 1 > limit_min;
        if (masked_tile) {
#pragma unroll
          for (int cch = 0; cch < 4; ++cch)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (ja * kPfKeys + cch * 32 + e > limit) v[cch][e] = __float_as_uint(-INFINITY);
        }
      }
#pragma unroll
      for (int cch = 0; cch < 4; ++cch)
#pragma unroll
        for (int e = 0; e < 16; ++e)
          mx[e & 7] = fmax3(mx[e & 7], __uint_as_float(v[cch][2 * e]), __uint_as_float(v[cch][2 * e + 1]));
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * p.c;  // exp2 domain (c > 0)
      // lazy max: keep m unless this tile's max passes it by more than kPfLazyMax
      const bool bump = mt > m + kPfLazyMax;
      const float mn = bump ? mt : m;
      const float alpha = !bump ? 1.f : (m == -INFINITY ? 0.f : fast_exp2(m - mn));
      const float mref = mn == -INFINITY ? 0.f : mn;  // no visible key yet (a later KV split): p = 0
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      // P = 2^(s c - mref) over the first 64 columns of this tile's S (all of S is in registers
      // already), one half of the keys at a time so the scores and the packed words are not live
      // together.
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t w[32];  // 16-bit pairs: keys 2e, 2e+1 of this half
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int cch = half * 2 + (e >> 4), k2 = 2 * (e & 15);
          const float2 xy = ffma2(make_float2(__uint_as_float(v[cch][k2]), __uint_as_float(v[cch][k2 + 1])),
                                  make_float2(p.c, p.c), make_float2(-mref, -mref));
          const float a = fast_exp2(xy.x);
          const float bb = fast_exp2(xy.y);
          const float2 r2 = fadd2(make_float2(rs4[2 * (e & 1)], rs4[2 * (e & 1) + 1]), make_float2(a, bb));
          rs4[2 * (e & 1)] = r2.x;
          rs4[2 * (e & 1) + 1] = r2.y;
          w[e] = Mma<T>::pack(a, bb);
        }
        tmem_st32(tS + lb + half * 32, w);
      }
      const float rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      l = l * alpha + rs;
      m = mn;
      // s_full's commit covers P V of tile j-1 (issued before S of tile j), so O is current here
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          uint32_t o[32];
          tmem_ld32(tO + lb + cch * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + lb + cch * 32, o);
        }
      }
      tmem_wait_st();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    if (ok && ntile > 0)
      ok = __all_sync(0xffffffffu, !s_abort && mbar_wait(&o_full[x], (ntile - 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin));
    if (!ok) {
      s_abort = 1;
    } else {
      if (ntile > 0) tmem_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int head = h * kPfGroup + wq;
      if (p.nsplit > 1) {
        // normalised fp32 partial + natural-log LSE (an empty split: zeros and -inf)
        const int64_t row = (int64_t)pos * p.hq + head;
        const int64_t rows = (int64_t)p.lq * p.hq;
        float* orow = p.o_part + ((int64_t)split * rows + row) * 128;
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          uint32_t o[32];
          if (ntile > 0) {
            tmem_ld32(tO + lb + cch * 32, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
          if (pos < p.lq) {
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4)
              *reinterpret_cast<float4*>(orow + cch * 32 + q4 * 4) =
                  make_float4(__uint_as_float(o[4 * q4]) * inv, __uint_as_float(o[4 * q4 + 1]) * inv,
                              __uint_as_float(o[4 * q4 + 2]) * inv, __uint_as_float(o[4 * q4 + 3]) * inv);
          }
        }
        if (pos < p.lq)
          p.lse_part[(int64_t)split * rows + row] = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : -INFINITY;
      } else {
        T* orow = static_cast<T*>(p.out) + (int64_t)pos * p.so_p + (int64_t)head * p.so_h;
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          uint32_t o[32];
          tmem_ld32(tO + lb + cch * 32, o);
          tmem_wait_ld();
          if (pos < p.lq) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint4 w;
              w.x = Mma<T>::pack(__uint_as_float(o[8 * q4 + 0]) * inv, __uint_as_float(o[8 * q4 + 1]) * inv);
              w.y = Mma<T>::pack(__uint_as_float(o[8 * q4 + 2]) * inv, __uint_as_float(o[8 * q4 + 3]) * inv);
              w.z = Mma<T>::pack(__uint_as_float(o[8 * q4 + 4]) * inv, __uint_as_float(o[8 * q4 + 5]) * inv);
              w.w = Mma<T>::pack(__uint_as_float(o[8 * q4 + 6]) * inv, __uint_as_float(o[8 * q4 + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + cch * 32 + q4 * 8) = w;
            }
          }
        }
      }
    }
  }
  // every MMA has completed before the TMEM columns are freed (bounded: a lost commit only errs)
  tmem_fence_before();
  __syncthreads();
  if (warp == 0) {
    mbar_wait(&fin, 0, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
    tmem_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tc
