// GQA prefill attention on the 5th-generation tensor cores (tcgen05), for sm_100a.
//
// Reference semantics: the prefill branch of threadcut/attention.py:43-46 — softmax(scale q k^T) v
// with the query heads of each KV head sharing it (repeat_kv), causal with the cache offset: query
// position p of lq new tokens sees keys [0, lk - lq + p] of the lk-token cache (the HF mask of a
// prefill over a cache). fp32 accumulation, output in the input dtype.
//
// One CTA per (32 query positions, KV head): the 4 query heads of the GQA group x 32 positions form
// the 128 rows of every MMA, so each K/V tile is read once for the group and never expanded.
//   warp 4 (one lane): TMA — Q once (2 boxes of 64 columns, 128-byte swizzle), then K and V tiles of
//                      128 keys through a 2-stage ring (64 KB per stage).
//   warp 5 (one lane): tcgen05.mma issue — S = Q K^T (M 128 x N 128 keys x K 128, A and B K-major,
//                      fp32 in TMEM columns [0,128)), then O += P V (A = P K-major from shared
//                      memory, B = V MN-major straight from the V tile, fp32 in TMEM [128,256)).
//                      S of tile j+1 is issued before P V of tile j, so it overlaps the softmax.
//   warps 0-3:         softmax — thread t owns TMEM lane t = one row (query head h*4 + warp,
//                      position p0 + lane): it reads its 128 scores with tcgen05.ld, masks, keeps
//                      the running max m and sum l in registers, writes P (bf16/f16) into one of
//                      two swizzled P buffers, and rescales its O row in TMEM (tcgen05.ld/st) only
//                      when a row's max jumps by more than 2^8 (the max is otherwise kept stale, so
//                      the softmax of tile j+1 never waits for P V of tile j). The epilogue divides
//                      by l and stores (or, with KV splits, writes fp32 partials and the LSE).
// mbarriers order the roles (q_full, kv_full/kv_empty per stage, s_full/s_free, p_full, o_full);
// every wait is bounded, a failed wait makes all roles skip to the end, and the MMA lane's final
// commit is waited for before the TMEM columns are freed, on every path.
#pragma once

#include <type_traits>

#include "tc_common.cuh"

namespace tc {

constexpr int kPfQ = 32;          // query positions per CTA (x 4 heads = 128 MMA rows)
constexpr int kPfKeys = 128;      // keys per K/V tile
constexpr int kPfThreads = 192;   // warps 0-3 softmax, 4 TMA, 5 MMA
constexpr int kPfGroup = 4;       // query heads per KV head handled by the kernel
constexpr int kPfSmem = 1024 + 32768 + 2 * 65536 + 2 * 32768;  // alignment slack, Q, 2 K/V stages, 2 P
// A row keeps its running max until a tile's max exceeds it by more than this (log2 units): P stays
// below 2^8 (exact enough in 16 bits) and O is rescaled in TMEM only on such jumps.
constexpr float kPfLazyMax = 8.f;
constexpr uint32_t kPfSpin = 1u << 20;  // mbarrier polls before a wait gives up (about a second)

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
};

// Byte offset of 16-byte chunk c (8 elements) of row r in a tile stored as 64-column boxes of R rows
// with the 128-byte swizzle (chunk c of row r at chunk position (c & 7) ^ (r & 7) of its box row).
__device__ __forceinline__ uint32_t pf_swz(int r, int c, int R) {
  return (uint32_t)((c >> 3) * (R * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                      // 2 boxes x 128 rows x 128 B
  uint8_t* sKV = smem + 32768;             // stage s: K at +65536*s, V at +65536*s + 32768
  uint8_t* sP = smem + 32768 + 2 * 65536;  // P of tile j at sP + (j & 1) * 32768: 2 boxes x 128 rows x 128 B
  // one p_full / o_full per P buffer, so a barrier is never more than one phase ahead of its waiter
  __shared__ __align__(8) uint64_t q_full, kv_full[2], kv_empty[2], s_full, s_free, p_full[2], o_full[2], fin;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int p0 = qb * kPfQ;
  const int off = p.lk - p.lq;  // key j is visible to position pos iff j <= off + pos
  const int kend = p.lk < off + p0 + kPfQ ? p.lk : off + p0 + kPfQ;
  const int ntot = (kend + kPfKeys - 1) / kPfKeys;  // >= 1: key 0 is visible to every position
  // this split's tiles [t_lo, t_lo + ntile) of the block's ntot (as even as integer division allows)
  const int t_lo = (int)((int64_t)ntot * split / p.nsplit);
  const int ntile = (int)((int64_t)ntot * (split + 1) / p.nsplit) - t_lo;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_free, 4);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&p_full[s], 4);
      mbar_init(&o_full[s], 1);
    }
    mbar_init(&fin, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 0) tmem_alloc(&s_tmem, 256);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tS = s_tmem, tO = s_tmem + 128;

  if (warp == 4) {
    // ---------------- TMA producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      prefetch_tensormap(&p.tmq);
      prefetch_tensormap(&p.tmk);
      prefetch_tensormap(&p.tmv);
      mbar_arrive_expect_tx(&q_full, 32768u);
      for (int bx = 0; bx < 2; ++bx) tma_load_4d(sQ + bx * 16384, &p.tmq, bx * 64, p0, h * kPfGroup, 0, &q_full, pol);
      int armed = 0;  // K/V tiles whose copies were issued
      for (int j = 0; j < ntile; ++j) {
        const int s = j & 1;
        if (s_abort) break;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin)) {
          s_abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 65536u);
        uint8_t* st = sKV + s * 65536;
        for (int bx = 0; bx < 2; ++bx) {
          tma_load_4d(st + bx * 16384, &p.tmk, bx * 64, (t_lo + j) * kPfKeys, h, 0, &kv_full[s], pol);
          tma_load_4d(st + 32768 + bx * 16384, &p.tmv, bx * 64, (t_lo + j) * kPfKeys, h, 0, &kv_full[s], pol);
        }
        armed = j + 1;
      }
      // copies still in flight after an abort must land before the CTA leaves (normally these
      // phases completed long ago and the waits return at once)
      for (int j = armed - 2 > 0 ? armed - 2 : 0; j < armed; ++j)
        mbar_wait(&kv_full[j & 1], (j >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
      mbar_wait(&q_full, 0, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
    }
  } else if (warp == 5) {
    // ---------------- tcgen05.mma issue
    if (lane == 0) {
      const uint32_t idS = umma_idesc_f16(kBf16, false, 128, 128);
      const uint32_t idO = umma_idesc_f16(kBf16, true, 128, 128);
      const uint32_t q0 = smem_u32(sQ), p0a = smem_u32(sP);
      auto issue_s = [&](int j) {  // S = Q K_j^T over d in 8 steps of 16
        const uint32_t k0 = smem_u32(sKV + (j & 1) * 65536);
        for (int kd = 0; kd < 8; ++kd) {
          const uint32_t o = (uint32_t)((kd >> 2) * 16384 + (kd & 3) * 32);
          umma_f16(tS, umma_desc_sw128(q0 + o, 16, 1024), umma_desc_sw128(k0 + o, 16, 1024), idS, kd > 0);
        }
      };
      auto issue_pv = [&](int j) {  // O (+)= P_j V_j over the 128 keys in 8 steps of 16
        const uint32_t v0 = smem_u32(sKV + (j & 1) * 65536 + 32768);
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t pa = p0a + (uint32_t)((j & 1) * 32768 + (kk >> 2) * 16384 + (kk & 3) * 32);
          umma_f16(tO, umma_desc_sw128(pa, 16, 1024), umma_desc_sw128(v0 + kk * 2048, 16384, 1024), idO,
                   j > 0 || kk > 0);
        }
      };
      bool ok = ntile > 0 && mbar_wait(&q_full, 0, TC_DEVERR_PIPE_TIMEOUT, kPfSpin) &&
                mbar_wait(&kv_full[0], 0, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
      if (ok) {
        tmem_fence_after();
        issue_s(0);
        umma_commit(&s_full);
      }
      for (int j = 0; ok && j < ntile; ++j) {
        if (j + 1 < ntile) {
          ok = !s_abort && mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin) &&
               mbar_wait(&s_free, j & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
          if (!ok) break;
          tmem_fence_after();
          issue_s(j + 1);
          umma_commit(&s_full);
        }
        ok = !s_abort && mbar_wait(&p_full[j & 1], (j >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
        if (!ok) break;
        tmem_fence_after();
        issue_pv(j);
        umma_commit(&o_full[j & 1]);
        umma_commit(&kv_empty[j & 1]);
      }
      if (!ok && ntile > 0) s_abort = 1;
      umma_commit(&fin);  // completes once every MMA issued above has
    }
  } else {
    // ---------------- softmax: thread t = TMEM lane t = row (head h*4 + warp, position p0 + lane)
    const int pos = p0 + lane;
    const int limit = off + pos;       // last visible key of this row
    const int limit_min = off + p0;    // smallest limit in the CTA
    const uint32_t lb = (uint32_t)(warp * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntile; ++j) {
      ok = !s_abort && mbar_wait(&s_full, j & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
      if (!ok) break;
      tmem_fence_after();
      uint32_t v[4][32];
#pragma unroll
      for (int cch = 0; cch < 4; ++cch) tmem_ld32(tS + lb + cch * 32, v[cch]);
      tmem_wait_ld();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free);
      // scores in the exp2 domain, masked past this row's last visible key
      const int ja = t_lo + j;  // absolute tile index
      const bool masked_tile = (ja + 1) * kPfKeys - 1 > limit_min;
      float mt = -INFINITY;
#pragma unroll
      for (int cch = 0; cch < 4; ++cch)
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float x = __uint_as_float(v[cch][e]) * p.c;
          if (masked_tile && ja * kPfKeys + cch * 32 + e > limit) x = -INFINITY;
          v[cch][e] = __float_as_uint(x);
          mt = fmaxf(mt, x);
        }
      // lazy max: keep m unless this tile's max passes it by more than kPfLazyMax
      const bool bump = mt > m + kPfLazyMax;
      const float mn = bump ? mt : m;
      const float alpha = !bump ? 1.f : (m == -INFINITY ? 0.f : fast_exp2(m - mn));
      // a row with no visible key yet (only possible in a later KV split): every p is 0
      const float mref = mn == -INFINITY ? 0.f : mn;
      float rs = 0.f;
      uint32_t pk[4][16];  // P as packed 16-bit pairs
#pragma unroll
      for (int cch = 0; cch < 4; ++cch)
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = fast_exp2(__uint_as_float(v[cch][2 * e]) - mref);
          const float bb = fast_exp2(__uint_as_float(v[cch][2 * e + 1]) - mref);
          rs += a + bb;
          pk[cch][e] = Mma<T>::pack(a, bb);
        }
      l = l * alpha + rs;
      m = mn;
      if (j >= 2) {
        // P buffer j & 1 was last read by P V of tile j - 2
        ok = !s_abort && mbar_wait(&o_full[j & 1], ((j - 2) >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
        if (!ok) break;
      }
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // a row of this warp raised its max: O must hold tiles < j before it is rescaled
        ok = !s_abort && mbar_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
        if (!ok) break;
        tmem_fence_after();
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          uint32_t o[32];
          tmem_ld32(tO + lb + cch * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + lb + cch * 32, o);
        }
        tmem_wait_st();
      }
      // P row (128 keys) into the swizzled A-operand buffer: chunk c = keys 8c..8c+7
      const int r = threadIdx.x;
#pragma unroll
      for (int cch = 0; cch < 4; ++cch)
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          *reinterpret_cast<uint4*>(sP + (j & 1) * 32768 + pf_swz(r, cch * 4 + q4, 128)) =
              make_uint4(pk[cch][4 * q4], pk[cch][4 * q4 + 1], pk[cch][4 * q4 + 2], pk[cch][4 * q4 + 3]);
      fence_proxy_async_smem();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
    }
    if (ok && ntile > 0)
      ok = !s_abort && mbar_wait(&o_full[(ntile - 1) & 1], ((ntile - 1) >> 1) & 1, TC_DEVERR_PIPE_TIMEOUT, kPfSpin);
    if (!ok) {
      s_abort = 1;
    } else {
      if (ntile > 0) tmem_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int head = h * kPfGroup + warp;
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
        if (pos < p.lq) p.lse_part[(int64_t)split * rows + row] = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : -INFINITY;
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
    tmem_dealloc(s_tmem, 256);
  }
}

}  // namespace tc
