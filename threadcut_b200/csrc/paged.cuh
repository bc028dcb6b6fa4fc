// Paged K/V cache kernels (the paged layout the reference names as its next step,
// threadcut README.md:141-144: drop B by freeing pages, rotate C in place with no move).
//
// A layer's K (and V) pool is [pages][heads][page rows][d] with element strides (s_page, s_h,
// s_row); a sequence is a list of row runs inside pages. Device tables describe the rows a kernel
// touches and are never trusted: every access is bounds-checked against the pool, so a bad table
// skips rows instead of writing outside the pool.
//   paged_rotate_kernel: re-rotates keys in place by one RoPE delta (the splice of C), every layer in
//                        one launch; a tile-table entry (page, first row, rows <= 32) per 32-row tile
//                        of C. Bytes = read + write of C's keys only (values never move).
//   paged_write_kernel:  writes t new rows per head (K and V of one layer) to their (page, row) slots.
//   paged_gather_kernel: one layer's K and V copied out in logical order (contiguous views for the
//                        attention paths that do not read pages).
#pragma once

#include <stdint.h>

namespace tc {

constexpr int kPagedTileRows = 32;  // rows per tile-table entry (the decode kernel's tile height)

struct PagedRotateParams {
  void* kp[kMaxLayers];  // K pool of each layer
  int layers, hkv, d;
  int64_t page_rows, num_pages;
  int64_t s_page, s_h, s_row;
  const int32_t* tiles;  // [n_tiles][3]: page, first row, rows
  int64_t n_tiles;
  float cs[kMaxRopeDim];
};

template <typename T, int VEC>
__global__ void __launch_bounds__(256) paged_rotate_kernel(const __grid_constant__ PagedRotateParams p) {
  __shared__ float s_cs[kMaxRopeDim];
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) s_cs[i] = p.cs[i];
  __syncthreads();
  const int half = p.d / 2, cph = half / VEC;
  const int per_tile = kPagedTileRows * cph;  // tasks per (layer, tile, head)
  const int64_t tasks = (int64_t)p.layers * p.n_tiles * p.hkv * per_tile;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < tasks; t += (int64_t)gridDim.x * blockDim.x) {
    const int in_tile = (int)(t % per_tile);
    const int64_t lth = t / per_tile;  // (layer, tile, head)
    const int h = (int)(lth % p.hkv);
    const int64_t lt = lth / p.hkv;
    const int64_t tile = lt % p.n_tiles;
    const int layer = (int)(lt / p.n_tiles);
    const int row = in_tile / cph, ch = in_tile - row * cph;
    const int32_t* tt = p.tiles + 3 * tile;
    const int64_t page = tt[0], r0 = tt[1];
    const int rows = tt[2];
    if (row >= rows) continue;
    const int64_t pr = r0 + row;
    if (page < 0 || page >= p.num_pages || r0 < 0 || pr >= p.page_rows) continue;
    T* x0 = static_cast<T*>(p.kp[layer]) + page * p.s_page + h * p.s_h + pr * p.s_row + ch * VEC;
    Chunk<T, VEC> x = ld_chunk<T, VEC>(x0), y = ld_chunk<T, VEC>(x0 + half);
    rotate_pair<T, VEC>(x, y, s_cs, half, ch * VEC);
    st_chunk<T, VEC>(x0, x);
    st_chunk<T, VEC>(x0 + half, y);
  }
}

struct PagedWriteParams {
  const void* k_src;  // [hkv][t][d] with element strides (src_sh, src_st) for K, (vsrc_sh, vsrc_st) for V
  const void* v_src;
  void* kp;           // this layer's pools
  void* vp;
  int hkv, d;
  int64_t t;
  int64_t src_sh, src_st, vsrc_sh, vsrc_st;
  int64_t page_rows, num_pages;
  int64_t s_page, s_h, s_row;
  const int32_t* slots;  // [t][2]: page, row
};

template <typename T, int VEC>
__global__ void __launch_bounds__(256) paged_write_kernel(const __grid_constant__ PagedWriteParams p) {
  const int cpr = p.d / VEC;  // chunks per row
  const int64_t per = p.t * p.hkv * cpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < 2 * per; i += (int64_t)gridDim.x * blockDim.x) {
    const bool isv = i >= per;
    const int64_t u = isv ? i - per : i;
    const int ch = (int)(u % cpr);
    const int64_t hr = u / cpr;  // (head, new row)
    const int64_t r = hr % p.t;
    const int h = (int)(hr / p.t);
    const int64_t page = p.slots[2 * r], pr = p.slots[2 * r + 1];
    if (page < 0 || page >= p.num_pages || pr < 0 || pr >= p.page_rows) continue;
    const T* src = static_cast<const T*>(isv ? p.v_src : p.k_src) + h * (isv ? p.vsrc_sh : p.src_sh) +
                   r * (isv ? p.vsrc_st : p.src_st) + ch * VEC;
    T* dst = static_cast<T*>(isv ? p.vp : p.kp) + page * p.s_page + h * p.s_h + pr * p.s_row + ch * VEC;
    st_chunk<T, VEC>(dst, ld_chunk<T, VEC>(src));
  }
}

struct PagedGatherParams {
  const void* kp;  // one layer's pools
  const void* vp;
  void* k_out;     // [hkv][n][d] with element strides (out_sh, out_sn)
  void* v_out;
  int hkv, d;
  int64_t n;
  int64_t out_sh, out_sn;
  int64_t page_rows, num_pages;
  int64_t s_page, s_h, s_row;
  const int32_t* tiles;  // [n_tiles][4]: page, first row, rows <= 32, logical position of the first row
  int64_t n_tiles;
};

// Contiguous copy of one layer's sequence (rows in logical order), K and V: one 16-byte chunk
// (or element) per task, tasks ordered (tile, head, row, chunk) so a warp reads and writes whole rows.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) paged_gather_kernel(const __grid_constant__ PagedGatherParams p) {
  const int cpr = p.d / VEC;
  const int per_tile = kPagedTileRows * cpr;
  const int64_t per = p.n_tiles * p.hkv * per_tile;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < 2 * per; i += (int64_t)gridDim.x * blockDim.x) {
    const bool isv = i >= per;
    const int64_t u = isv ? i - per : i;
    const int in_tile = (int)(u % per_tile);
    const int64_t th = u / per_tile;
    const int h = (int)(th % p.hkv);
    const int64_t tile = th / p.hkv;
    const int row = in_tile / cpr, ch = in_tile - row * cpr;
    const int32_t* tt = p.tiles + 4 * tile;
    if (row >= tt[2]) continue;
    const int64_t page = tt[0], pr = (int64_t)tt[1] + row, pos = (int64_t)tt[3] + row;
    if (page < 0 || page >= p.num_pages || tt[1] < 0 || pr >= p.page_rows || pos < 0 || pos >= p.n) continue;
    const T* src = static_cast<const T*>(isv ? p.vp : p.kp) + page * p.s_page + h * p.s_h + pr * p.s_row + ch * VEC;
    T* dst = static_cast<T*>(isv ? p.v_out : p.k_out) + h * p.out_sh + pos * p.out_sn + ch * VEC;
    st_chunk<T, VEC>(dst, ld_chunk<T, VEC>(src));
  }
}

}  // namespace tc
