/*
 * threadcut_b200 — C ABI of the B200 (sm_100a) decode-attention / KV-splice kernels.
 *
 * Every entry point takes plain device pointers, element strides and sizes plus a cudaStream_t
 * passed as `void*` (NULL = legacy default stream). Nothing here allocates, frees or synchronises
 * unless its comment says so; tensors stay owned by the caller. All functions return a TC_* status
 * (0 = TC_OK) and never abort the process. Launch errors are reported as TC_ERR_CUDA.
 *
 * Reference interfaces replaced (file:line inside the threadcut project):
 *   tc_decode_attention*      threadcut/flash_decode.py:57-69   decode_attention(q, k, v, scale, split, block)
 *                             (+ the folded decode branch of threadcut/attention.py:35-42,47)
 *   tc_shift_keys             threadcut/kv.py:20-25             shift_keys(keys, delta, inv_freq)
 *   tc_splice_inplace         threadcut/kv.py:83-92             GrowingLayer.splice(s, inv_freq)
 *                             threadcut/kv.py:28-33             splice(cache, s, inv_freq), all layers
 *   tc_splice_copy            threadcut/kv.py:34-41             splice(...) copy path (non-growing caches)
 *   tc_merge_partials         threadcut/flash_decode.py:68-69   softmax(lse) merge of split partials
 *   tc_decode_attention_paged, tc_prefill_attention_paged, tc_paged_rotate_keys, tc_paged_write,
 *   tc_paged_gather
 *                             threadcut/README.md:141-144       the paged KV layout named there as the next
 *                             step (no reference code): decode over pages (flash_decode.py:57-69 semantics),
 *                             splice as page drop + in-place key rotation (kv.py:28-41,83-92 semantics),
 *                             append into page slots (kv.py:64-77 GrowingLayer.update semantics)
 *   tc_add_rmsnorm, tc_qk_norm_rope, tc_silu_mul, tc_gemv, tc_gemv_swiglu
 *                             threadcut/engine.py:66-73         the per-token model call, run by
 *                             transformers' Qwen3 layer (RMSNorm, q/k norm + RoPE, SwiGLU) there; here
 *                             one launch each in the tensor-parallel decode step
 */
#ifndef THREADCUT_B200_H
#define THREADCUT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
enum {
  TC_OK = 0,
  TC_ERR_INVALID = 1,   /* a size/shape/argument is outside the supported range           */
  TC_ERR_ALIGN = 2,     /* a pointer or stride breaks an alignment rule of the kernel      */
  TC_ERR_DTYPE = 3,     /* unsupported dtype code                                          */
  TC_ERR_WORKSPACE = 4, /* workspace missing or smaller than the *_workspace_size() figure */
  TC_ERR_CUDA = 5       /* a CUDA runtime call or kernel launch failed                      */
};

/* ---- element types ------------------------------------------------------------------- */
enum { TC_F32 = 0, TC_F16 = 1, TC_BF16 = 2 };

/* ---- device-side error bits (see tc_device_errors) ------------------------------------ */
enum {
  TC_DEVERR_PIPE_TIMEOUT = 1, /* a K/V staging wait (mbarrier) ran past its poll limit        */
  TC_DEVERR_FLAG_TIMEOUT = 2, /* an in-place splice wait on another tile ran past its limit  */
  TC_DEVERR_PEER_TIMEOUT = 4  /* a wait for another GPU's rows of a sum ran past its limit    */
};

/* Human-readable name of a TC_* status. */
const char* tc_status_string(int status);

/* ABI version of this library (bumped on any signature change). */
int tc_abi_version(void);

/* Reads (and, if clear != 0, resets) the device error bits of the CURRENT device. This call
 * synchronises the device. Returns the bits, or -1 if the CUDA calls failed. */
int tc_device_errors(int clear);

/* Programmatic dependent launch for this process's later launches (on by default, or off when
 * the environment holds TC_PDL=0): on, a kernel starts while its predecessor in the stream ends
 * and waits for it before reading its results; off, kernels run one after another, so per-kernel
 * device times add up to a step (for launch lists). A CUDA graph keeps the mode it was captured
 * with. Returns the previous mode (1 on, 0 off). No reference counterpart (launch tuning). */
int tc_set_pdl(int on);

/* ======================================================================================
 * Decode attention (one query token per sequence, grouped-query heads folded per KV head).
 *
 * Layout: q[hkv, g, d] (query head hq = kv_head*g + i, as q.reshape(hkv, g, d) in
 * threadcut/attention.py:39), k/v[hkv, n, d], out[hkv, g, d]; the last dimension is contiguous,
 * the other strides are free (a GrowingLayer view has head stride cap*d). Result in the input
 * dtype; math in fp32: softmax(scale * q k^T) v, exactly what flash_decode.py:_partial computes.
 *
 * Limits: d in {16, 32, 64, 128, 256}: 16-bit K/V with d in {64, 128, 256} and 16-byte aligned rows
 * run the tensor-core TMA kernel, everything else (fp32 included, d <= 128) the generic kernel;
 * 1 <= g <= 16, n >= 0 (n == 0 gives
 * zeros, as the reference's empty merge does). splits = 0 picks the KV partition from the SM
 * count; splits > 0 forces that many KV slices per (sequence, head) (capped at 128).
 *
 * Workspace: at least tc_decode_attention_workspace_size(...) bytes of device memory whose first
 * 16*batch*hkv bytes (per-head tickets and counters) are ZERO before the first call; every call
 * leaves them zero again. Beyond that prefix a call writes partial results, so reusing a workspace
 * for a larger batch*hkv needs the larger prefix zeroed first (keep one workspace per batch*hkv).
 * Calls that share a workspace must be ordered (same stream).
 * ====================================================================================== */
size_t tc_decode_attention_workspace_size(int batch, int hkv, int g, int d, int64_t max_n,
                                          int64_t total_tokens, int splits, int dtype);

int tc_decode_attention(const void* q, const void* k, const void* v, void* out,
                        int hkv, int g, int d, int64_t n,
                        int64_t q_stride_h, int64_t q_stride_g,
                        int64_t k_stride_h, int64_t k_stride_n,
                        int64_t v_stride_h, int64_t v_stride_n,
                        int64_t out_stride_h, int64_t out_stride_g,
                        float scale, int splits, int dtype,
                        void* workspace, size_t workspace_bytes, void* stream);

/* tc_decode_attention plus a declaration that lets the kernel start reading K/V before the kernel
 * ahead of it in the stream has finished: rows [0, stable_rows) of K and V (clamped to n) are
 * written by no kernel that may still be running when this launch starts. The kernel is launched
 * with programmatic dependent launch; when the kernel ahead of it is one of these decode kernels
 * it lets this one start early, and this one then loads the stable rows of its first pipeline
 * stages before waiting for that kernel to finish; q and every other input are read after the
 * wait. In a decode step every row but the one just appended is stable (stable_rows = n - 1).
 * stable_rows = 0 is tc_decode_attention exactly. (No counterpart in the reference: its decode
 * reads the cache after the append has completed.) */
int tc_decode_attention_stable(const void* q, const void* k, const void* v, void* out,
                               int hkv, int g, int d, int64_t n,
                               int64_t q_stride_h, int64_t q_stride_g,
                               int64_t k_stride_h, int64_t k_stride_n,
                               int64_t v_stride_h, int64_t v_stride_n,
                               int64_t out_stride_h, int64_t out_stride_g,
                               float scale, int splits, int dtype, int64_t stable_rows,
                               void* workspace, size_t workspace_bytes, void* stream);

/* GrowingLayer.update of one token fused with the decode that follows it (threadcut/kv.py:64-77
 * then flash_decode.py:57-69): k_new/v_new [hkv, d] (head strides k_new_stride_h/v_new_stride_h,
 * last dim contiguous) are written as row n-1 of the cache views k/v [hkv, n, d], and `out` is
 * attention of q over all n rows, rows [0, n-1) read from the cache and row n-1 from k_new/v_new.
 * One launch with the tensor-core kernel (the CTA whose tile holds row n-1 patches it into its
 * staged tile and stores it to the cache); otherwise two strided copies, then the decode. The
 * cache rows [0, n-1) must not be written by the caller meanwhile; stable_rows as for
 * tc_decode_attention_stable. (The reference appends with a separate copy before attention.) */
int tc_decode_attention_append(const void* q, const void* k_new, const void* v_new, void* k, void* v, void* out,
                               int hkv, int g, int d, int64_t n,
                               int64_t q_stride_h, int64_t q_stride_g,
                               int64_t k_new_stride_h, int64_t v_new_stride_h,
                               int64_t k_stride_h, int64_t k_stride_n,
                               int64_t v_stride_h, int64_t v_stride_n,
                               int64_t out_stride_h, int64_t out_stride_g,
                               float scale, int splits, int dtype, int64_t stable_rows,
                               void* workspace, size_t workspace_bytes, void* stream);

/* tc_decode_attention_append with the Qwen3 q/k norm and RoPE in front of it, one launch: q
 * [hkv, g, d] and k_new [hkv, d] are the raw projections; each query row and each k_new row gets
 * RMSNorm over d (weights q_norm_weight / k_norm_weight [d], eps) and the rotate-half RoPE with
 * cos_t/sin_t [d], with exactly tc_qk_norm_rope's arithmetic, and the rotated k_new is the row
 * written to the cache (v_new as given). Replaces, for one decode token, transformers' Qwen3Attention
 * steps q_norm, k_norm, apply_rotary_pos_emb and the cache update in front of the plugin call
 * (threadcut/attention.py:30-42, kv.py:64-77). bf16/fp16, d in {64, 128, 256}, 16-byte aligned K/V
 * and rows only (TC_ERR_ALIGN / TC_ERR_INVALID otherwise: no other kernel does this fusion); q,
 * k_new, the weights and cos/sin are read after the previous kernel in the stream completes. */
int tc_decode_attention_append_rope(const void* q, const void* k_new, const void* v_new, void* k, void* v,
                                    void* out, int hkv, int g, int d, int64_t n,
                                    int64_t q_stride_h, int64_t q_stride_g,
                                    int64_t k_new_stride_h, int64_t v_new_stride_h,
                                    int64_t k_stride_h, int64_t k_stride_n,
                                    int64_t v_stride_h, int64_t v_stride_n,
                                    int64_t out_stride_h, int64_t out_stride_g,
                                    const void* q_norm_weight, const void* k_norm_weight,
                                    const void* cos_t, const void* sin_t, float eps,
                                    float scale, int splits, int dtype, int64_t stable_rows,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* split(cached, new, min_suffix, suffix) of threadcut/match.py:33-48 on the device: token ids as
 * int32 device arrays (n_new >= 1). Writes (a, c0, c) of the resulting Split as three int64 to the
 * device pointer out3; identical to the host rule, ties included (the first start with the longest
 * match). Workspace: tc_split_workspace_size(n_cached) bytes, 8-byte aligned, no initial contents.
 * (No counterpart in the reference: it splits on the host with numpy.) */
size_t tc_split_workspace_size(int64_t n_cached);
int tc_split(const int32_t* cached, int64_t n_cached, const int32_t* new_tokens, int64_t n_new,
             int min_suffix, int suffix, int64_t* out3, void* workspace, size_t workspace_bytes,
             void* stream);

/* GQA prefill attention on the tcgen05 tensor cores (threadcut/attention.py:43-46 without the
 * repeat_kv expansion): q [hq, lq, d] (strides q_stride_h, q_stride_p), k/v [hkv, lk, d], out
 * [lq, hq, d] (strides out_stride_p, out_stride_h); query position p attends to keys
 * [0, lk - lq + p] (a prefill of lq new tokens over an lk-token cache that ends with them).
 * bf16/f16, d = 128, hq = 4*hkv, 1 <= lq <= lk; 16-byte aligned bases and strides. Other shapes
 * return TC_ERR_INVALID / TC_ERR_ALIGN. splits = 0 picks the number of KV splits from the SM count
 * (tc_prefill_splits); with more than one, fp32 partials are merged by log-sum-exp (out must then be
 * contiguous [lq, hq, d], else one split is used) in `workspace` of tc_prefill_workspace_size()
 * bytes (no initial contents). */
int tc_prefill_splits(int hkv, int lq, int lk);
size_t tc_prefill_workspace_size(int hq, int hkv, int lq, int lk, int splits);
int tc_prefill_attention(const void* q, const void* k, const void* v, void* out,
                         int hq, int hkv, int lq, int lk, int d,
                         int64_t q_stride_h, int64_t q_stride_p,
                         int64_t k_stride_h, int64_t k_stride_n,
                         int64_t v_stride_h, int64_t v_stride_n,
                         int64_t out_stride_p, int64_t out_stride_h,
                         float scale, int splits, int dtype,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Decode attention that allocates nothing, for callers that cannot hand us device memory: for
 * example a plugin running inside another runtime that owns every device allocation and forbids
 * allocating in its execute hook, a loop where the implicit synchronisation of cudaMalloc is not
 * acceptable, or plain C code with no allocator at hand. Same arguments and result as
 * tc_decode_attention, minus the workspace. (This entry point has no counterpart in the reference.)
 *
 * Its scratch is one fixed 4 MiB array compiled into the library; every GPU that loads the library
 * keeps it for the life of the process. Problems whose workspace (tc_decode_attention_workspace_size
 * with batch 1) exceeds 4 MiB are rejected with TC_ERR_WORKSPACE; Qwen3-4B's geometry (8 KV heads,
 * 4 query heads each, head_dim 128) fits at every context length. The first call on a device looks
 * up the array's device address (with that device current), so make that first call before any
 * stream capture; the address is looked up again after the device's context changed (a
 * cudaDeviceReset loads the library's device code anew). All calls share the one array and it
 * keeps the last call's contents: each call
 * clears what must start at zero, but calls that run at the same time on the GPU (different streams,
 * different host threads) race with each other — order them. */
int tc_decode_attention_noalloc(const void* q, const void* k, const void* v, void* out,
                                int hkv, int g, int d, int64_t n,
                                int64_t q_stride_h, int64_t q_stride_g,
                                int64_t k_stride_h, int64_t k_stride_n,
                                int64_t v_stride_h, int64_t v_stride_n,
                                int64_t out_stride_h, int64_t out_stride_g,
                                float scale, int splits, int dtype, void* stream);

/* Batched decode over `batch` sequences sharing one strided K/V tensor [batch, hkv, n, d].
 * `lengths` (device int32[batch], may be NULL = all n) gives each sequence's valid length
 * (<= n); the folded SDPA branch of threadcut/attention.py:41-42 (b > 1) is the reference. */
int tc_decode_attention_batched(const void* q, const void* k, const void* v, void* out,
                                int batch, int hkv, int g, int d, int64_t n,
                                const int32_t* lengths,
                                int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_g,
                                int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_n,
                                int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_n,
                                int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_g,
                                float scale, int splits, int dtype,
                                void* workspace, size_t workspace_bytes, void* stream);

/* Ragged decode: sequence b has its own K/V allocation k_ptrs[b]/v_ptrs[b] of shape
 * [hkv, cap_b >= lengths[b], d] with head stride head_strides[b] (elements) and token stride
 * kv_stride_n, shared by K and V. k_ptrs, v_ptrs, head_strides and lengths are DEVICE arrays.
 * Every K/V base must be 16-byte aligned and head/token strides multiples of 8 elements (16-bit
 * types) — the caller guarantees this; it cannot be checked without reading device memory.
 * `tensormaps` (DEVICE, 64-byte aligned, may be NULL) holds the 2*batch maps written by
 * tc_ragged_encode_tensormaps for these caches; with it 16-bit caches of d in {64,128,256} take
 * the tensor-core TMA kernel, without it the generic kernel.
 * max_n >= every length; total_tokens = sum of lengths (a scheduling hint; 0 = batch*max_n). */
int tc_decode_attention_ragged(const void* q, void* out,
                               const void* const* k_ptrs, const void* const* v_ptrs,
                               const int64_t* head_strides, const int32_t* lengths, const void* tensormaps,
                               int batch, int hkv, int g, int d, int64_t max_n, int64_t total_tokens,
                               int64_t kv_stride_n,
                               int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_g,
                               int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_g,
                               float scale, int splits, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of the tensor-map array for `batch` ragged sequences (2 maps of 128 bytes each). */
size_t tc_ragged_tensormaps_size(int batch);

/* Encodes, on the host, the K and V tensor maps of each ragged sequence into host_out
 * (tc_ragged_tensormaps_size(batch) bytes): k_ptrs/v_ptrs/caps/head_strides are HOST arrays here;
 * cap_b is the row capacity of sequence b's allocation (rows in [length, cap) are masked). Copy the
 * result to 64-byte aligned device memory and pass it to tc_decode_attention_ragged. 16-bit dtypes,
 * d in {64, 128, 256}. */
int tc_ragged_encode_tensormaps(void* host_out, const void* const* k_ptrs, const void* const* v_ptrs,
                                const int64_t* caps, const int64_t* head_strides, int64_t kv_stride_n,
                                int batch, int hkv, int d, int dtype);

/* ======================================================================================
 * Paged K/V cache. A layer's K and V pools are [pages][hkv][page_rows][d] (element strides
 * pool_stride_page/_h/_row, last dim contiguous, 16-byte aligned rows); one sequence is an ordered
 * list of row runs inside pages. Tile tables are DEVICE int32 arrays [n_tiles][3] = (page, first
 * row, rows) with 1 <= rows <= 32 and first row + rows <= page_rows; every kernel bounds-checks
 * them against the pool (a bad entry is skipped or clamped, never accessed out of the pool).
 *
 * tc_decode_attention_paged: decode attention (as tc_decode_attention) of q [hkv][g][d] over the
 * n_tokens rows the tile table lists, in any order (decode has no mask beyond the rows listed).
 * 16-bit dtypes, d in {64, 128, 256}, page_rows >= 32. k_new/v_new (both or neither): the step's
 * new row [hkv][d] (head strides k_new_stride_h/v_new_stride_h) is the last row of the last tile;
 * the cache still holds stale data there and the launch writes the row into the pools while it
 * decodes (fused append). stable_tiles (as stable_rows of tc_decode_attention_stable): tiles
 * [0, stable_tiles) of the table, and the rows they list, are written by no kernel that can still
 * be running when this launch starts, so it may load them before the previous kernel in the stream
 * has finished; 0 is the plain call. In a decode step over several layers every tile qualifies
 * except those holding rows the previous launch wrote. Workspace:
 * tc_decode_attention_workspace_size(1, hkv, g, d, 32 * n_tiles, 0, splits, dtype) bytes, first
 * 16*hkv bytes ZERO before the first call.
 * ====================================================================================== */
int tc_decode_attention_paged(const void* q, const void* k_pool, const void* v_pool, void* out,
                              int hkv, int g, int d, int64_t page_rows, int64_t num_pages,
                              int64_t pool_stride_page, int64_t pool_stride_h, int64_t pool_stride_row,
                              const int32_t* tiles, int64_t n_tiles, int64_t n_tokens,
                              const void* k_new, const void* v_new, int64_t k_new_stride_h,
                              int64_t v_new_stride_h,
                              int64_t q_stride_h, int64_t q_stride_g, int64_t out_stride_h, int64_t out_stride_g,
                              float scale, int splits, int dtype, int64_t stable_tiles,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Causal prefill over a paged cache (as tc_prefill_attention, the causal-over-cache mask: query p
 * sees logical keys [0, lk - lq + p]): the lk logical keys are the rows of a sub-tile table
 * `ktab` (DEVICE int32 [n_sub][4] = page, first row, rows <= 32, logical position of the first
 * row; consecutive in logical order, 16-byte aligned), key tile j being sub-tiles [4j, 4j + 4);
 * qb_tiles (DEVICE int32, one per 64-query block) = the key tiles with a logical start below
 * min(lk, lk - lq + 64 * (block + 1)), at least 1. Pool rows that no sub-tile lists must hold
 * finite values (masked slots meet them with a zero weight). hq = 4 * hkv, d = 128, 16-bit.
 * Workspace as tc_prefill_workspace_size(hq, hkv, lq, 128 * ceil(n_sub / 4), splits). */
int tc_prefill_attention_paged(const void* q, const void* k_pool, const void* v_pool, void* out, int hq, int hkv,
                               int lq, int lk, int d, int64_t page_rows, int64_t num_pages, int64_t pool_stride_page,
                               int64_t pool_stride_h, int64_t pool_stride_row, const int32_t* ktab, int64_t n_sub,
                               const int32_t* qb_tiles, int64_t q_stride_h, int64_t q_stride_p,
                               int64_t out_stride_p, int64_t out_stride_h, float scale, int splits, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Re-rotates, in place, the keys of the rows the tile table lists in every layer's K pool
 * (k_pools: HOST array of `layers` device pointers, layers <= 128) by one RoPE delta (cos_sin as
 * in tc_shift_keys): the splice of C in a paged cache, where B's pages are dropped by the caller
 * and no row moves. Values are not touched. Each row is read and written by one thread. */
int tc_paged_rotate_keys(void* const* k_pools, int layers, int hkv, int d, int64_t page_rows, int64_t num_pages,
                         int64_t pool_stride_page, int64_t pool_stride_h, int64_t pool_stride_row,
                         const int32_t* tiles, int64_t n_tiles, const float* cos_sin, int dtype, void* stream);

/* Writes t new rows per head (K and V sources [hkv][t][d] with the given strides) of one layer to
 * their slots: DEVICE int32 array [t][2] = (page, row). */
int tc_paged_write(const void* k_src, const void* v_src, void* k_pool, void* v_pool, int hkv, int d, int64_t t,
                   int64_t src_stride_h, int64_t src_stride_t, int64_t vsrc_stride_h, int64_t vsrc_stride_t,
                   int64_t page_rows, int64_t num_pages, int64_t pool_stride_page, int64_t pool_stride_h,
                   int64_t pool_stride_row, const int32_t* slots, int dtype, void* stream);

/* One layer's sequence copied out of the pools in logical order: k_out/v_out [hkv][n][d] (element
 * strides out_stride_h/out_stride_n, last dim contiguous); `tiles` is the DEVICE int32 [n_tiles][4]
 * table of tc_prefill_attention_paged (page, first row, rows, logical position of the first row).
 * Rows whose logical position falls outside [0, n) are skipped. */
int tc_paged_gather(const void* k_pool, const void* v_pool, void* k_out, void* v_out, int hkv, int d, int64_t n,
                    int64_t out_stride_h, int64_t out_stride_n, int64_t page_rows, int64_t num_pages,
                    int64_t pool_stride_page, int64_t pool_stride_h, int64_t pool_stride_row, const int32_t* tiles,
                    int64_t n_tiles, int dtype, void* stream);

/* ======================================================================================
 * RoPE key shift: out = k*cos(delta*theta) + rotate_half(k)*sin(delta*theta), in fp32 with the
 * products and the sum rounded separately (as torch evaluates threadcut/kv.py:25), then rounded
 * to the storage dtype. `cos_sin` is a HOST array of d floats: d/2 cosines then d/2 sines of
 * delta*inv_freq[i]; it is copied into the launch, so it may be freed on return.
 * keys/out: [outer, n, d] with the given strides (last dim contiguous). d even, d <= 512.
 * ====================================================================================== */
int tc_shift_keys(const void* keys, void* out, int64_t outer, int64_t n, int d,
                  int64_t in_stride_outer, int64_t in_stride_n,
                  int64_t out_stride_outer, int64_t out_stride_n,
                  const float* cos_sin, int dtype, void* stream);

/* ======================================================================================
 * In-place splice A.B.C -> A.C of `layers` growing K/V buffers in ONE launch
 * (GrowingLayer.splice on every layer): rows [c0, c0+c) of each head move to [a, a+c); keys are
 * re-rotated by -(c0-a) positions (cos_sin of delta = a-c0, as in tc_shift_keys), values copied.
 * Source and destination may overlap: tiles are handed out in order and a tile writes only after
 * the tiles whose sources it overwrites have been read (bounded waits, TC_DEVERR_FLAG_TIMEOUT).
 * kbufs/vbufs: HOST arrays of `layers` device pointers (layers <= 128), each [hkv, cap, d] with
 * strides (stride_h, stride_n); c0 + c <= cap is checked (TC_ERR_INVALID otherwise).
 * c0 == a is a no-op (the reference clones C onto itself).
 * Workspace: tc_splice_workspace_size() bytes, first 16 bytes ZERO before the first use (left
 * zero again); `epoch` must differ from the epoch of every earlier call on this workspace
 * (a counter starting at 1 does).
 * ====================================================================================== */
size_t tc_splice_workspace_size(int layers, int hkv, int64_t c);

int tc_splice_inplace(void* const* kbufs, void* const* vbufs, int layers, int hkv, int d,
                      int64_t cap, int64_t a, int64_t c0, int64_t c, int64_t stride_h, int64_t stride_n,
                      const float* cos_sin, int dtype,
                      void* workspace, size_t workspace_bytes, uint32_t epoch, void* stream);

/* Copy splice into fresh buffers (the non-GrowingLayer path of threadcut/kv.py:34-41):
 * out[:, :a] = in[:, :a]; out[:, a:a+c] = shift(in[:, c0:c0+c]) for keys (plain copy for
 * values, or when c0 == a). In and out must not overlap. Strides per tensor, last dim contiguous. */
int tc_splice_copy(const void* k_in, const void* v_in, void* k_out, void* v_out,
                   int hkv, int d, int64_t a, int64_t c0, int64_t c,
                   int64_t in_stride_h, int64_t in_stride_n,
                   int64_t out_stride_h, int64_t out_stride_n,
                   const float* cos_sin, int dtype, void* stream);

/* ======================================================================================
 * Log-sum-exp merge of `parts` partial attention results (the merge of
 * threadcut/flash_decode.py:68-69, also the cross-GPU combine of sequence-sharded decode):
 * o_parts: fp32 [parts, rows, d], each part's output normalised by its own softmax sum;
 * lse_parts: fp32 [parts, rows] natural-log log-sum-exp of the scaled scores (-inf = empty part).
 * out[rows, d] (row stride out_stride_row) = sum_p softmax_p(lse)[p] * o_parts[p].
 * ====================================================================================== */
int tc_merge_partials(const float* o_parts, const float* lse_parts, void* out, float* lse_out,
                      int parts, int64_t rows, int d, int64_t out_stride_row,
                      int dtype, void* stream);

/* Decode attention that also returns each row's natural-log log-sum-exp (fp32 [hkv, g], may be
 * NULL): the partial-result form used by sequence-sharded decode. Same rules as
 * tc_decode_attention. */
int tc_decode_attention_lse(const void* q, const void* k, const void* v, void* out, float* lse,
                            int hkv, int g, int d, int64_t n,
                            int64_t q_stride_h, int64_t q_stride_g,
                            int64_t k_stride_h, int64_t k_stride_n,
                            int64_t v_stride_h, int64_t v_stride_n,
                            int64_t out_stride_h, int64_t out_stride_g,
                            float scale, int splits, int dtype,
                            void* workspace, size_t workspace_bytes, void* stream);

/* The partial form of a KV slice for sequence-sharded decode across GPUs: like
 * tc_decode_attention_lse, but the output is written unrounded as fp32 [hkv, g, d] (strides of
 * out_f32 in elements) and `lse` is required. Partials of disjoint token ranges of one sequence
 * combine exactly with tc_merge_partials (threadcut/flash_decode.py:68-69 does the same merge over
 * the slices of one GPU). */
int tc_decode_attention_partial(const void* q, const void* k, const void* v, float* out_f32, float* lse,
                                int hkv, int g, int d, int64_t n,
                                int64_t q_stride_h, int64_t q_stride_g,
                                int64_t k_stride_h, int64_t k_stride_n,
                                int64_t v_stride_h, int64_t v_stride_n,
                                int64_t out_stride_h, int64_t out_stride_g,
                                float scale, int splits, int dtype,
                                void* workspace, size_t workspace_bytes, void* stream);

/* tc_decode_attention_partial with the stable-rows declaration of tc_decode_attention_stable (the
 * per-rank step of a sequence-sharded decode, where every row of the rank's slice but the newest
 * is stable). No counterpart in the reference beyond tc_decode_attention_partial's. */
int tc_decode_attention_partial_stable(const void* q, const void* k, const void* v, float* out_f32, float* lse,
                                       int hkv, int g, int d, int64_t n,
                                       int64_t q_stride_h, int64_t q_stride_g,
                                       int64_t k_stride_h, int64_t k_stride_n,
                                       int64_t v_stride_h, int64_t v_stride_n,
                                       int64_t out_stride_h, int64_t out_stride_g,
                                       float scale, int splits, int dtype, int64_t stable_rows,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* Per-token layer ops of the tensor-parallel decode step (threadcut_b200/tp.py), each one launch in
 * place of a chain of torch ops of transformers' Qwen3 layer (modeling_qwen3.py; threadcut runs
 * that layer through transformers, threadcut/engine.py:66-73). Row-major contiguous tensors of
 * `dtype`; rounding to dtype after each torch op they replace.
 *
 * tc_add_rmsnorm: for each of `rows` rows of `hidden` elements, h += delta (delta may be NULL:
 * no add), out = weight * dtype(h * rsqrt(mean(h^2) + eps)) (Qwen3RMSNorm.forward, with the
 * residual add of Qwen3DecoderLayer.forward before it). h is updated in place. */
int tc_add_rmsnorm(void* h, const void* delta, const void* weight, void* out, int64_t rows, int hidden,
                   float eps, int dtype, void* stream);

/* tc_qk_norm_rope: in place on q [q_heads][d] and k [k_heads][d]: per-head RMSNorm with
 * q_weight / k_weight [d] (q_norm / k_norm), then x*cos + rotate_half(x)*sin with cos, sin [d] of
 * dtype (apply_rotary_pos_emb). d even, at most 1024. */
int tc_qk_norm_rope(void* q, void* k, const void* q_weight, const void* k_weight, const void* cos_t,
                    const void* sin_t, int q_heads, int k_heads, int d, float eps, int dtype, void* stream);

/* tc_gemv: out[i] = sum_k x[k] * w[i][k] for i < n (x [k], w [n][k] row-major, out [n]): the one-token
 * projections of the step (nn.Linear with no bias), fp32 accumulation rounded once to dtype. 16-bit
 * dtypes, k a multiple of 8 and at most 24576, x and w 16-byte aligned (else TC_ERR_ALIGN). */
int tc_gemv(const void* x, const void* w, void* out, int64_t n, int k, int dtype, void* stream);

/* tc_gemv_swiglu: tc_gemv of x = dtype(dtype(silu(gate)) * up) computed from gate_up [2k] (gate and
 * up side by side: the fused gate/up projection's output), i.e. tc_silu_mul followed by tc_gemv in
 * one launch (Qwen3MLP's down_proj(act_fn(gate_proj(x)) * up_proj(x))), bit-identical to the two. */
int tc_gemv_swiglu(const void* gate_up, const void* w, void* out, int64_t n, int k, int dtype, void* stream);

/* tc_silu_mul: out[r][i] = dtype(silu(gate_up[r][i])) * gate_up[r][inter + i] for `rows` rows
 * (Qwen3MLP: act_fn(gate_proj(x)) * up_proj(x), gate and up side by side in one row). */
int tc_silu_mul(const void* gate_up, void* out, int64_t rows, int inter, int dtype, void* stream);

/* ---- sums over the GPUs of a tensor-parallel step, through peer memory ------------------
 * No counterpart in the reference (threadcut runs one GPU); they replace the collective library's
 * all-reduce after the two row-split projections of each layer of threadcut_b200/tp.py.
 *
 * Peer regions: every rank allocates one region (tc_peer_alloc, at set-up: cudaMalloc + zero +
 * cudaIpcGetMemHandle), hands the tc_peer_handle_bytes() handle bytes to the other ranks (any
 * host transport), and maps theirs (tc_peer_open, cudaIpcOpenMemHandle). Kernels then read and
 * write peers' regions with plain loads and stores over NVLink; nothing here uses TMA or multicast.
 * tc_peer_close unmaps a peer's region, tc_peer_free frees the own one. */
size_t tc_peer_handle_bytes(void);
int tc_peer_alloc(size_t bytes, void** dev_ptr, void* handle_out);
int tc_peer_open(const void* handle, void** dev_ptr);
int tc_peer_close(void* dev_ptr);
int tc_peer_free(void* dev_ptr);

/* Bytes of the all-reduce region of one rank for `world` ranks summing vectors of `rows` elements
 * (a control word, then two slots of world x rows 8-byte words). */
size_t tc_allreduce_region_bytes(int world, int64_t rows);

/* tc_gemv_allreduce: the rows of tc_gemv (x [k] . w[n][k]^T, fp32 accumulation), each sent as an
 * fp32 word tagged with the sum's number to every rank's region (regions[p]: rank p's region as
 * mapped in this process, p < world <= 8; regions[rank] is this rank's own). n = the regions'
 * `rows`. Must be followed, on every rank and in the same order, by tc_allreduce_add_rmsnorm.
 * tc_allreduce_add_rmsnorm: delta = dtype(sum over ranks of their rows, in rank order, fp32), then
 * tc_add_rmsnorm with that delta: h += delta (rounded) in place, out = RMSNorm(h) * weight. It waits
 * (bounded; TC_DEVERR_PEER_TIMEOUT) for every rank's rows of the current sum. hidden = rows <= 8192.
 * Every rank ends with the same bits in h and out. */
int tc_gemv_allreduce(const void* x, const void* w, int64_t n, int k, void* const* regions, int world, int rank,
                      int dtype, void* stream);
/* tc_gemv_allreduce of the SwiGLU activation of gate_up [2k], as tc_gemv_swiglu. */
int tc_gemv_allreduce_swiglu(const void* gate_up, const void* w, int64_t n, int k, void* const* regions, int world,
                             int rank, int dtype, void* stream);
int tc_allreduce_add_rmsnorm(void* h, const void* weight, void* out, int hidden, float eps, void* region,
                             int world, int dtype, void* stream);

/* The residual form, with no summing kernel: tc_gemv_allreduce_residual sends its rows like
 * tc_gemv_allreduce, then each CTA waits (bounded; TC_DEVERR_PEER_TIMEOUT) for the other ranks'
 * words of its own rows and adds the sum into the residual: h[i] = dtype(h[i] + dtype(sum over
 * ranks, rank order)), the arithmetic of tc_allreduce_add_rmsnorm (every rank ends with the same
 * bits of h [n]); it also records, in this rank's region, the sum of squares of the new h. With
 * world == 1 no word is sent (regions[0] is this rank's region) and h += the rounded product.
 * tc_gemv_rmsnorm, after it: out [n] = RMSNorm(h) * norm_weight (hidden = k, eps; 1/rms from the
 * recorded sums of squares, in a fixed order) times w [n][k]^T — the norm is the GEMV's input
 * staging. Together they replace the transformers Qwen3 residual add + RMSNorm + next projection
 * of the per-token model call (threadcut/engine.py:66-73) in the tensor-parallel step, two
 * launches where tc_gemv_allreduce + tc_allreduce_add_rmsnorm + tc_gemv are three. Every rank
 * calls them in the same order, each residual sum followed by one tc_gemv_rmsnorm before the next
 * residual sum; the region must be tc_allreduce_region_bytes(world, n) bytes, zeroed. */
int tc_gemv_allreduce_residual(const void* x, const void* w, int64_t n, int k, void* const* regions, int world,
                               int rank, void* h, int dtype, void* stream);
/* tc_gemv_allreduce_residual of the SwiGLU activation of gate_up [2k], as tc_gemv_swiglu. */
int tc_gemv_allreduce_residual_swiglu(const void* gate_up, const void* w, int64_t n, int k, void* const* regions,
                                      int world, int rank, void* h, int dtype, void* stream);
int tc_gemv_rmsnorm(const void* h, const void* norm_weight, const void* region, float eps, const void* w, void* out,
                    int64_t n, int k, int dtype, void* stream);
/* tc_gemv_rmsnorm of the MLP's gate/up projection with its rows interleaved (row 2i: the gate row
 * of intermediate i, row 2i + 1: its up row; n even), writing the SwiGLU activation instead of
 * the projection: out [n/2], out[i] = T(T(silu(gate_i)) * up_i) with gate_i and up_i the
 * projection's outputs rounded to the dtype, tc_silu_mul's arithmetic. The down projection after it
 * then takes a plain input (tc_gemv_allreduce_residual) instead of computing the activation in
 * every CTA (tc_gemv_allreduce_residual_swiglu). Replaces the gate_proj/up_proj + act_fn * up of
 * transformers' Qwen3 MLP in the per-token model call (threadcut/engine.py:66-73). */
int tc_gemv_rmsnorm_swiglu(const void* h, const void* norm_weight, const void* region, float eps, const void* w,
                           void* out, int64_t n, int k, int dtype, void* stream);

/* All-gather + log-sum-exp merge of sequence-shard partials through peer memory, one launch: every
 * rank's fp32 partial o_local [rows][d] (normalised) and natural-log lse_local [rows] of its token
 * slice (tc_decode_attention_partial*) are pushed into every other rank's region (regions as for
 * tc_gemv_allreduce, each of tc_gather_region_bytes(world, rows, d) bytes, zeroed), and out [rows][d]
 * (row stride out_stride_row, dtype) and lse_out (optional) are the merge of all ranks' partials in
 * rank order: the arithmetic of tc_merge_partials (threadcut/flash_decode.py:68-69 over the ranks),
 * the same bits on every rank. Waits (bounded; TC_DEVERR_PEER_TIMEOUT) for the other ranks' data.
 * Every rank calls it in the same order; d % 4 == 0, o_local 16-byte aligned. No counterpart in the
 * reference (one GPU): it replaces an NCCL all-gather of the partials plus tc_merge_partials. */
size_t tc_gather_region_bytes(int world, int64_t rows, int d);
int tc_peer_gather_merge(const float* o_local, const float* lse_local, void* out, float* lse_out, int64_t rows, int d,
                         int64_t out_stride_row, void* const* regions, int world, int rank, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* THREADCUT_B200_H */
