// threadcut_b200 C ABI: host launchers for the decode-attention and splice kernels.
// This is the library's only translation unit; it includes every kernel header.
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "decode_attn.cuh"
#include "rope_splice.cuh"
#include "paged.cuh"
#include "split.cuh"
#include "prefill_attn.cuh"
#include "layer_ops.cuh"
#include "peer.cuh"
#include "gemv_stream.cuh"

using namespace tc;

namespace {

std::mutex g_mu;
std::set<std::pair<const void*, int>> g_smem_configured;
int g_sm_count[256] = {0};

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return 0;
  return d;
}

int sm_count(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev < 0 || dev >= 256) return 148;
  if (g_sm_count[dev] == 0) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
    g_sm_count[dev] = c;
  }
  return g_sm_count[dev];
}

// Opt a kernel into more than 48 KB of dynamic shared memory, once per (kernel, device).
cudaError_t set_smem(const void* fn, int bytes, int dev) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  std::lock_guard<std::mutex> lk(g_mu);
  const auto key = std::make_pair(fn, dev);
  if (g_smem_configured.count(key)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) g_smem_configured.insert(key);
  return e;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

size_t esize(int dtype) { return dtype == TC_F32 ? 4 : 2; }
bool valid_dtype(int dtype) { return dtype == TC_F32 || dtype == TC_F16 || dtype == TC_BF16; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool stride16(int64_t s, int dtype) { return ((s * (int64_t)esize(dtype)) & 15) == 0; }
size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

bool mma_dim(int d) { return d == 64 || d == 128 || d == 256; }
bool gen_dim(int d) { return d == 16 || d == 32 || d == 64 || d == 128; }

// ------------------------------------------------------------------------------- tensor maps
// cuTensorMapEncodeTiled is reached through the runtime's driver entry point, so the library
// does not link libcuda directly.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 4-D map (d, rows, heads, batch) of a 16-bit K or V tensor, box 64 x kTile x 1 x 1, 128-byte
// swizzle, rows past `rows` read as zeros. Strides in elements; extents of 1 get a harmless
// stride. Returns false if the driver rejects the description (the caller then uses the generic
// kernel).
bool encode_kv_map(CUtensorMap* m, const void* base, int dtype, int d, int64_t rows, int64_t heads, int64_t batch,
                   int64_t s_row, int64_t s_head, int64_t s_batch) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (fn == nullptr || base == nullptr) return false;
  if (rows < 1) rows = 1;
  if (heads == 1 || s_head <= 0) s_head = s_row * rows;
  if (batch == 1 || s_batch <= 0) s_batch = s_head * heads;
  const cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)s_row * 2, (cuuint64_t)s_head * 2, (cuuint64_t)s_batch * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)kTile, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, dtype == TC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D 16-bit tensor map (128-byte swizzle, zero fill): dims innermost first, strides in elements of
// dims 1..3, box in elements.
bool encode_map4(CUtensorMap* m, const void* base, int dtype, const int64_t (&dims)[4], const int64_t (&strides)[3],
                 const uint32_t (&box)[4]) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (fn == nullptr || base == nullptr) return false;
  const cuuint64_t gd[4] = {(cuuint64_t)dims[0], (cuuint64_t)dims[1], (cuuint64_t)dims[2], (cuuint64_t)dims[3]};
  const cuuint64_t gs[3] = {(cuuint64_t)strides[0] * 2, (cuuint64_t)strides[1] * 2, (cuuint64_t)strides[2] * 2};
  const cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, dtype == TC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
            const_cast<void*>(base), gd, gs, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ------------------------------------------------------------------------------- decode planning
struct DecodePlan {
  int64_t tps = 1;         // tiles per split
  int64_t max_splits = 1;  // grid.x
};

DecodePlan plan_decode(int batch, int hkv, int64_t max_n, int64_t total_tokens, bool ragged, int splits_req,
                       int ctas_per_sm, int sms) {
  DecodePlan pl;
  const int64_t slots = (int64_t)sms * ctas_per_sm;
  const int64_t tiles = max_n > 0 ? cdiv(max_n, kTile) : 1;
  int64_t tps;
  if (splits_req > 0) {
    int64_t s = splits_req;
    if (s > kMaxSplits) s = kMaxSplits;
    if (s > tiles) s = tiles;
    tps = cdiv(tiles, s);
  } else if (!ragged) {
    // one resident wave: every (sequence, head) gets slots/(batch*hkv) slices of equal length
    int64_t s = slots / ((int64_t)batch * hkv);
    if (s < 1) s = 1;
    if (s > tiles) s = tiles;
    if (s > kMaxSplits) s = kMaxSplits;
    tps = cdiv(tiles, s);
  } else {
    // ragged lengths: many equal-size slices that the block scheduler load-balances
    const int64_t tt = total_tokens > 0 ? total_tokens : (int64_t)batch * max_n;
    const int64_t total_tiles = (int64_t)hkv * (cdiv(tt, kTile) + batch);
    tps = cdiv(total_tiles, 2 * slots);
    if (tps < 1) tps = 1;
    if (tps > 64) tps = 64;
  }
  if (tps < cdiv(tiles, kMaxSplits)) tps = cdiv(tiles, kMaxSplits);
  pl.tps = tps;
  pl.max_splits = cdiv(tiles, tps);
  return pl;
}

struct WsLayout {
  size_t counters = 0, ml = 0, o = 0, total = 0;
};

// Control region at the start of a decode workspace: kCtrWords uint32 per (sequence, head) (start
// ticket, published partials, mergers done), zero between calls.
size_t decode_counter_bytes(int64_t rows) { return round256(sizeof(unsigned int) * tc::kCtrWords * (size_t)rows); }

WsLayout decode_ws_layout(int batch, int hkv, int g, int d, int64_t max_splits) {
  WsLayout w;
  const int64_t rows = (int64_t)batch * hkv;
  w.counters = 0;
  w.ml = decode_counter_bytes(rows);
  w.o = w.ml + round256(sizeof(float) * rows * max_splits * g * 2);
  w.total = w.o + round256(sizeof(float) * rows * max_splits * g * d);
  return w;
}

// Programmatic dependent launch (the kernel's prologue overlaps the previous kernel's tail); set
// TC_PDL=0 in the environment, or call tc_set_pdl(0), to launch plainly (each kernel then starts
// after the previous one ends, so per-kernel device times add up to the step).
std::atomic<int> g_pdl{-1};

bool pdl_enabled() {
  int v = g_pdl.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = std::getenv("TC_PDL");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
    int expect = -1;
    g_pdl.compare_exchange_strong(expect, v, std::memory_order_relaxed);
    v = g_pdl.load(std::memory_order_relaxed);
  }
  return v != 0;
}

template <typename Kern, typename Params>
cudaError_t launch_ex(Kern fn, dim3 grid, dim3 block, int smem, cudaStream_t st, const Params& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

// Any kernel with programmatic dependent launch (as launch_ex), arguments passed through.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, fn, args...);
}

template <typename T, int D, int NG>
cudaError_t launch_mma(const DecodeParams& p, dim3 grid, cudaStream_t st, int dev) {
  auto fn = p.tiles != nullptr ? decode_mma_kernel<T, D, NG, true> : decode_mma_kernel<T, D, NG, false>;
  const int smem = MmaGeom<D>::kSmem;
  const int threads = 32 * (kCWarps + 1);
  cudaError_t e = set_smem(reinterpret_cast<const void*>(fn), smem, dev);
  if (e != cudaSuccess) return e;
  return launch_ex(fn, grid, dim3(threads), smem, st, p);
}

template <typename T, int D>
cudaError_t launch_gen(const DecodeParams& p, dim3 grid, cudaStream_t st, int dev) {
  auto fn = decode_generic_kernel<T, D>;
  const int smem = GenGeom<D>::kSmem;
  cudaError_t e = set_smem(reinterpret_cast<const void*>(fn), smem, dev);
  if (e != cudaSuccess) return e;
  return launch_ex(fn, grid, dim3(32 * kGenWarps), smem, st, p);
}

template <typename T>
cudaError_t dispatch_mma(const DecodeParams& p, int d, dim3 grid, cudaStream_t st, int dev) {
  const bool two = p.g > 8;
  switch (d) {
    case 64: return two ? launch_mma<T, 64, 2>(p, grid, st, dev) : launch_mma<T, 64, 1>(p, grid, st, dev);
    case 128: return two ? launch_mma<T, 128, 2>(p, grid, st, dev) : launch_mma<T, 128, 1>(p, grid, st, dev);
    case 256: return two ? launch_mma<T, 256, 2>(p, grid, st, dev) : launch_mma<T, 256, 1>(p, grid, st, dev);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t dispatch_gen(const DecodeParams& p, int d, dim3 grid, cudaStream_t st, int dev) {
  switch (d) {
    case 16: return launch_gen<T, 16>(p, grid, st, dev);
    case 32: return launch_gen<T, 32>(p, grid, st, dev);
    case 64: return launch_gen<T, 64>(p, grid, st, dev);
    case 128: return launch_gen<T, 128>(p, grid, st, dev);
  }
  return cudaErrorInvalidValue;
}

// Shared by every decode entry point. `kv_aligned` says whether every K/V row start is 16-byte
// aligned (the bulk-copy rule); the 16-bit tensor-core kernel is used only then.
int run_decode(DecodeParams p, int dtype, int d, bool ragged, int64_t max_n, int64_t total_tokens, int splits_req,
               bool kv_aligned, float scale, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (p.hkv < 1 || p.hkv > 65535 || p.g < 1 || p.g > 16 || p.batch < 1 || p.batch > 65535 || max_n < 0)
    return TC_ERR_INVALID;
  if (!(scale == scale) || scale == INFINITY || scale == -INFINITY) return TC_ERR_INVALID;
  if (p.q == nullptr || p.out == nullptr) return TC_ERR_INVALID;
  bool use_mma = dtype != TC_F32 && kv_aligned && mma_dim(d);
  if (use_mma && p.k_ptrs != nullptr) {
    use_mma = p.tm_ragged != nullptr;  // ragged caches need their pre-encoded maps
  } else if (p.tiles != nullptr) {
    if (!use_mma) return TC_ERR_INVALID;  // paged: the caller encoded the pool maps
  } else if (use_mma) {
    use_mma = encode_kv_map(&p.tmk, p.k, dtype, d, max_n, p.hkv, p.batch, p.sk_n, p.sk_h, p.sk_b) &&
              encode_kv_map(&p.tmv, p.v, dtype, d, max_n, p.hkv, p.batch, p.sv_n, p.sv_h, p.sv_b);
  }
  if (!use_mma && !gen_dim(d)) return mma_dim(d) ? TC_ERR_ALIGN : TC_ERR_INVALID;
  // the fused q/k norm + RoPE exists in the tensor-core kernel only, with the fused append
  if (p.nq_w != nullptr && (!use_mma || p.k_app == nullptr || p.tiles != nullptr || p.k_ptrs != nullptr))
    return mma_dim(d) && dtype != TC_F32 ? TC_ERR_ALIGN : TC_ERR_INVALID;
  if (p.k_app != nullptr && !use_mma) {
    // fused append needs the tensor-core kernel: write the row with two strided copies, then decode
    const size_t es = esize(dtype);
    const int64_t row = max_n - 1;
    if (cudaMemcpy2DAsync(const_cast<char*>(static_cast<const char*>(p.k)) + (p.sk_n * row) * es, p.sk_h * es,
                          p.k_app, p.sa_k * es, d * es, p.hkv, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpy2DAsync(const_cast<char*>(static_cast<const char*>(p.v)) + (p.sv_n * row) * es, p.sv_h * es,
                          p.v_app, p.sa_v * es, d * es, p.hkv, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return TC_ERR_CUDA;
    p.k_app = p.v_app = nullptr;
  }
  const int dev = current_device();
  const DecodePlan pl = plan_decode(p.batch, p.hkv, max_n, total_tokens, ragged, splits_req,
                                    use_mma ? kMmaCtasPerSm : kGenCtasPerSm, sm_count(dev));
  const WsLayout w = decode_ws_layout(p.batch, p.hkv, p.g, d, pl.max_splits);
  if (ws == nullptr || ws_bytes < w.total) return TC_ERR_WORKSPACE;
  uint8_t* wb = static_cast<uint8_t*>(ws);
  p.counters = reinterpret_cast<unsigned int*>(wb + w.counters);
  p.ws_ml = reinterpret_cast<float2*>(wb + w.ml);
  p.ws_o = reinterpret_cast<float*>(wb + w.o);
  p.tiles_per_split = (int)pl.tps;
  p.max_splits = (int)pl.max_splits;
  p.c = scale * kLog2e;
  const dim3 grid((unsigned)pl.max_splits, (unsigned)p.hkv, (unsigned)p.batch);
  cudaError_t e;
  if (use_mma) {
    e = dtype == TC_BF16 ? dispatch_mma<__nv_bfloat16>(p, d, grid, st, dev) : dispatch_mma<__half>(p, d, grid, st, dev);
  } else {
    e = dtype == TC_F32    ? dispatch_gen<float>(p, d, grid, st, dev)
        : dtype == TC_BF16 ? dispatch_gen<__nv_bfloat16>(p, d, grid, st, dev)
                           : dispatch_gen<__half>(p, d, grid, st, dev);
  }
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

DecodeParams base_params() {
  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  return p;
}

// ------------------------------------------------------------------------------- splice helpers
int rope_vec(int dtype, int half, const void* const* ptrs, int nptrs, const int64_t* strides, int nstrides) {
  const int vec = dtype == TC_F32 ? 4 : 8;
  if (half % vec != 0) return 1;
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] != nullptr && !aligned16(ptrs[i])) return 1;
  for (int i = 0; i < nstrides; ++i)
    if (!stride16(strides[i], dtype)) return 1;
  return vec;
}

bool load_cos_sin(float* dst, const float* cos_sin, int d) {
  if (cos_sin == nullptr) return false;
  std::memcpy(dst, cos_sin, sizeof(float) * d);
  return true;
}

template <typename T, int VEC>
cudaError_t launch_shift(const ShiftParams& p, int blocks, cudaStream_t st) {
  shift_keys_kernel<T, VEC><<<blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}
template <typename T, int VEC>
cudaError_t launch_splice_copy(const SpliceCopyParams& p, int blocks, cudaStream_t st) {
  splice_copy_kernel<T, VEC><<<blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}
template <typename T, int VEC>
cudaError_t launch_paged_rotate(const PagedRotateParams& p, int blocks, cudaStream_t st) {
  paged_rotate_kernel<T, VEC><<<blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}
template <typename T, int VEC>
cudaError_t launch_paged_write(const PagedWriteParams& p, int blocks, cudaStream_t st) {
  paged_write_kernel<T, VEC><<<blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}
template <typename T, int VEC>
cudaError_t launch_paged_gather(const PagedGatherParams& p, int blocks, cudaStream_t st) {
  paged_gather_kernel<T, VEC><<<blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}
template <typename T, int VEC>
cudaError_t launch_splice_inplace(const SpliceParams& p, int blocks, cudaStream_t st) {
  splice_inplace_kernel<T, VEC><<<blocks, kSpliceThreads, 0, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_splice_bulk(const SpliceParams& p, int blocks, cudaStream_t st, int dev) {
  auto fn = splice_bulk_kernel<T>;
  const int smem = kBulkStages * 2 * kBulkUnitBytes;
  const cudaError_t e = set_smem(reinterpret_cast<const void*>(fn), smem, dev);
  if (e != cudaSuccess) return e;
  fn<<<blocks, kBulkThreads, smem, st>>>(p);
  return cudaGetLastError();
}

// Calls F<T, VEC>(args...) for the runtime (dtype, vec) pair.
#define TC_ROPE_DISPATCH(LAUNCH, dtype, vec, ...)                                                     \
  ((dtype) == TC_F32    ? ((vec) == 4 ? LAUNCH<float, 4>(__VA_ARGS__) : LAUNCH<float, 1>(__VA_ARGS__)) \
   : (dtype) == TC_F16  ? ((vec) == 8 ? LAUNCH<__half, 8>(__VA_ARGS__) : LAUNCH<__half, 1>(__VA_ARGS__)) \
                        : ((vec) == 8 ? LAUNCH<__nv_bfloat16, 8>(__VA_ARGS__)                           \
                                      : LAUNCH<__nv_bfloat16, 1>(__VA_ARGS__)))

int64_t splice_rows_per_unit(int d, int vec) {
  const int cph = (d / 2) / vec;
  const int64_t r = (int64_t)kSpliceThreads * kSpliceTasksPerThread / cph;
  return r < 1 ? 1 : r;
}

int grid_for(int64_t tasks, int threads, int sms, int per_sm) {
  int64_t b = cdiv(tasks, threads);
  const int64_t cap = (int64_t)sms * per_sm;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

// ------------------------------------------------------------------------------- no-allocation decode
// Scratch for tc_decode_attention_noalloc: a fixed array that lives in every GPU's memory for as
// long as the library is loaded, so that entry point never allocates. Host code must not pass the
// symbol itself to a kernel (on the host it only stands in for the device array); it asks the
// runtime for the device address once per device, below.
constexpr size_t kNoAllocScratchBytes = 4u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[256] = {};
unsigned long long g_noalloc_ctx[256] = {};  // id of the context the address above belongs to

// Unique id of the calling thread's current CUDA context (ids are never reused, unlike context
// handles), 0 if there is none or the driver lacks cuCtxGetId. Reached through the runtime's
// driver entry point, like the tensor-map encoder.
unsigned long long current_ctx_id() {
  static PFN_cuCtxGetCurrent_v4000 get_cur = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_cur == nullptr || get_id == nullptr || get_cur(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_noalloc_scratch on the current device. It is looked up (with the device
// current) on the first call for that device, and again whenever the device's context changed
// since (after cudaDeviceReset the module is loaded anew and the array may sit elsewhere).
int noalloc_scratch(void** addr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TC_ERR_CUDA;
  if (dev < 0 || dev >= 256) return TC_ERR_INVALID;
  // 0 before the runtime has made a context current on this thread: the lookup below then runs
  // (and makes it current), and the next call records the id
  const unsigned long long ctx = current_ctx_id();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr || ctx == 0 || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return TC_ERR_CUDA;
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *addr = g_noalloc_addr[dev];
  return TC_OK;
}
}  // namespace

extern "C" {

const char* tc_status_string(int status) {
  switch (status) {
    case TC_OK: return "ok";
    case TC_ERR_INVALID: return "invalid argument (size, shape or pointer outside the supported range)";
    case TC_ERR_ALIGN: return "alignment rule broken (pointer or stride)";
    case TC_ERR_DTYPE: return "unsupported dtype";
    case TC_ERR_WORKSPACE: return "workspace missing or too small";
    case TC_ERR_CUDA: return "CUDA launch or runtime error";
  }
  return "unknown status";
}

int tc_abi_version(void) { return 1; }

int tc_set_pdl(int on) {
  const int prev = pdl_enabled() ? 1 : 0;
  g_pdl.store(on ? 1 : 0, std::memory_order_relaxed);
  return prev;
}

int tc_device_errors(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_errors, sizeof(v)) != cudaSuccess) return -1;
  if (clear) {
    const unsigned int z = 0;
    if (cudaMemcpyToSymbol(g_device_errors, &z, sizeof(z)) != cudaSuccess) return -1;
  }
  return (int)v;
}

size_t tc_decode_attention_workspace_size(int batch, int hkv, int g, int d, int64_t max_n, int64_t total_tokens,
                                          int splits, int dtype) {
  (void)dtype;
  if (batch < 1 || hkv < 1 || g < 1 || d < 1 || max_n < 0) return 0;
  const int sms = sm_count(current_device());
  // the plan differs between the tensor-core and the generic kernel and between uniform and
  // ragged lengths; size for the largest so one figure serves every entry point
  int64_t ms = 1;
  for (int ragged = 0; ragged < 2; ++ragged)
    for (int cps : {kMmaCtasPerSm, kGenCtasPerSm}) {
      const DecodePlan pl = plan_decode(batch, hkv, max_n, total_tokens, ragged != 0, splits, cps, sms);
      if (pl.max_splits > ms) ms = pl.max_splits;
    }
  return decode_ws_layout(batch, hkv, g, d, ms).total;
}

int tc_decode_attention(const void* q, const void* k, const void* v, void* out, int hkv, int g, int d, int64_t n,
                        int64_t q_stride_h, int64_t q_stride_g, int64_t k_stride_h, int64_t k_stride_n,
                        int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h, int64_t out_stride_g,
                        float scale, int splits, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return tc_decode_attention_lse(q, k, v, out, nullptr, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h,
                                 k_stride_n, v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits,
                                 dtype, workspace, workspace_bytes, stream);
}

namespace {
// The fused q/k norm + RoPE of tc_decode_attention_append_rope.
struct NormRope {
  const void* q_weight;
  const void* k_weight;
  const void* cos_t;
  const void* sin_t;
  float eps;
};

int decode_single(const void* q, const void* k, const void* v, void* out, float* lse, bool out_f32, int hkv, int g,
                  int d, int64_t n, int64_t q_stride_h, int64_t q_stride_g, int64_t k_stride_h, int64_t k_stride_n,
                  int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h, int64_t out_stride_g, float scale,
                  int splits, int dtype, void* workspace, size_t workspace_bytes, void* stream,
                  int64_t stable_rows = 0, const void* k_app = nullptr, const void* v_app = nullptr,
                  int64_t sa_k = 0, int64_t sa_v = 0, const NormRope* nr = nullptr) {
  if (n > 0 && (k == nullptr || v == nullptr)) return TC_ERR_INVALID;
  if (stable_rows < 0) return TC_ERR_INVALID;
  DecodeParams p = base_params();
  if (nr != nullptr) {
    p.nq_w = nr->q_weight;
    p.nk_w = nr->k_weight;
    p.rope_cos = nr->cos_t;
    p.rope_sin = nr->sin_t;
    p.norm_eps = nr->eps;
    p.norm_inv_d = 1.0f / (float)d;
  }
  p.stable_rows = stable_rows < n ? stable_rows : n;
  p.k_app = k_app;
  p.v_app = v_app;
  p.sa_k = sa_k;
  p.sa_v = sa_v;
  p.q = q;
  p.out = out;
  p.lse = lse;
  p.out_f32 = out_f32 ? 1 : 0;
  p.lse_b = (int64_t)hkv * g;
  p.k = k;
  p.v = v;
  p.n = n;
  p.sq_h = q_stride_h;
  p.sq_g = q_stride_g;
  p.so_h = out_stride_h;
  p.so_g = out_stride_g;
  p.sk_h = k_stride_h;
  p.sk_n = k_stride_n;
  p.sv_h = v_stride_h;
  p.sv_n = v_stride_n;
  p.hkv = hkv;
  p.g = g;
  p.batch = 1;
  const bool al = aligned16(k) && aligned16(v) && stride16(k_stride_h, dtype) && stride16(k_stride_n, dtype) &&
                  stride16(v_stride_h, dtype) && stride16(v_stride_n, dtype);
  return run_decode(p, dtype, d, false, n, n, splits, al, scale, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream));
}
}  // namespace

int tc_decode_attention_stable(const void* q, const void* k, const void* v, void* out, int hkv, int g, int d,
                               int64_t n, int64_t q_stride_h, int64_t q_stride_g, int64_t k_stride_h,
                               int64_t k_stride_n, int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h,
                               int64_t out_stride_g, float scale, int splits, int dtype, int64_t stable_rows,
                               void* workspace, size_t workspace_bytes, void* stream) {
  return decode_single(q, k, v, out, nullptr, false, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h, k_stride_n,
                       v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype, workspace,
                       workspace_bytes, stream, stable_rows);
}

int tc_decode_attention_append(const void* q, const void* k_new, const void* v_new, void* k, void* v, void* out,
                               int hkv, int g, int d, int64_t n, int64_t q_stride_h, int64_t q_stride_g,
                               int64_t k_new_stride_h, int64_t v_new_stride_h, int64_t k_stride_h,
                               int64_t k_stride_n, int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h,
                               int64_t out_stride_g, float scale, int splits, int dtype, int64_t stable_rows,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 1 || k_new == nullptr || v_new == nullptr) return TC_ERR_INVALID;
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  // the appended row is copied as 16-byte chunks by the tensor-core kernel; a misaligned one makes
  // the host fall back to strided copies (decided in run_decode through the K/V alignment)
  const bool row_al = aligned16(k_new) && aligned16(v_new) && stride16(k_new_stride_h, dtype) &&
                      stride16(v_new_stride_h, dtype);
  if (!row_al) {
    const size_t es = esize(dtype);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpy2DAsync(static_cast<char*>(k) + (k_stride_n * (n - 1)) * es, k_stride_h * es, k_new,
                          k_new_stride_h * es, d * es, hkv, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpy2DAsync(static_cast<char*>(v) + (v_stride_n * (n - 1)) * es, v_stride_h * es, v_new,
                          v_new_stride_h * es, d * es, hkv, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return TC_ERR_CUDA;
    return decode_single(q, k, v, out, nullptr, false, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h,
                         k_stride_n, v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype,
                         workspace, workspace_bytes, stream, 0);
  }
  return decode_single(q, k, v, out, nullptr, false, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h, k_stride_n,
                       v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype, workspace,
                       workspace_bytes, stream, stable_rows, k_new, v_new, k_new_stride_h, v_new_stride_h);
}

int tc_decode_attention_append_rope(const void* q, const void* k_new, const void* v_new, void* k, void* v, void* out,
                                    int hkv, int g, int d, int64_t n, int64_t q_stride_h, int64_t q_stride_g,
                                    int64_t k_new_stride_h, int64_t v_new_stride_h, int64_t k_stride_h,
                                    int64_t k_stride_n, int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h,
                                    int64_t out_stride_g, const void* q_norm_weight, const void* k_norm_weight,
                                    const void* cos_t, const void* sin_t, float eps, float scale, int splits,
                                    int dtype, int64_t stable_rows, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  if (n < 1 || q == nullptr || k_new == nullptr || v_new == nullptr || q_norm_weight == nullptr ||
      k_norm_weight == nullptr || cos_t == nullptr || sin_t == nullptr || !(eps >= 0.f))
    return TC_ERR_INVALID;
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (dtype == TC_F32 || !mma_dim(d)) return TC_ERR_INVALID;
  if (!(aligned16(k_new) && aligned16(v_new) && stride16(k_new_stride_h, dtype) && stride16(v_new_stride_h, dtype)))
    return TC_ERR_ALIGN;
  const NormRope nr{q_norm_weight, k_norm_weight, cos_t, sin_t, eps};
  return decode_single(q, k, v, out, nullptr, false, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h, k_stride_n,
                       v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype, workspace,
                       workspace_bytes, stream, stable_rows, k_new, v_new, k_new_stride_h, v_new_stride_h, &nr);
}

int tc_decode_attention_lse(const void* q, const void* k, const void* v, void* out, float* lse, int hkv, int g,
                            int d, int64_t n, int64_t q_stride_h, int64_t q_stride_g, int64_t k_stride_h,
                            int64_t k_stride_n, int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h,
                            int64_t out_stride_g, float scale, int splits, int dtype, void* workspace,
                            size_t workspace_bytes, void* stream) {
  return decode_single(q, k, v, out, lse, false, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h, k_stride_n,
                       v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype, workspace,
                       workspace_bytes, stream);
}

int tc_decode_attention_partial(const void* q, const void* k, const void* v, float* out_f32, float* lse, int hkv,
                                int g, int d, int64_t n, int64_t q_stride_h, int64_t q_stride_g, int64_t k_stride_h,
                                int64_t k_stride_n, int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h,
                                int64_t out_stride_g, float scale, int splits, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (lse == nullptr) return TC_ERR_INVALID;
  return decode_single(q, k, v, out_f32, lse, true, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h, k_stride_n,
                       v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype, workspace,
                       workspace_bytes, stream);
}

int tc_decode_attention_partial_stable(const void* q, const void* k, const void* v, float* out_f32, float* lse,
                                       int hkv, int g, int d, int64_t n, int64_t q_stride_h, int64_t q_stride_g,
                                       int64_t k_stride_h, int64_t k_stride_n, int64_t v_stride_h,
                                       int64_t v_stride_n, int64_t out_stride_h, int64_t out_stride_g, float scale,
                                       int splits, int dtype, int64_t stable_rows, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if (lse == nullptr) return TC_ERR_INVALID;
  return decode_single(q, k, v, out_f32, lse, true, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h, k_stride_n,
                       v_stride_h, v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype, workspace,
                       workspace_bytes, stream, stable_rows);
}

int tc_decode_attention_batched(const void* q, const void* k, const void* v, void* out, int batch, int hkv, int g,
                                int d, int64_t n, const int32_t* lengths, int64_t q_stride_b, int64_t q_stride_h,
                                int64_t q_stride_g, int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_n,
                                int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_b,
                                int64_t out_stride_h, int64_t out_stride_g, float scale, int splits, int dtype,
                                void* workspace, size_t workspace_bytes, void* stream) {
  if (n > 0 && (k == nullptr || v == nullptr)) return TC_ERR_INVALID;
  DecodeParams p = base_params();
  p.q = q;
  p.out = out;
  p.k = k;
  p.v = v;
  p.lengths = lengths;
  p.n = n;
  p.sq_b = q_stride_b;
  p.sq_h = q_stride_h;
  p.sq_g = q_stride_g;
  p.so_b = out_stride_b;
  p.so_h = out_stride_h;
  p.so_g = out_stride_g;
  p.sk_b = k_stride_b;
  p.sk_h = k_stride_h;
  p.sk_n = k_stride_n;
  p.sv_b = v_stride_b;
  p.sv_h = v_stride_h;
  p.sv_n = v_stride_n;
  p.hkv = hkv;
  p.g = g;
  p.batch = batch;
  const bool al = aligned16(k) && aligned16(v) && stride16(k_stride_b, dtype) && stride16(k_stride_h, dtype) &&
                  stride16(k_stride_n, dtype) && stride16(v_stride_b, dtype) && stride16(v_stride_h, dtype) &&
                  stride16(v_stride_n, dtype);
  return run_decode(p, dtype, d, lengths != nullptr, n, 0, splits, al, scale, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream));
}

int tc_decode_attention_ragged(const void* q, void* out, const void* const* k_ptrs, const void* const* v_ptrs,
                               const int64_t* head_strides, const int32_t* lengths, const void* tensormaps,
                               int batch, int hkv, int g, int d,
                               int64_t max_n, int64_t total_tokens, int64_t kv_stride_n, int64_t q_stride_b,
                               int64_t q_stride_h, int64_t q_stride_g, int64_t out_stride_b, int64_t out_stride_h,
                               int64_t out_stride_g, float scale, int splits, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (k_ptrs == nullptr || v_ptrs == nullptr || head_strides == nullptr || lengths == nullptr) return TC_ERR_INVALID;
  DecodeParams p = base_params();
  p.q = q;
  p.out = out;
  p.k_ptrs = k_ptrs;
  p.v_ptrs = v_ptrs;
  p.head_strides = head_strides;
  p.tm_ragged = static_cast<const CUtensorMap*>(tensormaps);
  if (tensormaps != nullptr && (reinterpret_cast<uintptr_t>(tensormaps) & 63u) != 0) return TC_ERR_ALIGN;
  p.lengths = lengths;
  p.n = max_n;
  p.sq_b = q_stride_b;
  p.sq_h = q_stride_h;
  p.sq_g = q_stride_g;
  p.so_b = out_stride_b;
  p.so_h = out_stride_h;
  p.so_g = out_stride_g;
  p.sk_n = kv_stride_n;
  p.sv_n = kv_stride_n;
  p.hkv = hkv;
  p.g = g;
  p.batch = batch;
  // base alignment and head strides are the caller's contract (device arrays); the token
  // stride is checked here
  const bool al = stride16(kv_stride_n, dtype);
  return run_decode(p, dtype, d, true, max_n, total_tokens, splits, al, scale, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream));
}

size_t tc_ragged_tensormaps_size(int batch) { return batch > 0 ? 2 * (size_t)batch * sizeof(CUtensorMap) : 0; }

int tc_ragged_encode_tensormaps(void* host_out, const void* const* k_ptrs, const void* const* v_ptrs,
                                const int64_t* caps, const int64_t* head_strides, int64_t kv_stride_n, int batch,
                                int hkv, int d, int dtype) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (host_out == nullptr || k_ptrs == nullptr || v_ptrs == nullptr || caps == nullptr || head_strides == nullptr ||
      batch < 1 || hkv < 1 || !mma_dim(d))
    return TC_ERR_INVALID;
  if (!stride16(kv_stride_n, dtype)) return TC_ERR_ALIGN;
  for (int b = 0; b < batch; ++b) {
    if (caps[b] < 0) return TC_ERR_INVALID;
    if (!aligned16(k_ptrs[b]) || !aligned16(v_ptrs[b]) || !stride16(head_strides[b], dtype)) return TC_ERR_ALIGN;
    CUtensorMap mk, mv;
    if (!encode_kv_map(&mk, k_ptrs[b], dtype, d, caps[b], hkv, 1, kv_stride_n, head_strides[b], 0) ||
        !encode_kv_map(&mv, v_ptrs[b], dtype, d, caps[b], hkv, 1, kv_stride_n, head_strides[b], 0))
      return TC_ERR_CUDA;
    std::memcpy(static_cast<uint8_t*>(host_out) + (2 * (size_t)b) * sizeof(CUtensorMap), &mk, sizeof(mk));
    std::memcpy(static_cast<uint8_t*>(host_out) + (2 * (size_t)b + 1) * sizeof(CUtensorMap), &mv, sizeof(mv));
  }
  return TC_OK;
}

int tc_merge_partials(const float* o_parts, const float* lse_parts, void* out, float* lse_out, int parts,
                      int64_t rows, int d, int64_t out_stride_row, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (parts < 1 || rows < 0 || d < 1 || rows > 0x7fffffff || o_parts == nullptr || lse_parts == nullptr ||
      out == nullptr)
    return TC_ERR_INVALID;
  if (rows == 0) return TC_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int threads = d >= 128 ? 128 : ((d + 31) / 32) * 32;
  const dim3 grid((unsigned)rows);
  if (dtype == TC_F32)
    merge_partials_kernel<float><<<grid, threads, 0, st>>>(o_parts, lse_parts, static_cast<float*>(out), lse_out,
                                                          parts, rows, d, out_stride_row);
  else if (dtype == TC_F16)
    merge_partials_kernel<__half><<<grid, threads, 0, st>>>(o_parts, lse_parts, static_cast<__half*>(out), lse_out,
                                                           parts, rows, d, out_stride_row);
  else
    merge_partials_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
        o_parts, lse_parts, static_cast<__nv_bfloat16*>(out), lse_out, parts, rows, d, out_stride_row);
  return cudaGetLastError() == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_shift_keys(const void* keys, void* out, int64_t outer, int64_t n, int d, int64_t in_stride_outer,
                  int64_t in_stride_n, int64_t out_stride_outer, int64_t out_stride_n, const float* cos_sin,
                  int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (d < 2 || d % 2 || d > kMaxRopeDim || outer < 0 || n < 0 || cos_sin == nullptr) return TC_ERR_INVALID;
  if (outer == 0 || n == 0) return TC_OK;
  if (keys == nullptr || out == nullptr) return TC_ERR_INVALID;
  ShiftParams p;
  std::memset(&p, 0, sizeof(p));
  p.in = keys;
  p.out = out;
  p.outer = outer;
  p.n = n;
  p.in_so = in_stride_outer;
  p.in_sn = in_stride_n;
  p.out_so = out_stride_outer;
  p.out_sn = out_stride_n;
  p.d = d;
  load_cos_sin(p.cs, cos_sin, d);
  const void* ptrs[2] = {keys, out};
  const int64_t strides[4] = {in_stride_outer, in_stride_n, out_stride_outer, out_stride_n};
  const int vec = rope_vec(dtype, d / 2, ptrs, 2, strides, 4);
  const int64_t tasks = outer * n * ((d / 2) / vec);
  const int blocks = grid_for(tasks, 256, sm_count(current_device()), 16);
  const cudaError_t e = TC_ROPE_DISPATCH(launch_shift, dtype, vec, p, blocks, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

// ------------------------------------------------------------------------------- paged cache
int tc_decode_attention_paged(const void* q, const void* k_pool, const void* v_pool, void* out, int hkv, int g,
                              int d, int64_t page_rows, int64_t num_pages, int64_t pool_stride_page,
                              int64_t pool_stride_h, int64_t pool_stride_row, const int32_t* tiles, int64_t n_tiles,
                              int64_t n_tokens, const void* k_new, const void* v_new, int64_t k_new_stride_h,
                              int64_t v_new_stride_h, int64_t q_stride_h, int64_t q_stride_g, int64_t out_stride_h,
                              int64_t out_stride_g, float scale, int splits, int dtype, int64_t stable_tiles,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (stable_tiles < 0) return TC_ERR_INVALID;
  if (!mma_dim(d) || hkv < 1 || g < 1 || page_rows < kTile || page_rows > (1 << 30) || num_pages < 1 ||
      num_pages > (1 << 30) || n_tiles < 0 || n_tiles > ((int64_t)1 << 31) / kTile || n_tokens < 0)
    return TC_ERR_INVALID;
  if (k_pool == nullptr || v_pool == nullptr || (n_tiles > 0 && tiles == nullptr)) return TC_ERR_INVALID;
  if ((k_new == nullptr) != (v_new == nullptr)) return TC_ERR_INVALID;
  if (!aligned16(k_pool) || !aligned16(v_pool) || !stride16(pool_stride_page, dtype) ||
      !stride16(pool_stride_h, dtype) || !stride16(pool_stride_row, dtype))
    return TC_ERR_ALIGN;
  if (k_new != nullptr && (!aligned16(k_new) || !aligned16(v_new) || !stride16(k_new_stride_h, dtype) ||
                           !stride16(v_new_stride_h, dtype)))
    return TC_ERR_ALIGN;
  DecodeParams p = base_params();
  if (!encode_kv_map(&p.tmk, k_pool, dtype, d, page_rows, hkv, num_pages, pool_stride_row, pool_stride_h,
                     pool_stride_page) ||
      !encode_kv_map(&p.tmv, v_pool, dtype, d, page_rows, hkv, num_pages, pool_stride_row, pool_stride_h,
                     pool_stride_page))
    return TC_ERR_INVALID;
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  p.stable_tiles = stable_tiles < n_tiles ? stable_tiles : n_tiles;
  p.q = q;
  p.out = out;
  p.lse_b = (int64_t)hkv * g;
  p.k = k_pool;
  p.v = v_pool;
  p.n = n_tokens;
  p.sq_h = q_stride_h;
  p.sq_g = q_stride_g;
  p.so_h = out_stride_h;
  p.so_g = out_stride_g;
  p.sk_b = pool_stride_page;
  p.sk_h = pool_stride_h;
  p.sk_n = pool_stride_row;
  p.sv_b = pool_stride_page;
  p.sv_h = pool_stride_h;
  p.sv_n = pool_stride_row;
  p.hkv = hkv;
  p.g = g;
  p.batch = 1;
  p.k_app = n_tiles > 0 ? k_new : nullptr;
  p.v_app = n_tiles > 0 ? v_new : nullptr;
  p.sa_k = k_new_stride_h;
  p.sa_v = v_new_stride_h;
  return run_decode(p, dtype, d, false, n_tiles * kTile, n_tiles * kTile, splits, true, scale, workspace,
                    workspace_bytes, static_cast<cudaStream_t>(stream));
}

int tc_paged_rotate_keys(void* const* k_pools, int layers, int hkv, int d, int64_t page_rows, int64_t num_pages,
                         int64_t pool_stride_page, int64_t pool_stride_h, int64_t pool_stride_row,
                         const int32_t* tiles, int64_t n_tiles, const float* cos_sin, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (layers < 1 || layers > kMaxLayers || hkv < 1 || d < 2 || d % 2 || d > kMaxRopeDim || page_rows < 1 ||
      num_pages < 1 || n_tiles < 0 || k_pools == nullptr || cos_sin == nullptr)
    return TC_ERR_INVALID;
  if (n_tiles == 0) return TC_OK;
  if (tiles == nullptr) return TC_ERR_INVALID;
  PagedRotateParams p;
  std::memset(&p, 0, sizeof(p));
  for (int l = 0; l < layers; ++l) {
    if (k_pools[l] == nullptr) return TC_ERR_INVALID;
    p.kp[l] = k_pools[l];
  }
  p.layers = layers;
  p.hkv = hkv;
  p.d = d;
  p.page_rows = page_rows;
  p.num_pages = num_pages;
  p.s_page = pool_stride_page;
  p.s_h = pool_stride_h;
  p.s_row = pool_stride_row;
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  load_cos_sin(p.cs, cos_sin, d);
  const int64_t strides[3] = {pool_stride_page, pool_stride_h, pool_stride_row};
  const int vec = rope_vec(dtype, d / 2, k_pools, layers, strides, 3);
  const int64_t tasks = (int64_t)layers * n_tiles * hkv * kPagedTileRows * ((d / 2) / vec);
  const int blocks = grid_for(tasks, 256, sm_count(current_device()), 8);
  const cudaError_t e =
      TC_ROPE_DISPATCH(launch_paged_rotate, dtype, vec, p, blocks, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_paged_write(const void* k_src, const void* v_src, void* k_pool, void* v_pool, int hkv, int d, int64_t t,
                   int64_t src_stride_h, int64_t src_stride_t, int64_t vsrc_stride_h, int64_t vsrc_stride_t,
                   int64_t page_rows, int64_t num_pages, int64_t pool_stride_page, int64_t pool_stride_h,
                   int64_t pool_stride_row, const int32_t* slots, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (hkv < 1 || d < 1 || t < 0 || page_rows < 1 || num_pages < 1) return TC_ERR_INVALID;
  if (t == 0) return TC_OK;
  if (k_src == nullptr || v_src == nullptr || k_pool == nullptr || v_pool == nullptr || slots == nullptr)
    return TC_ERR_INVALID;
  PagedWriteParams p;
  std::memset(&p, 0, sizeof(p));
  p.k_src = k_src;
  p.v_src = v_src;
  p.kp = k_pool;
  p.vp = v_pool;
  p.hkv = hkv;
  p.d = d;
  p.t = t;
  p.src_sh = src_stride_h;
  p.src_st = src_stride_t;
  p.vsrc_sh = vsrc_stride_h;
  p.vsrc_st = vsrc_stride_t;
  p.page_rows = page_rows;
  p.num_pages = num_pages;
  p.s_page = pool_stride_page;
  p.s_h = pool_stride_h;
  p.s_row = pool_stride_row;
  p.slots = slots;
  const void* ptrs[4] = {k_src, v_src, k_pool, v_pool};
  const int64_t strides[7] = {src_stride_h, src_stride_t, vsrc_stride_h, vsrc_stride_t,
                              pool_stride_page, pool_stride_h, pool_stride_row};
  // whole rows move as 16-byte chunks when d allows it (rope_vec checks d/2; check d itself here)
  int vec = rope_vec(dtype, d / 2, ptrs, 4, strides, 7);
  if (d % vec != 0) vec = 1;
  const int64_t tasks = 2 * t * hkv * (d / vec);
  const int blocks = grid_for(tasks, 256, sm_count(current_device()), 8);
  const cudaError_t e =
      TC_ROPE_DISPATCH(launch_paged_write, dtype, vec, p, blocks, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_paged_gather(const void* k_pool, const void* v_pool, void* k_out, void* v_out, int hkv, int d, int64_t n,
                    int64_t out_stride_h, int64_t out_stride_n, int64_t page_rows, int64_t num_pages,
                    int64_t pool_stride_page, int64_t pool_stride_h, int64_t pool_stride_row, const int32_t* tiles,
                    int64_t n_tiles, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (hkv < 1 || d < 1 || n < 0 || n_tiles < 0 || page_rows < 1 || num_pages < 1) return TC_ERR_INVALID;
  if (n == 0 || n_tiles == 0) return TC_OK;
  if (k_pool == nullptr || v_pool == nullptr || k_out == nullptr || v_out == nullptr || tiles == nullptr)
    return TC_ERR_INVALID;
  PagedGatherParams p;
  std::memset(&p, 0, sizeof(p));
  p.kp = k_pool;
  p.vp = v_pool;
  p.k_out = k_out;
  p.v_out = v_out;
  p.hkv = hkv;
  p.d = d;
  p.n = n;
  p.out_sh = out_stride_h;
  p.out_sn = out_stride_n;
  p.page_rows = page_rows;
  p.num_pages = num_pages;
  p.s_page = pool_stride_page;
  p.s_h = pool_stride_h;
  p.s_row = pool_stride_row;
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  const void* ptrs[4] = {k_pool, v_pool, k_out, v_out};
  const int64_t strides[5] = {out_stride_h, out_stride_n, pool_stride_page, pool_stride_h, pool_stride_row};
  int vec = rope_vec(dtype, d / 2, ptrs, 4, strides, 5);
  if (d % vec != 0) vec = 1;
  const int64_t tasks = 2 * n_tiles * hkv * kPagedTileRows * (d / vec);
  const int blocks = grid_for(tasks, 256, sm_count(current_device()), 8);
  const cudaError_t e =
      TC_ROPE_DISPATCH(launch_paged_gather, dtype, vec, p, blocks, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

size_t tc_splice_workspace_size(int layers, int hkv, int64_t c) {
  if (layers < 1 || hkv < 1 || c < 0) return 0;
  // a unit covers at least kSpliceThreads*kSpliceTasksPerThread / (kMaxRopeDim/2) = 2 rows (the
  // scalar path on the widest rows), which bounds the number of per-unit flags from above
  const int64_t worst = c > 0 ? cdiv(c, 2) : 0;
  return 16 + sizeof(unsigned int) * (size_t)layers * hkv * (size_t)worst;
}

int tc_splice_inplace(void* const* kbufs, void* const* vbufs, int layers, int hkv, int d, int64_t cap, int64_t a,
                      int64_t c0, int64_t c, int64_t stride_h, int64_t stride_n, const float* cos_sin, int dtype,
                      void* workspace, size_t workspace_bytes, uint32_t epoch, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (layers < 1 || layers > kMaxLayers || hkv < 1 || d < 2 || d % 2 || d > kMaxRopeDim || a < 0 || c < 0 ||
      c0 < a || c0 + c > cap || kbufs == nullptr || vbufs == nullptr)
    return TC_ERR_INVALID;
  if (c == 0 || c0 == a) return TC_OK;  // nothing moves (kv.py:85-87 clones C onto itself)
  if (cos_sin == nullptr || epoch == 0) return TC_ERR_INVALID;
  for (int l = 0; l < layers; ++l)
    if (kbufs[l] == nullptr || vbufs[l] == nullptr) return TC_ERR_INVALID;
  SpliceParams p;
  std::memset(&p, 0, sizeof(p));
  for (int l = 0; l < layers; ++l) {
    p.kb[l] = kbufs[l];
    p.vb[l] = vbufs[l];
  }
  const int64_t strides[2] = {stride_h, stride_n};
  int vec = rope_vec(dtype, d / 2, const_cast<const void* const*>(kbufs), layers, strides, 2);
  if (vec > 1 && rope_vec(dtype, d / 2, const_cast<const void* const*>(vbufs), layers, strides, 2) == 1) vec = 1;
  p.layers = layers;
  p.hkv = hkv;
  p.d = d;
  p.rows_per_unit = (int)splice_rows_per_unit(d, vec);
  p.a = a;
  p.c0 = c0;
  p.c = c;
  p.gap = c0 - a;
  p.nchunks = cdiv(c, p.rows_per_unit);
  p.sh = stride_h;
  p.sn = stride_n;
  p.epoch = epoch;
  load_cos_sin(p.cs, cos_sin, d);
  const size_t need = 16 + sizeof(unsigned int) * (size_t)layers * hkv * (size_t)p.nchunks;
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) return TC_ERR_WORKSPACE;
  p.ws = static_cast<SpliceWs*>(workspace);
  const int64_t units = (int64_t)layers * hkv * p.nchunks;
  if (units >= (int64_t)0xffffffffLL) return TC_ERR_INVALID;  // unit tickets are 32-bit
  const int dev = current_device();
  const int sms = sm_count(dev);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (vec > 1 && stride_n == d) {
    // contiguous, aligned rows: a unit is one 16 KB block of K rows and one of V rows
    int64_t blocks = (int64_t)sms * kBulkCtasPerSm;
    if (blocks > units) blocks = units;
    e = dtype == TC_F32   ? launch_splice_bulk<float>(p, (int)blocks, st, dev)
        : dtype == TC_F16 ? launch_splice_bulk<__half>(p, (int)blocks, st, dev)
                          : launch_splice_bulk<__nv_bfloat16>(p, (int)blocks, st, dev);
  } else {
    int64_t blocks = (int64_t)sms * 6;
    if (blocks > units) blocks = units;
    e = TC_ROPE_DISPATCH(launch_splice_inplace, dtype, vec, p, (int)blocks, st);
  }
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_splice_copy(const void* k_in, const void* v_in, void* k_out, void* v_out, int hkv, int d, int64_t a,
                   int64_t c0, int64_t c, int64_t in_stride_h, int64_t in_stride_n, int64_t out_stride_h,
                   int64_t out_stride_n, const float* cos_sin, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (hkv < 1 || d < 2 || d % 2 || d > kMaxRopeDim || a < 0 || c < 0 || c0 < a) return TC_ERR_INVALID;
  if (a + c == 0) return TC_OK;
  if (k_in == nullptr || v_in == nullptr || k_out == nullptr || v_out == nullptr) return TC_ERR_INVALID;
  const bool rotate = c > 0 && c0 != a;
  if (rotate && cos_sin == nullptr) return TC_ERR_INVALID;
  SpliceCopyParams p;
  std::memset(&p, 0, sizeof(p));
  p.kin = k_in;
  p.vin = v_in;
  p.kout = k_out;
  p.vout = v_out;
  p.hkv = hkv;
  p.a = a;
  p.c0 = c0;
  p.c = c;
  p.in_sh = in_stride_h;
  p.in_sn = in_stride_n;
  p.out_sh = out_stride_h;
  p.out_sn = out_stride_n;
  p.d = d;
  p.rotate = rotate ? 1 : 0;
  if (rotate) load_cos_sin(p.cs, cos_sin, d);
  const void* ptrs[4] = {k_in, v_in, k_out, v_out};
  const int64_t strides[4] = {in_stride_h, in_stride_n, out_stride_h, out_stride_n};
  const int vec = rope_vec(dtype, d / 2, ptrs, 4, strides, 4);
  const int64_t tasks = (int64_t)hkv * (a + c) * ((d / 2) / vec);
  const int blocks = grid_for(tasks, 256, sm_count(current_device()), 16);
  const cudaError_t e =
      TC_ROPE_DISPATCH(launch_splice_copy, dtype, vec, p, blocks, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_decode_attention_noalloc(const void* q, const void* k, const void* v, void* out, int hkv, int g, int d,
                                int64_t n, int64_t q_stride_h, int64_t q_stride_g, int64_t k_stride_h,
                                int64_t k_stride_n, int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_h,
                                int64_t out_stride_g, float scale, int splits, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  const size_t need = tc_decode_attention_workspace_size(1, hkv, g, d, n, n, splits, dtype);
  if (need == 0) return TC_ERR_INVALID;
  if (need > kNoAllocScratchBytes) return TC_ERR_WORKSPACE;  // the problem is larger than the fixed array
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != TC_OK) return rc;
  // the control words at the start of the workspace must be zero; they are left zero by every
  // finished call, but an earlier call that failed part-way could have left them set
  if (cudaMemsetAsync(scratch, 0, decode_counter_bytes(hkv), static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return TC_ERR_CUDA;
  return tc_decode_attention(q, k, v, out, hkv, g, d, n, q_stride_h, q_stride_g, k_stride_h, k_stride_n, v_stride_h,
                             v_stride_n, out_stride_h, out_stride_g, scale, splits, dtype, scratch,
                             kNoAllocScratchBytes, stream);
}

size_t tc_split_workspace_size(int64_t n_cached) {
  if (n_cached < 0) return 0;
  return sizeof(SplitWs) + 2 * sizeof(int64_t) * (size_t)(n_cached > 0 ? n_cached : 1);  // candidates + slots
}

int tc_split(const int32_t* cached, int64_t n_cached, const int32_t* new_tokens, int64_t n_new, int min_suffix,
             int suffix, int64_t* out3, void* workspace, size_t workspace_bytes, void* stream) {
  if (n_new < 1 || n_cached < 0 || n_cached >= (int64_t)0xffffffffLL || min_suffix < 1 || out3 == nullptr ||
      new_tokens == nullptr || (n_cached > 0 && cached == nullptr))
    return TC_ERR_INVALID;
  if (workspace == nullptr || workspace_bytes < tc_split_workspace_size(n_cached) ||
      reinterpret_cast<uintptr_t>(workspace) % 8 != 0)
    return TC_ERR_WORKSPACE;
  SplitParams p;
  p.cached = cached;
  p.fresh = new_tokens;
  p.n_cached = n_cached;
  p.n_new = n_new;
  p.min_suffix = min_suffix;
  p.suffix = suffix ? 1 : 0;
  p.cap = n_cached > 0 ? n_cached : 1;
  p.ws = static_cast<SplitWs*>(workspace);
  p.out = out3;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = sm_count(current_device());
  const int64_t m = n_cached < n_new ? n_cached : n_new;
  split_init_kernel<<<1, 32, 0, st>>>(p);
  split_lcp_kernel<<<grid_for(m > 0 ? m : 1, kSplitThreads, sms, 8), kSplitThreads, 0, st>>>(p);
  split_window_kernel<<<grid_for(n_cached > 0 ? n_cached : 1, kSplitThreads, sms, 8), kSplitThreads, 0, st>>>(p);
  split_extend_kernel<<<sms * 4, kExtendThreads, 0, st>>>(p);
  split_best_kernel<<<sms, kSplitThreads, 0, st>>>(p);
  split_finish_kernel<<<1, 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

// KV splits of the prefill kernel (one CTA per SM): none when (query blocks x KV heads) already make
// two waves; else the smallest count (<= 16, >= 8 tiles per split) whose CTAs fill their waves of
// SMs at least 95 %, else the count with the fullest waves.
int prefill_splits(int hkv, int lq, int lk, int sms) {
  const int64_t base = (int64_t)((lq + kPfQ * kPfTiles - 1) / (kPfQ * kPfTiles)) * hkv;
  if (base >= 2 * (int64_t)sms) return 1;
  const int64_t tiles = ((int64_t)lk + kPfKeys - 1) / kPfKeys;
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= 16 && (s == 1 || tiles / s >= 8); ++s) {
    const int64_t ctas = base * s;
    const int64_t waves = (ctas + sms - 1) / sms;
    const double eff = (double)ctas / (double)(waves * sms);
    if (eff >= 0.95) return s;
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

size_t prefill_ws_bytes(int hq, int lq, int splits) {
  if (splits <= 1) return 0;
  return sizeof(float) * (size_t)splits * (size_t)lq * (size_t)hq * (128 + 1);
}

int tc_prefill_splits(int hkv, int lq, int lk) {
  if (hkv < 1 || lq < 1 || lk < lq) return 0;
  return prefill_splits(hkv, lq, lk, sm_count(current_device()));
}

size_t tc_prefill_workspace_size(int hq, int hkv, int lq, int lk, int splits) {
  if (hkv < 1 || lq < 1 || lk < lq) return 0;
  const int s = splits > 0 ? (splits > 16 ? 16 : splits) : prefill_splits(hkv, lq, lk, sm_count(current_device()));
  return prefill_ws_bytes(hq, lq, s);
}

}  // extern "C"

namespace {
template <typename T, bool kPaged>
cudaError_t launch_prefill_t(const PrefillParams& p, dim3 grid, int dev, cudaStream_t s) {
  const cudaError_t e = set_smem(reinterpret_cast<const void*>(prefill_kernel<T, kPaged>), kPfSmem, dev);
  if (e != cudaSuccess) return e;
  prefill_kernel<T, kPaged><<<grid, kPfThreads, kPfSmem, s>>>(p);
  return cudaGetLastError();
}

// One prefill launch (grid: query blocks x KV heads x splits) and, with splits, the LSE merge.
int launch_prefill(const PrefillParams& p, int lq, int hkv, int ns, int64_t rows, void* out, int dtype, int dev,
                   void* stream, bool paged = false) {
  const dim3 grid((unsigned)((lq + kPfQ * kPfTiles - 1) / (kPfQ * kPfTiles)), (unsigned)hkv, (unsigned)ns);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == TC_BF16)
    e = paged ? launch_prefill_t<__nv_bfloat16, true>(p, grid, dev, s) : launch_prefill_t<__nv_bfloat16, false>(p, grid, dev, s);
  else
    e = paged ? launch_prefill_t<__half, true>(p, grid, dev, s) : launch_prefill_t<__half, false>(p, grid, dev, s);
  if (e != cudaSuccess) return TC_ERR_CUDA;
  if (ns > 1) return tc_merge_partials(p.o_part, p.lse_part, out, nullptr, ns, rows, 128, 128, dtype, stream);
  return TC_OK;
}
}  // namespace

extern "C" {

int tc_prefill_attention(const void* q, const void* k, const void* v, void* out, int hq, int hkv, int lq, int lk,
                         int d, int64_t q_stride_h, int64_t q_stride_p, int64_t k_stride_h, int64_t k_stride_n,
                         int64_t v_stride_h, int64_t v_stride_n, int64_t out_stride_p, int64_t out_stride_h,
                         float scale, int splits, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (d != 128 || hkv < 1 || hkv > 65535 || hq != kPfGroup * hkv || lq < 1 || lk < lq || q == nullptr ||
      k == nullptr || v == nullptr || out == nullptr || splits < 0)
    return TC_ERR_INVALID;
  if (!(scale == scale) || scale == INFINITY || scale == -INFINITY) return TC_ERR_INVALID;
  const int64_t st[8] = {q_stride_h, q_stride_p, k_stride_h, k_stride_n, v_stride_h, v_stride_n, out_stride_p,
                         out_stride_h};
  for (int64_t x : st)
    if (!stride16(x, dtype)) return TC_ERR_ALIGN;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return TC_ERR_ALIGN;
  const int dev = current_device();
  int ns = splits > 0 ? (splits > 16 ? 16 : splits) : prefill_splits(hkv, lq, lk, sm_count(dev));
  // split partials are merged into rows of d contiguous elements: needs the [lq, hq, d] layout
  if (ns > 1 && !(out_stride_h == 128 && out_stride_p == (int64_t)hq * 128)) ns = 1;
  const size_t need = prefill_ws_bytes(hq, lq, ns);
  if (ns > 1 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) return TC_ERR_WORKSPACE;
  PrefillParams p;
  std::memset(&p, 0, sizeof(p));
  const int64_t qd[4] = {128, lq, hq, 1}, qs[3] = {q_stride_p, q_stride_h, q_stride_h * hq};
  const int64_t kd[4] = {128, lk, hkv, 1}, ks[3] = {k_stride_n, k_stride_h, k_stride_h * hkv};
  const int64_t vs[3] = {v_stride_n, v_stride_h, v_stride_h * hkv};
  const uint32_t qbox[4] = {64, (uint32_t)kPfQ, (uint32_t)kPfGroup, 1}, kbox[4] = {64, (uint32_t)kPfKeys, 1, 1};
  if (!encode_map4(&p.tmq, q, dtype, qd, qs, qbox) || !encode_map4(&p.tmk, k, dtype, kd, ks, kbox) ||
      !encode_map4(&p.tmv, v, dtype, kd, vs, kbox))
    return TC_ERR_INVALID;
  p.out = out;
  p.so_p = out_stride_p;
  p.so_h = out_stride_h;
  p.lq = lq;
  p.lk = lk;
  p.hq = hq;
  p.hkv = hkv;
  p.c = scale * kLog2e;
  p.nsplit = ns;
  const int64_t rows = (int64_t)lq * hq;
  if (ns > 1) {
    p.o_part = static_cast<float*>(workspace);
    p.lse_part = p.o_part + (size_t)ns * rows * 128;
  }
  return launch_prefill(p, lq, hkv, ns, rows, out, dtype, dev, stream);
}

int tc_prefill_attention_paged(const void* q, const void* k_pool, const void* v_pool, void* out, int hq, int hkv,
                               int lq, int lk, int d, int64_t page_rows, int64_t num_pages, int64_t pool_stride_page,
                               int64_t pool_stride_h, int64_t pool_stride_row, const int32_t* ktab, int64_t n_sub,
                               const int32_t* qb_tiles, int64_t q_stride_h, int64_t q_stride_p,
                               int64_t out_stride_p, int64_t out_stride_h, float scale, int splits, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (d != 128 || hkv < 1 || hkv > 65535 || hq != kPfGroup * hkv || lq < 1 || lk < lq || q == nullptr ||
      k_pool == nullptr || v_pool == nullptr || out == nullptr || ktab == nullptr || qb_tiles == nullptr ||
      splits < 0 || n_sub < 1 || n_sub > (1 << 28) || page_rows < kTile || page_rows > (1 << 30) ||
      num_pages < 1 || num_pages >= (1 << 30))
    return TC_ERR_INVALID;
  if (!(scale == scale) || scale == INFINITY || scale == -INFINITY) return TC_ERR_INVALID;
  const int64_t st[7] = {q_stride_h, q_stride_p, out_stride_p, out_stride_h, pool_stride_page, pool_stride_h,
                         pool_stride_row};
  for (int64_t x : st)
    if (!stride16(x, dtype)) return TC_ERR_ALIGN;
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out) || !aligned16(ktab))
    return TC_ERR_ALIGN;
  const int dev = current_device();
  const int lk_tiles = (int)((n_sub + 3) / 4) * kPfKeys;  // key slots the tiles hold (planning only)
  int ns = splits > 0 ? (splits > 16 ? 16 : splits) : prefill_splits(hkv, lq, lk_tiles, sm_count(dev));
  if (ns > 1 && !(out_stride_h == 128 && out_stride_p == (int64_t)hq * 128)) ns = 1;
  const size_t need = prefill_ws_bytes(hq, lq, ns);
  if (ns > 1 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) return TC_ERR_WORKSPACE;
  PrefillParams p;
  std::memset(&p, 0, sizeof(p));
  const int64_t qd[4] = {128, lq, hq, 1}, qs[3] = {q_stride_p, q_stride_h, q_stride_h * hq};
  const uint32_t qbox[4] = {64, (uint32_t)kPfQ, (uint32_t)kPfGroup, 1};
  if (!encode_map4(&p.tmq, q, dtype, qd, qs, qbox) ||
      !encode_kv_map(&p.tmk, k_pool, dtype, d, page_rows, hkv, num_pages, pool_stride_row, pool_stride_h,
                     pool_stride_page) ||
      !encode_kv_map(&p.tmv, v_pool, dtype, d, page_rows, hkv, num_pages, pool_stride_row, pool_stride_h,
                     pool_stride_page))
    return TC_ERR_INVALID;
  p.ktab = reinterpret_cast<const int4*>(ktab);
  p.n_sub = (int)n_sub;
  p.oob_page = (int)num_pages;
  p.qb_tiles = qb_tiles;
  p.out = out;
  p.so_p = out_stride_p;
  p.so_h = out_stride_h;
  p.lq = lq;
  p.lk = lk;
  p.hq = hq;
  p.hkv = hkv;
  p.c = scale * kLog2e;
  p.nsplit = ns;
  const int64_t rows = (int64_t)lq * hq;
  if (ns > 1) {
    p.o_part = static_cast<float*>(workspace);
    p.lse_part = p.o_part + (size_t)ns * rows * 128;
  }
  return launch_prefill(p, lq, hkv, ns, rows, out, dtype, dev, stream, true);
}

}  // extern "C"

// ---------------------------------------------------------------- per-token layer ops (tensor-parallel step)
namespace {
template <typename T>
int launch_layer_op_t(int op, void* a, void* b, const void* c, const void* d0, const void* e, const void* f,
                      int64_t rows, int n0, int n1, int d, float eps, cudaStream_t st) {
  const bool vec = op == 0 && sizeof(T) == 2 && n0 % 8 == 0 && n0 / 8 <= kNormThreads * 4 &&
                   ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                     reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(d0)) & 15) == 0;
  cudaError_t err;
  if (op == 0) {
    if (vec)
      err = launch_pdl(add_rmsnorm_vec_kernel<T, 4>, dim3((unsigned)rows), dim3(kNormThreads), 0, st,
                       static_cast<T*>(a), static_cast<const T*>(c), static_cast<const T*>(d0), static_cast<T*>(b),
                       n0, 1.0f / (float)n0, eps);
    else
      err = launch_pdl(add_rmsnorm_kernel<T>, dim3((unsigned)rows), dim3(kNormThreads), 0, st, static_cast<T*>(a),
                       static_cast<const T*>(c), static_cast<const T*>(d0), static_cast<T*>(b), n0,
                       1.0f / (float)n0, eps);
  } else if (op == 1) {
    const int threads = ((d + 31) / 32) * 32;
    err = launch_pdl(qk_norm_rope_kernel<T>, dim3((unsigned)(n0 + n1)), dim3(threads), d * sizeof(float), st,
                     static_cast<T*>(a), static_cast<T*>(b), static_cast<const T*>(c), static_cast<const T*>(d0),
                     static_cast<const T*>(e), static_cast<const T*>(f), n0, d, 1.0f / (float)d, eps);
  } else {
    const int64_t total = rows * n0;
    const int64_t blocks = (total + kNormThreads - 1) / kNormThreads;
    err = launch_pdl(silu_mul_kernel<T>, dim3((unsigned)(blocks < 4096 ? blocks : 4096)), dim3(kNormThreads), 0, st,
                     static_cast<const T*>(c), static_cast<T*>(a), rows, n0);
  }
  return err == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int launch_layer_op(int dtype, int op, void* a, void* b, const void* c, const void* d0, const void* e, const void* f,
                    int64_t rows, int n0, int n1, int d, float eps, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TC_BF16) return launch_layer_op_t<__nv_bfloat16>(op, a, b, c, d0, e, f, rows, n0, n1, d, eps, st);
  if (dtype == TC_F16) return launch_layer_op_t<__half>(op, a, b, c, d0, e, f, rows, n0, n1, d, eps, st);
  return launch_layer_op_t<float>(op, a, b, c, d0, e, f, rows, n0, n1, d, eps, st);
}
}  // namespace

extern "C" {

int tc_add_rmsnorm(void* h, const void* delta, const void* weight, void* out, int64_t rows, int hidden, float eps,
                   int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (rows < 0 || rows > 0x7fffffff || hidden < 1 || !(eps >= 0.f)) return TC_ERR_INVALID;
  if (rows == 0) return TC_OK;
  if (h == nullptr || weight == nullptr || out == nullptr) return TC_ERR_INVALID;
  return launch_layer_op(dtype, 0, h, out, delta, weight, nullptr, nullptr, rows, hidden, 0, 0, eps, stream);
}

int tc_qk_norm_rope(void* q, void* k, const void* q_weight, const void* k_weight, const void* cos_t,
                    const void* sin_t, int q_heads, int k_heads, int d, float eps, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (q_heads < 0 || k_heads < 0 || d < 2 || d % 2 || d > 1024 || !(eps >= 0.f)) return TC_ERR_INVALID;
  if (q_heads + k_heads == 0) return TC_OK;
  if ((q_heads && (q == nullptr || q_weight == nullptr)) || (k_heads && (k == nullptr || k_weight == nullptr)) ||
      cos_t == nullptr || sin_t == nullptr)
    return TC_ERR_INVALID;
  return launch_layer_op(dtype, 1, q, k, q_weight, k_weight, cos_t, sin_t, 1, q_heads, k_heads, d, eps, stream);
}

}  // extern "C"

namespace {
template <typename T, bool SW, int RPW>
cudaError_t launch_gemv_r(unsigned grid, size_t smem, cudaStream_t st, const void* x, const void* w, void* out,
                          int64_t n, int k) {
  return launch_pdl(gemv_kernel<T, SW, RPW>, dim3(grid), dim3(kGemvWarps * 32), smem, st, static_cast<const T*>(x),
                    static_cast<const T*>(w), static_cast<T*>(out), n, k);
}

template <typename T>
cudaError_t launch_gemv_t(int rpw, bool swiglu, unsigned grid, size_t smem, cudaStream_t st, const void* x,
                          const void* w, void* out, int64_t n, int k) {
  if (swiglu) {
    if (rpw == 4) return launch_gemv_r<T, true, 4>(grid, smem, st, x, w, out, n, k);
    if (rpw == 2) return launch_gemv_r<T, true, 2>(grid, smem, st, x, w, out, n, k);
    return launch_gemv_r<T, true, 1>(grid, smem, st, x, w, out, n, k);
  }
  if (rpw == 4) return launch_gemv_r<T, false, 4>(grid, smem, st, x, w, out, n, k);
  if (rpw == 2) return launch_gemv_r<T, false, 2>(grid, smem, st, x, w, out, n, k);
  return launch_gemv_r<T, false, 1>(grid, smem, st, x, w, out, n, k);
}

// Input length from which the projections split K over the warps of a CTA; TC_GEMV_SPLITK_MIN
// overrides the default (a measurement switch).
int splitk_min() {
  static const int v = [] {
    const char* e = std::getenv("TC_GEMV_SPLITK_MIN");
    return e != nullptr ? std::atoi(e) : kSplitKMin;
  }();
  return v;
}

// The streaming GEMV (gemv_stream_kernel) unless TC_GEMV_STREAM=0 (a measurement switch: the
// register-streaming kernels below instead).
bool gemv_stream_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("TC_GEMV_STREAM");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

// Shared memory of one streaming-GEMV CTA in KB (TC_GEMV_STREAM_KB, a measurement switch; default
// the full budget: one CTA per SM).
int gemv_stream_budget() {
  static const int b = [] {
    const char* e = std::getenv("TC_GEMV_STREAM_KB");
    const int kb = e != nullptr ? std::atoi(e) : 0;
    return kb > 0 && kb * 1024 < kGsSmemBudget ? kb * 1024 : kGsSmemBudget;
  }();
  return b;
}

// CTAs of a streaming GEMV: one per SM (at most one per row), more when a CTA would keep more than
// kGsMaxRowsPerCta results (the sum forms).
int64_t stream_ctas(int64_t n, int sms, bool ar_mode) {
  int64_t c = n < sms ? n : sms;
  if (ar_mode && (n + c - 1) / c > kGsMaxRowsPerCta) c = (n + kGsMaxRowsPerCta - 1) / kGsMaxRowsPerCta;
  return c;
}

template <typename T>
cudaError_t launch_stream_t(bool swiglu, bool ar_mode, const ArPeers& ar, cudaStream_t st, const void* x,
                            const void* w, void* out, int64_t n, int k, int sms, int dev,
                            const NormIn* norm_in = nullptr, bool act_out = false) {
  const GsPlan g = gs_plan(k, gemv_stream_budget());
  int64_t c = stream_ctas(n, sms, ar_mode);
  if (act_out) {  // whole gate/up pairs per CTA, at most kGsMaxActRows rows
    const int64_t pairs = n / 2;
    c = pairs < sms ? pairs : sms;
    if (2 * ((pairs + c - 1) / c) > kGsMaxActRows) c = (pairs + kGsMaxActRows / 2 - 1) / (kGsMaxActRows / 2);
  }
  const int smem = g.x_bytes + g.nstages * g.stage_bytes;
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  T* op = static_cast<T*>(out);
  NormIn ni;
  std::memset(&ni, 0, sizeof(ni));
  if (norm_in != nullptr) ni = *norm_in;
  auto fn = act_out            ? gemv_stream_kernel<T, false, false, true, true>
            : norm_in != nullptr ? gemv_stream_kernel<T, false, false, true>
            : ar_mode ? (swiglu ? gemv_stream_kernel<T, true, true, false> : gemv_stream_kernel<T, false, true, false>)
                      : (swiglu ? gemv_stream_kernel<T, true, false, false> : gemv_stream_kernel<T, false, false, false>);
  // the opt-in is set once per (kernel, device) by set_smem: ask for the budget every plan fits in
  const cudaError_t e = set_smem(reinterpret_cast<const void*>(fn), kGsSmemBudget, dev);
  if (e != cudaSuccess) return e;
  return launch_pdl(fn, dim3((unsigned)c), dim3(kGsThreads), (size_t)smem, st, xp, wp, op, n, k, ar, g, ni);
}

template <typename T>
cudaError_t launch_splitk_t(bool swiglu, bool ar_mode, const ArPeers& ar, cudaStream_t st, const void* x,
                            const void* w, void* out, int64_t n, int k) {
  const dim3 grid((unsigned)((n + kSkRows - 1) / kSkRows));
  const size_t smem = (size_t)k * 2;
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  T* op = static_cast<T*>(out);
  if (ar_mode)
    return swiglu ? launch_pdl(gemv_splitk_kernel<T, true, true>, grid, dim3(kGemvWarps * 32), smem, st, xp, wp, op, n, k, ar)
                  : launch_pdl(gemv_splitk_kernel<T, false, true>, grid, dim3(kGemvWarps * 32), smem, st, xp, wp, op, n, k, ar);
  return swiglu ? launch_pdl(gemv_splitk_kernel<T, true, false>, grid, dim3(kGemvWarps * 32), smem, st, xp, wp, op, n, k, ar)
                : launch_pdl(gemv_splitk_kernel<T, false, false>, grid, dim3(kGemvWarps * 32), smem, st, xp, wp, op, n, k, ar);
}

int run_gemv(const void* x, const void* w, void* out, int64_t n, int k, int dtype, void* stream, bool swiglu) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (n < 0 || k < 8 || k % 8 || k > 24576) return TC_ERR_INVALID;
  if (n == 0) return TC_OK;
  if (x == nullptr || w == nullptr || out == nullptr) return TC_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return TC_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (gemv_stream_enabled()) {
    ArPeers none;
    std::memset(&none, 0, sizeof(none));
    const int dev = current_device();
    const cudaError_t e =
        dtype == TC_BF16 ? launch_stream_t<__nv_bfloat16>(swiglu, false, none, st, x, w, out, n, k, sm_count(dev), dev)
                         : launch_stream_t<__half>(swiglu, false, none, st, x, w, out, n, k, sm_count(dev), dev);
    return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
  }
  if (k >= splitk_min()) {  // long rows: K split over the warps of a CTA (see gemv_splitk_kernel)
    ArPeers none;
    std::memset(&none, 0, sizeof(none));
    const cudaError_t e = dtype == TC_BF16 ? launch_splitk_t<__nv_bfloat16>(swiglu, false, none, st, x, w, out, n, k)
                                           : launch_splitk_t<__half>(swiglu, false, none, st, x, w, out, n, k);
    return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
  }
  const int sms = sm_count(current_device());
  // rows per warp: 4 when there are enough rows for two CTAs of 4-row warps on every SM, 2 for one,
  // else 1 (more warps stream, each with fewer rows in flight)
  const int rpw = n >= (int64_t)sms * 2 * kGemvWarps * 4 ? 4 : (n >= (int64_t)sms * kGemvWarps * 2 ? 2 : 1);
  const int64_t want = (n + (int64_t)kGemvWarps * rpw - 1) / ((int64_t)kGemvWarps * rpw);
  const unsigned grid = (unsigned)(want < (int64_t)sms * 64 ? want : (int64_t)sms * 64);
  const size_t smem = (size_t)k * 2;
  cudaError_t e;
  if (dtype == TC_BF16)
    e = launch_gemv_t<__nv_bfloat16>(rpw, swiglu, grid, smem, st, x, w, out, n, k);
  else
    e = launch_gemv_t<__half>(rpw, swiglu, grid, smem, st, x, w, out, n, k);
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}
}  // namespace

extern "C" {

int tc_gemv(const void* x, const void* w, void* out, int64_t n, int k, int dtype, void* stream) {
  return run_gemv(x, w, out, n, k, dtype, stream, false);
}

int tc_gemv_swiglu(const void* gate_up, const void* w, void* out, int64_t n, int k, int dtype, void* stream) {
  return run_gemv(gate_up, w, out, n, k, dtype, stream, true);
}

int tc_silu_mul(const void* gate_up, void* out, int64_t rows, int inter, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (rows < 0 || inter < 1 || rows > ((int64_t)1 << 40) / inter) return TC_ERR_INVALID;
  if (rows == 0) return TC_OK;
  if (gate_up == nullptr || out == nullptr) return TC_ERR_INVALID;
  return launch_layer_op(dtype, 2, out, nullptr, gate_up, nullptr, nullptr, nullptr, rows, inter, 0, 0, 0.f, stream);
}

}  // extern "C"

// ---------------------------------------------------------------- sums over GPUs through peer memory
extern "C" {

size_t tc_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int tc_peer_alloc(size_t bytes, void** dev_ptr, void* handle_out) {
  if (bytes == 0 || dev_ptr == nullptr || handle_out == nullptr) return TC_ERR_INVALID;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return TC_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return TC_ERR_CUDA;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return TC_OK;
}

int tc_peer_open(const void* handle, void** dev_ptr) {
  if (handle == nullptr || dev_ptr == nullptr) return TC_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_peer_close(void* dev_ptr) {
  if (dev_ptr == nullptr) return TC_ERR_INVALID;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_peer_free(void* dev_ptr) {
  if (dev_ptr == nullptr) return TC_ERR_INVALID;
  return cudaFree(dev_ptr) == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

size_t tc_allreduce_region_bytes(int world, int64_t rows) {
  if (world < 1 || world > kArMaxWorld || rows < 1 || rows > 8192) return 0;
  return (size_t)kArDataOffset + (size_t)kArSlots * world * rows * sizeof(uint64_t);
}

namespace {
int run_gemv_allreduce(const void* x, const void* w, int64_t n, int k, void* const* regions, int world, int rank,
                       int dtype, void* stream, bool swiglu, void* residual = nullptr) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (residual != nullptr && (!gemv_stream_enabled() || (reinterpret_cast<uintptr_t>(residual) & 1)))
    return TC_ERR_INVALID;  // the residual form is a streaming-GEMV epilogue
  if (world < 1 || world > kArMaxWorld || rank < 0 || rank >= world || regions == nullptr) return TC_ERR_INVALID;
  if (n < 1 || n > 8192 || k < 8 || k % 8 || k > 24576) return TC_ERR_INVALID;
  if (x == nullptr || w == nullptr) return TC_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return TC_ERR_ALIGN;
  ArPeers ar;
  std::memset(&ar, 0, sizeof(ar));
  for (int p = 0; p < world; ++p) {
    if (regions[p] == nullptr || (reinterpret_cast<uintptr_t>(regions[p]) & 255)) return TC_ERR_INVALID;
    ar.data[p] = reinterpret_cast<uint64_t*>(static_cast<char*>(regions[p]) + kArDataOffset);
  }
  ar.seq = static_cast<const unsigned int*>(regions[rank]);
  ar.world = world;
  ar.rank = rank;
  ar.rows = n;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (residual != nullptr) {
    const int dev = current_device();
    if (stream_ctas(n, sm_count(dev), true) > kArSsParts) return TC_ERR_INVALID;
    ar.h = residual;
    ar.ss = reinterpret_cast<float*>(static_cast<char*>(regions[rank]) + kArSsOffset);
    ar.done = static_cast<unsigned int*>(regions[rank]) + 1;
  }
  if (gemv_stream_enabled()) {
    const int dev = current_device();
    const cudaError_t e =
        dtype == TC_BF16 ? launch_stream_t<__nv_bfloat16>(swiglu, true, ar, st, x, w, nullptr, n, k, sm_count(dev), dev)
                         : launch_stream_t<__half>(swiglu, true, ar, st, x, w, nullptr, n, k, sm_count(dev), dev);
    return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
  }
  if (k >= splitk_min()) {  // long rows: K split over the warps of a CTA
    const cudaError_t e = dtype == TC_BF16 ? launch_splitk_t<__nv_bfloat16>(swiglu, true, ar, st, x, w, nullptr, n, k)
                                           : launch_splitk_t<__half>(swiglu, true, ar, st, x, w, nullptr, n, k);
    return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
  }
  const dim3 grid((unsigned)((n + kArRows - 1) / kArRows));
  const size_t smem = (size_t)k * 2;
  cudaError_t e;
  if (dtype == TC_BF16) {
    using B = __nv_bfloat16;
    e = swiglu ? launch_pdl(gemv_allreduce_kernel<B, true>, grid, dim3(kArThreads), smem, st, static_cast<const B*>(x),
                            static_cast<const B*>(w), n, k, ar)
               : launch_pdl(gemv_allreduce_kernel<B, false>, grid, dim3(kArThreads), smem, st,
                            static_cast<const B*>(x), static_cast<const B*>(w), n, k, ar);
  } else {
    using H = __half;
    e = swiglu ? launch_pdl(gemv_allreduce_kernel<H, true>, grid, dim3(kArThreads), smem, st, static_cast<const H*>(x),
                            static_cast<const H*>(w), n, k, ar)
               : launch_pdl(gemv_allreduce_kernel<H, false>, grid, dim3(kArThreads), smem, st,
                            static_cast<const H*>(x), static_cast<const H*>(w), n, k, ar);
  }
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}
}  // namespace

int tc_gemv_allreduce(const void* x, const void* w, int64_t n, int k, void* const* regions, int world, int rank,
                      int dtype, void* stream) {
  return run_gemv_allreduce(x, w, n, k, regions, world, rank, dtype, stream, false);
}

int tc_gemv_allreduce_swiglu(const void* gate_up, const void* w, int64_t n, int k, void* const* regions, int world,
                             int rank, int dtype, void* stream) {
  return run_gemv_allreduce(gate_up, w, n, k, regions, world, rank, dtype, stream, true);
}

int tc_gemv_allreduce_residual(const void* x, const void* w, int64_t n, int k, void* const* regions, int world,
                               int rank, void* h, int dtype, void* stream) {
  if (h == nullptr) return TC_ERR_INVALID;
  return run_gemv_allreduce(x, w, n, k, regions, world, rank, dtype, stream, false, h);
}

int tc_gemv_allreduce_residual_swiglu(const void* gate_up, const void* w, int64_t n, int k, void* const* regions,
                                      int world, int rank, void* h, int dtype, void* stream) {
  if (h == nullptr) return TC_ERR_INVALID;
  return run_gemv_allreduce(gate_up, w, n, k, regions, world, rank, dtype, stream, true, h);
}

int tc_gemv_rmsnorm(const void* h, const void* norm_weight, const void* region, float eps, const void* w, void* out,
                    int64_t n, int k, int dtype, void* stream) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (n < 0 || k < 8 || k % 8 || k > 8 * kGsStageBatch * 32 * kGsConsumers || !(eps >= 0.f)) return TC_ERR_INVALID;
  if (n == 0) return TC_OK;
  if (h == nullptr || norm_weight == nullptr || region == nullptr || w == nullptr || out == nullptr)
    return TC_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(norm_weight) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(region)) & 15)
    return TC_ERR_ALIGN;
  if (!gemv_stream_enabled()) return TC_ERR_INVALID;  // the normalised input is a streaming-GEMV staging mode
  NormIn ni;
  ni.h = h;
  ni.weight = norm_weight;
  ni.ss = reinterpret_cast<const float*>(static_cast<const char*>(region) + kArSsOffset);
  ni.inv_h = 1.0f / (float)k;
  ni.eps = eps;
  ArPeers none;
  std::memset(&none, 0, sizeof(none));
  const int dev = current_device();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      dtype == TC_BF16 ? launch_stream_t<__nv_bfloat16>(false, false, none, st, h, w, out, n, k, sm_count(dev), dev, &ni)
                       : launch_stream_t<__half>(false, false, none, st, h, w, out, n, k, sm_count(dev), dev, &ni);
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_gemv_rmsnorm_swiglu(const void* h, const void* norm_weight, const void* region, float eps, const void* w,
                           void* out, int64_t n, int k, int dtype, void* stream) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (n < 0 || n % 2 || k < 8 || k % 8 || k > 8 * kGsStageBatch * 32 * kGsConsumers || !(eps >= 0.f))
    return TC_ERR_INVALID;
  if (n == 0) return TC_OK;
  if (h == nullptr || norm_weight == nullptr || region == nullptr || w == nullptr || out == nullptr)
    return TC_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(norm_weight) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(region)) & 15)
    return TC_ERR_ALIGN;
  if (!gemv_stream_enabled()) return TC_ERR_INVALID;  // a streaming-GEMV staging mode and epilogue
  NormIn ni;
  ni.h = h;
  ni.weight = norm_weight;
  ni.ss = reinterpret_cast<const float*>(static_cast<const char*>(region) + kArSsOffset);
  ni.inv_h = 1.0f / (float)k;
  ni.eps = eps;
  ArPeers none;
  std::memset(&none, 0, sizeof(none));
  const int dev = current_device();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      dtype == TC_BF16
          ? launch_stream_t<__nv_bfloat16>(false, false, none, st, h, w, out, n, k, sm_count(dev), dev, &ni, true)
          : launch_stream_t<__half>(false, false, none, st, h, w, out, n, k, sm_count(dev), dev, &ni, true);
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

int tc_allreduce_add_rmsnorm(void* h, const void* weight, void* out, int hidden, float eps, void* region,
                             int world, int dtype, void* stream) {
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ERR_DTYPE;
  if (world < 1 || world > kArMaxWorld || hidden < 1 || hidden > kArNormThreads * kArMaxPerThread || !(eps >= 0.f))
    return TC_ERR_INVALID;
  if (h == nullptr || weight == nullptr || out == nullptr || region == nullptr) return TC_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(region) & 255) return TC_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t* mine = reinterpret_cast<const uint64_t*>(static_cast<char*>(region) + kArDataOffset);
  unsigned int* seq = static_cast<unsigned int*>(region);
  const int64_t rows = hidden;
  cudaError_t e;
  if (dtype == TC_BF16)
    e = launch_pdl(allreduce_add_rmsnorm_kernel<__nv_bfloat16>, dim3(1), dim3(kArNormThreads), 0, st,
                   static_cast<__nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(weight),
                   static_cast<__nv_bfloat16*>(out), hidden, 1.0f / (float)hidden, eps, mine, seq, world, rows);
  else
    e = launch_pdl(allreduce_add_rmsnorm_kernel<__half>, dim3(1), dim3(kArNormThreads), 0, st,
                   static_cast<__half*>(h), static_cast<const __half*>(weight), static_cast<__half*>(out), hidden,
                   1.0f / (float)hidden, eps, mine, seq, world, rows);
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

}  // extern "C"

extern "C" {

size_t tc_gather_region_bytes(int world, int64_t rows, int d) {
  if (world < 1 || world > kArMaxWorld || rows < 1 || d < 4 || d % 4 || rows > ((int64_t)1 << 24)) return 0;
  return (size_t)kArCtrlBytes + 2 * (size_t)world * (size_t)gather_src_stride(rows, d) * sizeof(float);
}

int tc_peer_gather_merge(const float* o_local, const float* lse_local, void* out, float* lse_out, int64_t rows, int d,
                         int64_t out_stride_row, void* const* regions, int world, int rank, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return TC_ERR_DTYPE;
  if (tc_gather_region_bytes(world, rows, d) == 0 || rank < 0 || rank >= world || out_stride_row < d)
    return TC_ERR_INVALID;
  if (o_local == nullptr || lse_local == nullptr || out == nullptr || regions == nullptr) return TC_ERR_INVALID;
  if (!aligned16(o_local)) return TC_ERR_ALIGN;
  GatherPeers gp;
  std::memset(&gp, 0, sizeof(gp));
  for (int p = 0; p < world; ++p) {
    if (regions[p] == nullptr || (reinterpret_cast<uintptr_t>(regions[p]) & 255)) return TC_ERR_INVALID;
    gp.ctrl[p] = static_cast<unsigned int*>(regions[p]);
    gp.data[p] = reinterpret_cast<float*>(static_cast<char*>(regions[p]) + kArCtrlBytes);
  }
  gp.world = world;
  gp.rank = rank;
  gp.src_stride = gather_src_stride(rows, d);
  gp.slot_stride = (int64_t)world * gp.src_stride;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t mergers = (rows * (d / 4) + kGmThreads - 1) / kGmThreads;  // one thread per float4 of out
  const dim3 grid((unsigned)((world - 1) * kGmPushers + mergers));
  cudaError_t e;
  if (dtype == TC_BF16)
    e = launch_pdl(gather_merge_kernel<__nv_bfloat16>, grid, dim3(kGmThreads), 0, st, o_local, lse_local,
                   static_cast<__nv_bfloat16*>(out), lse_out, rows, d, out_stride_row, gp);
  else if (dtype == TC_F16)
    e = launch_pdl(gather_merge_kernel<__half>, grid, dim3(kGmThreads), 0, st, o_local, lse_local,
                   static_cast<__half*>(out), lse_out, rows, d, out_stride_row, gp);
  else
    e = launch_pdl(gather_merge_kernel<float>, grid, dim3(kGmThreads), 0, st, o_local, lse_local,
                   static_cast<float*>(out), lse_out, rows, d, out_stride_row, gp);
  return e == cudaSuccess ? TC_OK : TC_ERR_CUDA;
}

}  // extern "C"
