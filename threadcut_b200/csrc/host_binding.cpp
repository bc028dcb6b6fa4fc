// Host fast path of threadcut_b200.flash_decode.decode_attention (and decode_attention_partial):
// the tensor checks, the output
// allocation and the C-ABI call in one crossing from Python, instead of a ctypes call with 23
// converted arguments plus a dozen tensor attribute lookups in the interpreter. Host code only (no
// device code); it calls the library's tc_decode_attention_stable through a function pointer handed
// over by the ctypes loader, so it uses the very library instance the rest of the package loaded.
//
// decode(q, k, v, scale, splits, stable_rows, workspace) returns the output tensor, or None when
// anything is off (not CUDA, mixed devices or dtypes, wrong ranks or shapes, a non-contiguous last
// dimension, an unsupported dtype, or a non-zero status from the library): the caller then takes
// the checked Python path, which raises the documented exception for that case.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cstdint>

namespace {

using DecodeStableFn = int (*)(const void*, const void*, const void*, void*, int, int, int, int64_t, int64_t,
                               int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float, int, int,
                               int64_t, void*, size_t, void*);

using PartialStableFn = int (*)(const void*, const void*, const void*, float*, float*, int, int, int, int64_t,
                                int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float, int,
                                int, int64_t, void*, size_t, void*);

DecodeStableFn g_decode = nullptr;
PartialStableFn g_partial = nullptr;

void init(int64_t decode_stable_addr) { g_decode = reinterpret_cast<DecodeStableFn>(decode_stable_addr); }
void init_partial(int64_t partial_stable_addr) {
  g_partial = reinterpret_cast<PartialStableFn>(partial_stable_addr);
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return 0;
    case at::kHalf: return 1;
    case at::kBFloat16: return 2;
    default: return -1;
  }
}

py::object decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale, int64_t splits,
                  int64_t stable_rows, const at::Tensor& ws) {
  if (g_decode == nullptr) return py::none();
  if (!q.is_cuda() || !k.is_cuda() || !v.is_cuda() || !ws.is_cuda()) return py::none();
  const auto dev = q.device();
  if (k.device() != dev || v.device() != dev || ws.device() != dev) return py::none();
  if (q.dim() != 3 || k.dim() != 3 || v.dim() != 3) return py::none();
  if (k.scalar_type() != q.scalar_type() || v.scalar_type() != q.scalar_type()) return py::none();
  const int code = dtype_code(q.scalar_type());
  if (code < 0) return py::none();
  const int64_t hkv = q.size(0), g = q.size(1), d = q.size(2), n = k.size(1);
  if (k.size(0) != hkv || k.size(2) != d || v.sizes() != k.sizes()) return py::none();
  if (q.stride(2) != 1 || k.stride(2) != 1 || v.stride(2) != 1) return py::none();
  if (stable_rows < 0) return py::none();
  c10::cuda::CUDAGuard guard(dev);
  at::Tensor out = at::empty({hkv, g, d}, q.options());
  const cudaStream_t st = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  const int rc = g_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), (int)hkv, (int)g, (int)d, n,
                          q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
                          out.stride(0), out.stride(1), (float)scale, (int)splits, code, stable_rows,
                          ws.data_ptr(), (size_t)ws.numel(), st);
  if (rc != 0) return py::none();
  return py::cast(out);
}

// The same for decode_attention_partial: (out fp32 [hkv, g, d], lse fp32 [hkv, g]) through
// tc_decode_attention_partial_stable, or None.
py::object partial(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale, int64_t splits,
                   int64_t stable_rows, const at::Tensor& ws) {
  if (g_partial == nullptr) return py::none();
  if (!q.is_cuda() || !k.is_cuda() || !v.is_cuda() || !ws.is_cuda()) return py::none();
  const auto dev = q.device();
  if (k.device() != dev || v.device() != dev || ws.device() != dev) return py::none();
  if (q.dim() != 3 || k.dim() != 3 || v.dim() != 3) return py::none();
  if (k.scalar_type() != q.scalar_type() || v.scalar_type() != q.scalar_type()) return py::none();
  const int code = dtype_code(q.scalar_type());
  if (code < 0) return py::none();
  const int64_t hkv = q.size(0), g = q.size(1), d = q.size(2), n = k.size(1);
  if (k.size(0) != hkv || k.size(2) != d || v.sizes() != k.sizes()) return py::none();
  if (q.stride(2) != 1 || k.stride(2) != 1 || v.stride(2) != 1) return py::none();
  if (stable_rows < 0) return py::none();
  c10::cuda::CUDAGuard guard(dev);
  at::Tensor out = at::empty({hkv, g, d}, q.options().dtype(at::kFloat));
  at::Tensor lse = at::empty({hkv, g}, q.options().dtype(at::kFloat));
  const cudaStream_t st = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  const int rc = g_partial(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr<float>(), lse.data_ptr<float>(),
                           (int)hkv, (int)g, (int)d, n, q.stride(0), q.stride(1), k.stride(0), k.stride(1),
                           v.stride(0), v.stride(1), out.stride(0), out.stride(1), (float)scale, (int)splits, code,
                           stable_rows, ws.data_ptr(), (size_t)ws.numel(), st);
  if (rc != 0) return py::none();
  return py::make_tuple(out, lse);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("init", &init, "set the address of tc_decode_attention_stable");
  m.def("init_partial", &init_partial, "set the address of tc_decode_attention_partial_stable");
  m.def("decode", &decode, "checked decode_attention fast path; None means: take the Python path");
  m.def("partial", &partial, "checked decode_attention_partial fast path; None means: take the Python path");
}
