// Python fast path of the b200 QuantLinear call: the checks and the launch of
// b200_w4g64_linear (backends.py) done in C++ on at::Tensor arguments, calling
// the C ABI of libqi4_b200.so directly (no ctypes marshalling, no Python
// attribute lookups). The model calls the linear about 200 times per decoded
// token, so the host cost per call is part of the decode time.
//
// Contract and error behaviour are those of the Python wrapper, which follows
// torch_reference_linear (reference src/qwen_int4/backends.py:73-98) and the
// reference's validators (backends.py:36-41, 166-167): ValueError / TypeError
// with the same messages, raised before any launch; RuntimeError carrying the
// library's message when a launch fails. Packing and group size are checked
// by the Python caller before it takes this path.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include "../../include/qi4_b200.h"

namespace py = pybind11;

namespace {

constexpr int64_t kGroup = 64;

// A shape as Python prints a tuple: "(8960, 24)", "(8960,)".
std::string tuple_str(at::IntArrayRef s) {
  std::string r = "(";
  for (size_t i = 0; i < s.size(); ++i) {
    if (i) r += ", ";
    r += std::to_string(s[i]);
  }
  if (s.size() == 1) r += ",";
  return r + ")";
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kHalf: return QI4_DTYPE_F16;
    case at::kBFloat16: return QI4_DTYPE_BF16;
    case at::kFloat: return QI4_DTYPE_F32;
    default: return QI4_DTYPE_NONE;
  }
}

void validate(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales, const at::Tensor& zeros,
              const c10::optional<at::Tensor>& bias, int64_t N, int64_t K) {
  if (K <= 0 || N <= 0 || K % kGroup)
    throw py::value_error("linear dimensions must be positive and divisible by group size 64");
  if (x.dim() < 1 || x.size(-1) != K) throw py::value_error("activation feature dimension does not match QuantLinear");
  if (dtype_code(x.scalar_type()) == QI4_DTYPE_NONE)
    throw py::type_error("B200 backend activations must use FP16, BF16, or FP32");
  if (qweight.scalar_type() != at::kByte || zeros.scalar_type() != at::kByte)
    throw py::type_error("canonical packed weights and zero points must use uint8 storage");
  if (scales.scalar_type() != at::kHalf) throw py::type_error("canonical group scales must use FP16 storage");
  const int64_t groups = K / kGroup;
  const int64_t expected_weight = N * K / 2, expected_zero = (N * groups + 1) / 2;
  if (qweight.numel() != expected_weight)
    throw py::value_error("qweight must contain " + std::to_string(expected_weight) + " bytes, got " +
                          std::to_string(qweight.numel()));
  if (scales.dim() != 2 || scales.size(0) != N || scales.size(1) != groups)
    throw py::value_error("scales must have shape (" + std::to_string(N) + ", " + std::to_string(groups) +
                          "), got " + tuple_str(scales.sizes()));
  if (zeros.numel() != expected_zero)
    throw py::value_error("zeros must contain " + std::to_string(expected_zero) + " bytes, got " +
                          std::to_string(zeros.numel()));
  if (bias) {
    if (bias->dim() != 1 || bias->size(0) != N)
      throw py::value_error("bias must have shape (" + std::to_string(N) + ",), got " + tuple_str(bias->sizes()));
    if (dtype_code(bias->scalar_type()) == QI4_DTYPE_NONE) throw py::type_error("bias must use FP16, BF16, or FP32");
  }
  if (!(x.is_cuda() && qweight.is_cuda() && scales.is_cuda() && zeros.is_cuda() && (!bias || bias->is_cuda())))
    throw py::value_error("B200 backend inputs must be CUDA tensors");
  const auto d = x.get_device();
  if (qweight.get_device() != d || scales.get_device() != d || zeros.get_device() != d ||
      (bias && bias->get_device() != d))
    throw py::value_error("all B200 backend inputs must be on the same device");
  if (!qweight.is_contiguous()) throw py::value_error("qweight must be contiguous");
  if (!scales.is_contiguous()) throw py::value_error("scales must be contiguous");
  if (!zeros.is_contiguous()) throw py::value_error("zeros must be contiguous");
  if (bias && !bias->is_contiguous()) throw py::value_error("bias must be contiguous");
}

const char* status_name(int rc) {
  switch (rc) {
    case QI4_ERR_ARGUMENT: return "ARGUMENT";
    case QI4_ERR_DTYPE: return "DTYPE";
    case QI4_ERR_SHAPE: return "SHAPE";
    case QI4_ERR_ALIGNMENT: return "ALIGNMENT";
    case QI4_ERR_LAUNCH: return "LAUNCH";
    case QI4_ERR_DEVICE: return "DEVICE";
    default: return "UNKNOWN";
  }
}

// The library's status -> the exception the Python wrapper raises for it.
[[noreturn]] void raise_status(int rc, const char* what) {
  char buf[512];
  qi4_last_error(buf, sizeof(buf));
  const std::string msg = std::string(what) + " failed (" + status_name(rc) + "): " + buf;
  if (rc == QI4_ERR_ARGUMENT || rc == QI4_ERR_SHAPE || rc == QI4_ERR_ALIGNMENT) throw py::value_error(msg);
  if (rc == QI4_ERR_DTYPE) throw py::type_error(msg);
  throw std::runtime_error(msg);
}

at::Tensor linear(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales, const at::Tensor& zeros,
                  const c10::optional<at::Tensor>& bias, int64_t N, int64_t K) {
  validate(x, qweight, scales, zeros, bias, N, K);
  at::Tensor x2 = x.reshape({-1, K}).contiguous();
  if (reinterpret_cast<uintptr_t>(x2.data_ptr()) % 16) x2 = x2.clone();  // the kernels use 16-byte loads
  const int64_t M = x2.size(0);
  at::Tensor out = at::empty({M, N}, x.options());
  if (M > 0) {
    if (reinterpret_cast<uintptr_t>(qweight.data_ptr()) % 16)
      throw py::value_error("qweight storage must be 16-byte aligned for the B200 kernels");
    const c10::cuda::CUDAGuard guard(x.device());
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.get_device()).stream();
    const int rc = qi4_w4g64_linear_ex(x2.data_ptr(), dtype_code(x2.scalar_type()), M, K,
                                       static_cast<const uint8_t*>(qweight.data_ptr()),
                                       static_cast<const uint16_t*>(scales.data_ptr()),
                                       static_cast<const uint8_t*>(zeros.data_ptr()),
                                       bias ? bias->data_ptr() : nullptr,
                                       bias ? dtype_code(bias->scalar_type()) : QI4_DTYPE_NONE, out.data_ptr(), N,
                                       stream, QI4_ALGO_AUTO, 1);
    if (rc) raise_status(rc, "qi4_w4g64_linear");
  }
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape.back() = N;
  return out.view(shape);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ fast path of b200_w4g64_linear (checks + launch through the qi4 C ABI)";
  m.def("linear", &linear, "Canonical W4G64 linear on the B200 kernels (same contract as b200_w4g64_linear)",
        py::arg("x"), py::arg("qweight"), py::arg("scales"), py::arg("zeros"), py::arg("bias"),
        py::arg("out_features"), py::arg("in_features"));
}
