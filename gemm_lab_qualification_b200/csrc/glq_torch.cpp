// glq_torch.cpp -- the operator API's call path into libglq.so, in C++.
//
// The Python operators of kernels.py (triton_matmul_into, triton_bias_silu_into,
// triton_splitk_matmul_into and the Plans) check their arguments and call
// glq_linear_ex.  Doing both through Python attribute access and ctypes cost
// ~15 us per call on the host, more than the kernel itself, so a dependent
// chain of calls was host-bound.  This module does the same checks (same
// ValueError texts as kernels.py:132-145, 150-153, 259-262, 403-409, minus the
// contiguity rule) and the launch in one native call on torch's current
// stream.  Library failures come back as the glq_status so that Python raises
// the same GlqError as the ctypes binding.
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <sstream>
#include <string>
#include <tuple>
#include <vector>

#include <pybind11/stl.h>

#include "glq.h"

namespace {

std::string shape_str(const at::Tensor& t) {
  std::ostringstream s;
  s << '(';
  for (int64_t i = 0; i < t.dim(); ++i) s << (i ? ", " : "") << t.size(i);
  if (t.dim() == 1) s << ',';
  s << ')';
  return s.str();
}

void check_inputs(const at::Tensor& a, const at::Tensor& b, const std::string& op) {
  if (a.dim() != 2 || b.dim() != 2) throw py::value_error(op + " expects two rank-2 tensors");
  if (a.size(1) != b.size(0)) {
    throw py::value_error("incompatible dimensions: " + shape_str(a) + " and " + shape_str(b));
  }
  if (!a.is_cuda() || !b.is_cuda()) throw py::value_error(op + " requires CUDA tensors");
  if (a.device() != b.device()) throw py::value_error("input tensors must be on the same CUDA device");
  if (a.scalar_type() != b.scalar_type() ||
      (a.scalar_type() != at::kHalf && a.scalar_type() != at::kBFloat16)) {
    throw py::value_error("inputs must share dtype float16 or bfloat16");
  }
}

void check_output(const at::Tensor& out, const at::Tensor& a, int64_t m, int64_t n) {
  if (out.dim() != 2 || out.size(0) != m || out.size(1) != n || out.device() != a.device() ||
      out.scalar_type() != a.scalar_type()) {
    throw py::value_error("output tensor has the wrong shape, device, or dtype");
  }
  if (m && n && ((n > 1 && out.stride(1) != 1) || (m > 1 && out.stride(0) < n))) {
    throw py::value_error("output tensor must be contiguous");
  }
}

void check_bias(const at::Tensor& bias, const at::Tensor& a, int64_t n) {
  if (bias.dim() != 1 || bias.size(0) != n || bias.device() != a.device() || bias.scalar_type() != a.scalar_type()) {
    throw py::value_error("bias tensor has the wrong shape, device, or dtype");
  }
  if (n > 1 && bias.stride(0) != 1) throw py::value_error("bias tensor must be contiguous");
}

// Returns (glq_status, path, split).  `op` names the operator in messages.
std::tuple<int, int, int> linear(const std::string& op, const at::Tensor& a, const at::Tensor& b, at::Tensor& out,
                                 const c10::optional<at::Tensor>& bias, int epilogue, int split_k,
                                 const c10::optional<at::Tensor>& partial, int64_t flags) {
  check_inputs(a, b, op);
  const int64_t m = a.size(0), k = a.size(1), n = b.size(1);
  if (bias.has_value()) check_bias(*bias, a, n);
  check_output(out, a, m, n);
  const int dtype = a.scalar_type() == at::kHalf ? GLQ_DTYPE_F16 : GLQ_DTYPE_BF16;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  at::Tensor repack_ws;
  if (partial.has_value()) {
    ws = partial->data_ptr();
    ws_bytes = static_cast<size_t>(partial->numel()) * partial->element_size();
  } else if (m && n && k) {
    // Strided or unaligned operands: aligned copies in a workspace from
    // torch's caching allocator (stream-ordered, so it may be released as
    // soon as the launches are queued), then the tcgen05 / GEMV kernel.
    const size_t need = glq_linear_workspace_bytes(dtype, a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(),
                                                   b.stride(0), b.stride(1), m, n, k);
    if (need) {
      repack_ws = at::empty({static_cast<int64_t>(need)}, a.options().dtype(at::kByte));
      ws = repack_ws.data_ptr();
      ws_bytes = need;
    }
  }
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(a.device().index()).stream();
  int path = -1, split = 0;
  const int status = glq_linear_ex(dtype, a.data_ptr(),
                                   a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                                   bias.has_value() ? bias->data_ptr() : nullptr, epilogue, out.data_ptr(),
                                   out.stride(0), m, n, k, split_k, ws, ws_bytes, stream,
                                   static_cast<unsigned int>(flags), &path, &split);
  return {status, path, split};
}

// The fused-gather launch of the column-parallel layer (glq_linear_gather):
// per-rank output and signal-slot pointers as integers (peer mappings from
// torch symmetric memory).  Returns (glq_status, path, split).
std::tuple<int, int, int> linear_gather(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& bias,
                                        int epilogue, const std::vector<int64_t>& y_ptrs, int64_t y_row_stride,
                                        int64_t y_col_offset, int rank, const std::vector<int64_t>& signal_ptrs,
                                        int64_t counter, int64_t epoch, int split_k, int64_t flags) {
  check_inputs(a, b, "linear_gather");
  const int64_t m = a.size(0), k = a.size(1), n = b.size(1);
  if (bias.has_value()) check_bias(*bias, a, n);
  if (y_ptrs.size() != signal_ptrs.size() || y_ptrs.empty() || y_ptrs.size() > GLQ_MAX_RANKS) {
    throw py::value_error("one output and one signal pointer per rank, at most GLQ_MAX_RANKS ranks");
  }
  void* ys[GLQ_MAX_RANKS];
  uint64_t* sigs[GLQ_MAX_RANKS];
  for (size_t r = 0; r < y_ptrs.size(); ++r) {
    ys[r] = reinterpret_cast<void*>(y_ptrs[r]);
    sigs[r] = reinterpret_cast<uint64_t*>(signal_ptrs[r]);
  }
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(a.device().index()).stream();
  int path = -1, split = 0;
  const int status = glq_linear_gather(
      a.scalar_type() == at::kHalf ? GLQ_DTYPE_F16 : GLQ_DTYPE_BF16, a.data_ptr(), a.stride(0), a.stride(1),
      b.data_ptr(), b.stride(0), b.stride(1), bias.has_value() ? bias->data_ptr() : nullptr, epilogue, ys,
      y_row_stride, y_col_offset, m, n, k, split_k, rank, static_cast<int>(y_ptrs.size()), sigs,
      reinterpret_cast<unsigned int*>(counter), static_cast<uint64_t>(epoch), stream,
      static_cast<unsigned int>(flags), &path, &split);
  return {status, path, split};
}

}  // namespace

PYBIND11_MODULE(_glq_torch, mod) {
  mod.doc() = "Checks and launches of the gemm_lab operator API on libglq.so (torch current stream).";
  mod.def("linear", &linear, py::arg("op"), py::arg("a"), py::arg("b"), py::arg("out"), py::arg("bias"),
          py::arg("epilogue"), py::arg("split_k"), py::arg("partial"), py::arg("flags"));
  mod.def("linear_gather", &linear_gather, py::arg("a"), py::arg("b"), py::arg("bias"), py::arg("epilogue"),
          py::arg("y_ptrs"), py::arg("y_row_stride"), py::arg("y_col_offset"), py::arg("rank"),
          py::arg("signal_ptrs"), py::arg("counter"), py::arg("epoch"), py::arg("split_k"), py::arg("flags"));
}
