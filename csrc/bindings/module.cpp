// module.cpp -- pybind11/torch binding of libgicc (opengda_b200._C).
// Tensors are validated here; the kernels themselves live in libgicc.so.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "gicc/config.hpp"
#include "gicc/error.hpp"
#include "gicc/ops.hpp"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must be row-major (stride(1) == 1)");
}

at::Tensor gemm(const at::Tensor& A, const at::Tensor& B, c10::optional<at::Tensor> out, double alpha, bool out_f32,
                int64_t bn) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  TORCH_CHECK(A.size(1) == B.size(1), "A[M,K] and B[N,K] must share K");
  const c10::cuda::CUDAGuard g(A.device());
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  at::Tensor C;
  if (out.has_value()) {
    C = *out;
    TORCH_CHECK(C.is_cuda() && C.dim() == 2 && C.size(0) == M && C.size(1) == N && C.stride(1) == 1, "bad out");
    TORCH_CHECK(C.scalar_type() == (out_f32 ? at::kFloat : at::kBFloat16), "out dtype mismatch");
  } else {
    C = at::empty({M, N}, A.options().dtype(out_f32 ? at::kFloat : at::kBFloat16));
  }
  gicc::ops::gemm_bf16(A.data_ptr(), B.data_ptr(), C.data_ptr(), (int)M, (int)N, (int)K, A.stride(0), B.stride(0),
                       C.stride(0), out_f32, (float)alpha, (int)bn, cur_stream());
  return C;
}

at::Tensor gemm_fp32(const at::Tensor& A, const at::Tensor& B, c10::optional<at::Tensor> out, double alpha,
                     int64_t bn) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && A.scalar_type() == at::kFloat && B.scalar_type() == at::kFloat &&
                  A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1,
              "A[M,K], B[N,K]: fp32 CUDA matrices with unit column stride");
  TORCH_CHECK(A.size(1) == B.size(1), "A[M,K] and B[N,K] must share K");
  const c10::cuda::CUDAGuard g(A.device());
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  at::Tensor C;
  if (out.has_value()) {
    C = *out;
    TORCH_CHECK(C.is_cuda() && C.dim() == 2 && C.size(0) == M && C.size(1) == N && C.stride(1) == 1 &&
                    C.scalar_type() == at::kFloat, "bad out");
  } else {
    C = at::empty({M, N}, A.options());
  }
  at::Tensor work = at::empty({(M + N) * 3 * K}, A.options());
  gicc::ops::gemm_fp32(A.data_ptr<float>(), B.data_ptr<float>(), C.data_ptr<float>(), (int)M, (int)N, (int)K,
                       A.stride(0), B.stride(0), C.stride(0), (float)alpha, work.data_ptr<float>(), cur_stream(),
                       (int)bn);
  return C;
}

void gemm_tile_done_selftest(const at::Tensor& A, const at::Tensor& B, const at::Tensor& counters, int64_t skew_ns) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && A.size(1) == B.size(1), "A[M,K], B[N,K] contiguous");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.is_contiguous(), "int32 counters");
  const c10::cuda::CUDAGuard g(A.device());
  gicc::ops::gemm_tile_done_selftest(A.data_ptr(), B.data_ptr(), (int)A.size(0), (int)B.size(0), (int)A.size(1),
                                     static_cast<uint32_t*>(counters.data_ptr()), (uint32_t)skew_ns, cur_stream());
}

py::dict read_errors(bool clear) {
  gicc::ErrorRecord r = gicc::read_error_record(clear);
  py::dict d;
  d["code"] = r.code;
  d["status"] = gicc::status_name(r.code);
  d["where"] = gicc::where_name(r.where);
  d["rank"] = r.rank;
  d["peer"] = r.peer;
  d["value"] = r.value;
  d["expected"] = r.expected;
  d["count"] = r.count;
  return d;
}

at::ScalarType dtype_from_name(const std::string& n) {
  if (n == "bfloat16") return at::kBFloat16;
  if (n == "float16") return at::kHalf;
  if (n == "float32") return at::kFloat;
  if (n == "float64") return at::kDouble;
  if (n == "int32") return at::kInt;
  if (n == "int64") return at::kLong;
  if (n == "uint8") return at::kByte;
  if (n == "int8") return at::kChar;
  throw std::runtime_error("tensor_from_ptr: unsupported dtype " + n);
}

// Zero-copy tensor view of device memory owned elsewhere (symmetric buffers, peer
// mappings, multicast addresses).  The caller keeps the owner alive.
at::Tensor tensor_from_ptr(uint64_t ptr, std::vector<int64_t> shape, const std::string& dtype, int device) {
  auto opts = at::TensorOptions().dtype(dtype_from_name(dtype)).device(at::kCUDA, device);
  return at::from_blob(reinterpret_cast<void*>(static_cast<uintptr_t>(ptr)), shape, opts);
}

}  // namespace

void bind_runtime(py::module_& m);  // runtime.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "opengda_b200 native ops (sm_100a)";
  m.def("set_gemm_tuning", [](int group_m, int l2_hint, int pair_group_m, int pair_l2_hint, int pair_prefetch,
                              int pair_tma_store) {
    gicc::ops::GemmTuning t;
    t.group_m = group_m;
    t.l2_hint = l2_hint;
    t.pair_group_m = pair_group_m;
    t.pair_l2_hint = pair_l2_hint;
    t.pair_prefetch = pair_prefetch;
    t.pair_tma_store = pair_tma_store;
    gicc::ops::set_gemm_tuning(t);
  }, py::arg("group_m") = 16, py::arg("l2_hint") = 0, py::arg("pair_group_m") = 16, py::arg("pair_l2_hint") = 0,
     py::arg("pair_prefetch") = 0, py::arg("pair_tma_store") = 1);
  m.def("gemm_tuning", []() {
    const auto t = gicc::ops::gemm_tuning();
    py::dict d;
    d["group_m"] = t.group_m;
    d["l2_hint"] = t.l2_hint;
    d["pair_group_m"] = t.pair_group_m;
    d["pair_l2_hint"] = t.pair_l2_hint;
    d["pair_prefetch"] = t.pair_prefetch;
    d["pair_tma_store"] = t.pair_tma_store;
    return d;
  });
  m.def("gemm", &gemm, py::arg("A"), py::arg("B"), py::arg("out") = py::none(), py::arg("alpha") = 1.0,
        py::arg("out_f32") = false, py::arg("bn") = 0, "C = alpha * A @ B^T with the tcgen05 GEMM");
  m.def("gemm_fp32", &gemm_fp32, py::arg("A"), py::arg("B"), py::arg("out") = py::none(), py::arg("alpha") = 1.0,
        py::arg("bn") = 0,
        "fp32 C = alpha * A @ B^T on the tensor cores (three tf32 products)");
  m.def("gemm_tile_done_selftest", &gemm_tile_done_selftest, py::arg("A"), py::arg("B"), py::arg("counters"),
        py::arg("skew_ns") = 20000, "run the GEMM core with an epilogue that checks the tile-done ordering");
  m.def("config", [] {
    const gicc::Config c = gicc::config();
    py::dict d;
    d["timeout_ms"] = c.timeout_ms;
    d["bootstrap_timeout_ms"] = c.bootstrap_timeout_ms;
    d["log_level"] = c.log_level;
    d["checks"] = c.checks;
    d["disable_nvls"] = c.disable_nvls;
    d["debug_puts"] = c.debug_puts;
    d["signal_heap_bytes"] = c.signal_heap_bytes;
    return d;
  }, "the GICC_* environment, parsed and range checked (raises ValueError on a bad value)");
  m.def("config_summary", [] { return gicc::config().summary(); });
  m.def("log", [](int level, const std::string& msg) { gicc::log(level, "%s", msg.c_str()); });
  m.def("read_errors", &read_errors, py::arg("clear") = true, "read (and clear) the device error record");
  m.def("default_timeout_ns", &gicc::default_timeout_ns);
  m.def("tensor_from_ptr", &tensor_from_ptr, py::arg("ptr"), py::arg("shape"), py::arg("dtype"), py::arg("device"));
  bind_runtime(m);
}
