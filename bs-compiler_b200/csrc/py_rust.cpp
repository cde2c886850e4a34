// py_rust.cpp — the `basalto._rust` extension module.
//
// Same Python surface as the reference's PyO3 module (crates/basalto-tree/src/interceptor.rs:
// 527-580): class PyBasaltoInterceptor() with
//   compile_and_execute(op, dtype, shape, strides, job_id, device_ptr_x, device_ptr_y,
//                       device_ptr_z)
// which releases the GIL and raises RuntimeError on failure.  Keyword-only extras of this
// build: custom_coeffs (the Rust-level `custom_coeffs`), program (a packed bst_program)
// and stream (a cudaStream_t as int).  Without stream the call is synchronous, as the
// reference's launch is; with one (0 included: torch's default stream) it is queued on that
// stream and returns at once.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/basalto_b200.h"

namespace py = pybind11;

static void check(int rc) {
  if (rc != BST_OK) throw std::runtime_error(bst_last_error());
}

class PyBasaltoInterceptor {
 public:
  PyBasaltoInterceptor() { check(bst_interceptor_create(&h_)); }
  ~PyBasaltoInterceptor() { bst_interceptor_destroy(h_); }
  PyBasaltoInterceptor(const PyBasaltoInterceptor&) = delete;
  PyBasaltoInterceptor& operator=(const PyBasaltoInterceptor&) = delete;

  void compile_and_execute(const std::string& op, const std::string& dtype, const std::vector<int64_t>& shape,
                           const std::vector<int64_t>& strides, std::optional<std::string> job_id,
                           uint64_t device_ptr_x, uint64_t device_ptr_y, uint64_t device_ptr_z,
                           std::optional<std::vector<double>> custom_coeffs, std::optional<py::bytes> program,
                           std::optional<uint64_t> stream) {
    if (shape.empty() || shape.size() > 3)
      throw std::runtime_error("only 1-D, 2-D and 3-D are supported (shape has " + std::to_string(shape.size()) +
                               " dims)");
    if (shape.size() != strides.size()) throw std::runtime_error("shape and strides must have the same length");
    std::string prog_bytes;
    if (program) {
      prog_bytes = std::string(*program);
      if (prog_bytes.size() != sizeof(bst_program))
        throw std::runtime_error("program must be a packed bst_program of " + std::to_string(sizeof(bst_program)) +
                                 " bytes");
    }
    // A null stream makes the C ABI synchronous; the legacy default stream given explicitly (handle
    // 0, as torch reports it) is passed as CUDA's own handle for it, cudaStreamLegacy = 0x1.
    void* st = nullptr;
    if (stream) st = reinterpret_cast<void*>(*stream == 0 ? uint64_t(0x1) : *stream);
    const double* cc = custom_coeffs ? custom_coeffs->data() : nullptr;
    const int64_t nc = custom_coeffs ? int64_t(custom_coeffs->size()) : 0;
    int rc;
    {
      py::gil_scoped_release nogil;
      rc = bst_interceptor_compile_and_execute(
          h_, op.c_str(), dtype.c_str(), int32_t(shape.size()), shape.data(), strides.data(),
          job_id ? job_id->c_str() : nullptr, device_ptr_x, device_ptr_y, device_ptr_z, cc, nc,
          program ? reinterpret_cast<const bst_program*>(prog_bytes.data()) : nullptr, st);
    }
    check(rc);
  }

  int64_t cache_size() const { return bst_interceptor_cache_size(h_); }
  int64_t cache_hits() const { return bst_interceptor_cache_hits(h_); }
  std::string last_cache_key() const {
    char k[65] = {0};
    check(bst_interceptor_last_key(h_, k));
    return k;
  }

 private:
  bst_interceptor* h_ = nullptr;
};

PYBIND11_MODULE(_rust, m) {
  m.doc() = "B200-native Basalto interceptor (C++ host over sm_100a stencil kernels)";
  py::class_<PyBasaltoInterceptor>(m, "PyBasaltoInterceptor")
      .def(py::init<>())
      .def("compile_and_execute", &PyBasaltoInterceptor::compile_and_execute, py::arg("op"), py::arg("dtype"),
           py::arg("shape"), py::arg("strides"), py::arg("job_id"), py::arg("device_ptr_x"),
           py::arg("device_ptr_y"), py::arg("device_ptr_z"), py::kw_only(), py::arg("custom_coeffs") = py::none(),
           py::arg("program") = py::none(), py::arg("stream") = py::none())
      .def("cache_size", &PyBasaltoInterceptor::cache_size)
      .def("cache_hits", &PyBasaltoInterceptor::cache_hits)
      .def("last_cache_key", &PyBasaltoInterceptor::last_cache_key);
  m.def("abi_version", &bst_abi_version);
  m.def("launch_count", &bst_launch_count);
  m.def("extract_radius", [](const std::string& op) { return bst_extract_radius(op.c_str()); });
  m.attr("PROGRAM_NBYTES") = py::int_(sizeof(bst_program));
}
