// tied_ce_pybind.cpp — pybind11 device-pointer entry points of the B200 tied-CE
// library, in the form the reference's extension binds its CUDA kernels:
// every pointer is a std::uintptr_t (CuPy `.data.ptr` or torch `.data_ptr()`),
// sizes are integers, and a failing call throws std::runtime_error, which
// pybind11 raises as RuntimeError (NimbleML native/src/module.cpp:229-284,
// native/include/nimbleml/kernels.hpp:10-12). These m.def blocks are the ones
// a maintainer adds inside PYBIND11_MODULE(nimbleml_native, m); here they
// build the stand-alone module `nimbleml_tied_ce_native` against
// libnimbleml_tied_ce.so (nimbleml_b200/build_native.py).
#include <pybind11/pybind11.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "nimbleml_tied_ce.h"

namespace py = pybind11;

namespace {

template <typename T>
T* ptr(std::uintptr_t p) {
  return reinterpret_cast<T*>(p);
}

void check(int rc, const char* what) {
  if (rc != NIMBLE_OK) throw std::runtime_error(std::string(what) + ": " + nimble_tied_ce_last_error());
}

}  // namespace

PYBIND11_MODULE(nimbleml_tied_ce_native, m) {
  m.doc() = "B200 fused tied LM-head cross-entropy: device-pointer entry points";

  m.attr("DTYPE_F32") = static_cast<int>(NIMBLE_DTYPE_F32);
  m.attr("DTYPE_F16") = static_cast<int>(NIMBLE_DTYPE_F16);
  m.attr("DTYPE_BF16") = static_cast<int>(NIMBLE_DTYPE_BF16);
  m.attr("DTYPE_TF32") = static_cast<int>(NIMBLE_DTYPE_TF32);
  m.attr("STATUS_BAD_LABEL") = static_cast<int>(NIMBLE_STATUS_BAD_LABEL);
  m.attr("STATUS_WAIT_TIMEOUT") = static_cast<int>(NIMBLE_STATUS_WAIT_TIMEOUT);

  // Mirrors flash_sdpa_available (module.cpp:221-227).
  m.def("tied_ce_available", []() { return nimble_tied_ce_available() != 0; });

  m.def(
      "tied_ce_forward_workspace_size",
      [](std::int64_t n, std::int64_t d, std::int64_t v_local, int dtype) {
        std::size_t bytes = 0;
        check(nimble_tied_ce_forward_workspace_size(n, d, v_local, dtype, &bytes), "tied_ce_forward_workspace_size");
        return bytes;
      },
      py::arg("n_tokens"), py::arg("d_model"), py::arg("v_local"), py::arg("dtype"));

  m.def(
      "tied_ce_backward_workspace_size",
      [](std::int64_t n, std::int64_t d, std::int64_t v_local, int dtype, std::size_t slab_bytes) {
        std::size_t bytes = 0;
        check(nimble_tied_ce_backward_workspace_size(n, d, v_local, dtype, slab_bytes, &bytes),
              "tied_ce_backward_workspace_size");
        return bytes;
      },
      py::arg("n_tokens"), py::arg("d_model"), py::arg("v_local"), py::arg("dtype"), py::arg("slab_bytes") = 0);

  // Replaces the logits GEMM + row statistics of fused_tied_crossentropy_forward
  // (NimbleML/kernels/fused_tied_crossentropy.py:8-24) for one vocab shard.
  m.def(
      "tied_ce_forward_device",
      [](std::uintptr_t hidden, std::uintptr_t weights, std::uintptr_t labels, std::int64_t n, std::int64_t d,
         std::int64_t v_local, std::int64_t v_offset, int dtype, std::uintptr_t shard_max,
         std::uintptr_t shard_sumexp, std::uintptr_t shard_target, std::uintptr_t workspace,
         std::size_t workspace_bytes, std::uintptr_t status, std::uintptr_t stream) {
        int rc;
        {
          py::gil_scoped_release nogil;
          rc = nimble_tied_ce_forward(ptr<const void>(hidden), ptr<const void>(weights),
                                      ptr<const std::int64_t>(labels), n, d, v_local, v_offset, dtype,
                                      ptr<float>(shard_max), ptr<float>(shard_sumexp), ptr<float>(shard_target),
                                      ptr<void>(workspace), workspace_bytes, ptr<int>(status), ptr<void>(stream));
        }
        check(rc, "tied_ce_forward_device");
      },
      py::arg("hidden"), py::arg("weights"), py::arg("labels"), py::arg("n_tokens"), py::arg("d_model"),
      py::arg("v_local"), py::arg("v_offset"), py::arg("dtype"), py::arg("shard_max"), py::arg("shard_sumexp"),
      py::arg("shard_target"), py::arg("workspace"), py::arg("workspace_bytes"), py::arg("status"),
      py::arg("stream") = 0);

  // lse / loss over the merged shard statistics (fused_crossentropy.py:23-29).
  m.def(
      "tied_ce_combine_device",
      [](std::uintptr_t shard_max, std::uintptr_t shard_sumexp, std::uintptr_t shard_target, int n_shards,
         std::uintptr_t labels, std::int64_t n, std::int64_t vocab_size, std::int64_t ignore_index,
         std::uintptr_t out_max, std::uintptr_t out_sumexp, std::uintptr_t out_lse, std::uintptr_t out_loss,
         std::uintptr_t out_valid_count, std::uintptr_t status, std::uintptr_t stream) {
        int rc;
        {
          py::gil_scoped_release nogil;
          rc = nimble_tied_ce_combine(ptr<const float>(shard_max), ptr<const float>(shard_sumexp),
                                      ptr<const float>(shard_target), n_shards, ptr<const std::int64_t>(labels), n,
                                      vocab_size, ignore_index, ptr<float>(out_max), ptr<float>(out_sumexp),
                                      ptr<float>(out_lse), ptr<float>(out_loss), ptr<float>(out_valid_count),
                                      ptr<int>(status), ptr<void>(stream));
        }
        check(rc, "tied_ce_combine_device");
      },
      py::arg("shard_max"), py::arg("shard_sumexp"), py::arg("shard_target"), py::arg("n_shards"), py::arg("labels"),
      py::arg("n_tokens"), py::arg("vocab_size"), py::arg("ignore_index"), py::arg("out_max"), py::arg("out_sumexp"),
      py::arg("out_lse"), py::arg("out_loss"), py::arg("out_valid_count"), py::arg("status"), py::arg("stream") = 0);

  // Replaces fused_tied_crossentropy_backward (fused_tied_crossentropy.py:27-48).
  m.def(
      "tied_ce_backward_device",
      [](std::uintptr_t grad_scale, std::uintptr_t hidden, std::uintptr_t weights, std::uintptr_t labels,
         std::uintptr_t lse, std::uintptr_t valid_count, std::int64_t n, std::int64_t d, std::int64_t v_local,
         std::int64_t v_offset, std::int64_t ignore_index, int dtype, std::uintptr_t grad_hidden,
         int grad_hidden_dtype, std::uintptr_t grad_weights, int grad_weights_dtype, bool accumulate,
         std::size_t slab_bytes, std::uintptr_t workspace, std::size_t workspace_bytes, std::uintptr_t status,
         std::uintptr_t stream) {
        int rc;
        {
          py::gil_scoped_release nogil;
          rc = nimble_tied_ce_backward(ptr<const float>(grad_scale), ptr<const void>(hidden),
                                       ptr<const void>(weights), ptr<const std::int64_t>(labels),
                                       ptr<const float>(lse), ptr<const float>(valid_count), n, d, v_local, v_offset,
                                       ignore_index, dtype, ptr<void>(grad_hidden), grad_hidden_dtype,
                                       ptr<void>(grad_weights), grad_weights_dtype, accumulate ? 1 : 0, slab_bytes,
                                       ptr<void>(workspace), workspace_bytes, ptr<int>(status), ptr<void>(stream));
        }
        check(rc, "tied_ce_backward_device");
      },
      py::arg("grad_scale"), py::arg("hidden"), py::arg("weights"), py::arg("labels"), py::arg("lse"),
      py::arg("valid_count"), py::arg("n_tokens"), py::arg("d_model"), py::arg("v_local"), py::arg("v_offset"),
      py::arg("ignore_index"), py::arg("dtype"), py::arg("grad_hidden"), py::arg("grad_hidden_dtype"),
      py::arg("grad_weights"), py::arg("grad_weights_dtype"), py::arg("accumulate"), py::arg("slab_bytes"),
      py::arg("workspace"), py::arg("workspace_bytes"), py::arg("status"), py::arg("stream") = 0);
}
