// CUDA-core kernels of the engine (norms, routing, recurrent state updates, attention, sampling) and their
// torch bindings. Registered into the `_C` module by register_kernels().
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "kernels.h"

void register_fn(pybind11::module& m);
void register_ep(pybind11::module& m);
void register_train(pybind11::module& m);
void register_d3(pybind11::module& m);
void register_sample(pybind11::module& m);
void register_ple(pybind11::module& m);
void register_gemv(pybind11::module& m);
void register_tp(pybind11::module& m);
void register_mla(pybind11::module& m);
void register_dsa(pybind11::module& m);
void register_f8gemm(pybind11::module& m);
void register_moe_i8(pybind11::module& m);
void register_gdn_chunk(pybind11::module& m);

void register_kernels(pybind11::module& m) {
  register_fn(m);
  register_ep(m);
  register_train(m);
  register_d3(m);
  register_sample(m);
  register_ple(m);
  register_gemv(m);
  register_tp(m);
  register_mla(m);
  register_dsa(m);
  register_f8gemm(m);
  register_moe_i8(m);
  register_gdn_chunk(m);
}
