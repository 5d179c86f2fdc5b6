// Registration hooks for the kernel groups bound outside kernels_module.cpp.
#pragma once
#include <pybind11/pybind11.h>

namespace hk {
void register_more_kernels(pybind11::module_& m);
void register_tp_kernels(pybind11::module_& m);
void register_model_kernels(pybind11::module_& m);
void register_mg_kernels(pybind11::module_& m);
void register_ds_kernels(pybind11::module_& m);
}  // namespace hk
