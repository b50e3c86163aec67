// Registration hooks of the extension's op groups (each defined in its own .cu file and called
// once from bindings.cpp). Kept out of ops.h so adding an op group does not touch the header
// every kernel file includes.
#pragma once
#include <torch/extension.h>

namespace appcorr {
void register_elementwise_ops(pybind11::module_& m);
void register_attention_ops(pybind11::module_& m);
void register_comm_ops(pybind11::module_& m);
void register_sp_ops(pybind11::module_& m);
void register_msda_ops(pybind11::module_& m);
void register_conv_ops(pybind11::module_& m);
void register_attention_sm100_ops(pybind11::module_& m);
void register_pscore_sm100_ops(pybind11::module_& m);
void register_token_prune_ops(pybind11::module_& m);
}  // namespace appcorr
