// Registration hook for the RL kernels' Python bindings (implemented in bindings_rl.cpp).
#pragma once
#include <torch/extension.h>

void rlb_register_kernels(pybind11::module& m);
void rlb_register_p2p(pybind11::module& m);
void rlb_register_rnn(pybind11::module& m);
