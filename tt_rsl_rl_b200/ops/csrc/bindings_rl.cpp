// Python bindings of the RL kernels (rollout, GAE, gather, loss, optimizer, normalizer).
#include "kernels.cuh"

void rlb_register_kernels(pybind11::module& m) { (void)m; }
