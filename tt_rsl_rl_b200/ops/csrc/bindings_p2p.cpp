// Bindings of the inter-process buffer sharing (CUDA IPC) and the peer-to-peer collectives.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <string>

#include "p2p.cuh"

namespace {

using torch::Tensor;

void ok(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e)); }

// A zero-initialised device buffer from cudaMalloc (so that its IPC handle covers exactly this allocation).
Tensor ipc_alloc(int64_t nbytes, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  ok(cudaMalloc(&p, static_cast<size_t>(nbytes)), "cudaMalloc");
  ok(cudaMemset(p, 0, static_cast<size_t>(nbytes)), "cudaMemset");
  auto opts = torch::dtype(torch::kUInt8).device(torch::kCUDA, static_cast<c10::DeviceIndex>(device));
  return torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

pybind11::bytes ipc_handle(const Tensor& t) {
  cudaIpcMemHandle_t h;
  ok(cudaIpcGetMemHandle(&h, t.data_ptr()), "cudaIpcGetMemHandle");
  return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(const std::string& handle, int64_t device) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

rlb::P2PArgs make_args(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t rank,
                       const Tensor& epoch, int64_t timeout_ns, const c10::optional<Tensor>& status) {
  TORCH_CHECK(bufs.size() == flags.size() && !bufs.empty() && bufs.size() <= rlb::kMaxWorld, "p2p: world size");
  rlb::P2PArgs a{};
  a.world = static_cast<int>(bufs.size());
  a.rank = static_cast<int>(rank);
  for (size_t r = 0; r < bufs.size(); ++r) {
    a.peer_buf[r] = reinterpret_cast<const void*>(bufs[r]);
    a.peer_flags[r] = reinterpret_cast<unsigned int*>(flags[r]);
  }
  a.epoch = reinterpret_cast<unsigned int*>(epoch.data_ptr());
  a.timeout_ns = static_cast<uint64_t>(timeout_ns);
  a.status = (status.has_value() && status->defined()) ? reinterpret_cast<unsigned int*>(status->data_ptr()) : nullptr;
  return a;
}

void p2p_allreduce_f64(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t rank,
                       const Tensor& epoch, int64_t timeout_ns, const c10::optional<Tensor>& status, const Tensor& out,
                       int64_t n) {
  TORCH_CHECK(out.scalar_type() == torch::kFloat64 && out.numel() >= n, "p2p_allreduce_f64: out");
  ok(rlb::p2p_allreduce_f64(make_args(bufs, flags, rank, epoch, timeout_ns, status), out.data_ptr<double>(), n,
                            at::cuda::getCurrentCUDAStream()),
     "p2p_allreduce_f64");
}

void p2p_broadcast_f32(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t rank,
                       const Tensor& epoch, int64_t timeout_ns, const c10::optional<Tensor>& status, int64_t root,
                       const Tensor& dst, int64_t n) {
  TORCH_CHECK(dst.scalar_type() == torch::kFloat32 && dst.numel() >= n, "p2p_broadcast_f32: dst");
  ok(rlb::p2p_broadcast_f32(make_args(bufs, flags, rank, epoch, timeout_ns, status), static_cast<int>(root),
                            dst.data_ptr<float>(), n, at::cuda::getCurrentCUDAStream()),
     "p2p_broadcast_f32");
}

}  // namespace

void rlb_register_p2p(pybind11::module& m) {
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("p2p_allreduce_f64", &p2p_allreduce_f64);
  m.def("p2p_broadcast_f32", &p2p_broadcast_f32);
}
