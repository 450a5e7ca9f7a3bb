// Peer-memory plumbing: device buffers shareable across processes with CUDA
// IPC handles, mapped into every rank of an AFD world (NVLink / NVSwitch).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/library.h>

#include <cstring>

namespace {

void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, "afd_b200 ", what, " failed: ", cudaGetErrorString(e));
}

// Zero-filled device buffer owned by this process (cudaMalloc, so the whole
// allocation can be exported as one IPC handle).
at::Tensor ipc_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  check(cudaMalloc(&p, (size_t)nbytes), "cudaMalloc");
  check(cudaMemset(p, 0, (size_t)nbytes), "cudaMemset");
  check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  return at::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

at::Tensor ipc_handle(const at::Tensor& buf) {
  cudaIpcMemHandle_t h;
  c10::cuda::CUDAGuard g(buf.device());
  check(cudaIpcGetMemHandle(&h, buf.data_ptr()), "cudaIpcGetMemHandle");
  auto out = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

int64_t ipc_open(const at::Tensor& handle, int64_t device) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  check(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

bool can_access_peer(int64_t device, int64_t peer) {
  int ok = 0;
  check(cudaDeviceCanAccessPeer(&ok, (int)device, (int)peer), "cudaDeviceCanAccessPeer");
  return ok != 0;
}

}  // namespace

TORCH_LIBRARY_FRAGMENT(afd_b200, m) {
  m.def("ipc_alloc(int nbytes, int device) -> Tensor");
  m.def("ipc_handle(Tensor buf) -> Tensor");
  m.def("ipc_open(Tensor handle, int device) -> int");
  m.def("ipc_close(int ptr, int device) -> ()");
  m.def("can_access_peer(int device, int peer) -> bool");
}

TORCH_LIBRARY_IMPL(afd_b200, CompositeExplicitAutograd, m) {
  m.impl("ipc_alloc", &ipc_alloc);
  m.impl("ipc_handle", &ipc_handle);
  m.impl("ipc_open", &ipc_open);
  m.impl("ipc_close", &ipc_close);
  m.impl("can_access_peer", &can_access_peer);
}
