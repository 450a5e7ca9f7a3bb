// NCCL point-to-point on the caller's current CUDA stream (graph-capturable).
//
// torch.distributed's NCCL send/recv run on the process group's internal
// streams and synchronise through events, which a CUDA graph capture of a
// decode step does not take; ncclSend / ncclRecv issued straight onto the
// capturing stream become graph nodes and replay with it.  This is what the
// baseline NCCL connector uses on GPUs (one communicator per AFD subgroup,
// created from a unique id that the subgroup's first rank shares over gloo).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <nccl.h>
#include <torch/library.h>

#include <cstring>

namespace {

ncclComm_t as_comm(int64_t h) { return reinterpret_cast<ncclComm_t>(static_cast<intptr_t>(h)); }

void check(ncclResult_t r, const char* what) {
  TORCH_CHECK(r == ncclSuccess, what, " failed: ", ncclGetErrorString(r));
}

ncclDataType_t nccl_type(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return ncclBfloat16;
    case at::kHalf: return ncclFloat16;
    case at::kFloat: return ncclFloat32;
    case at::kInt: return ncclInt32;
    case at::kLong: return ncclInt64;
    case at::kByte: return ncclUint8;
    default: TORCH_CHECK(false, "nccl_p2p: unsupported dtype ", t.scalar_type());
  }
  return ncclUint8;
}

}  // namespace

// 128-byte unique id as a CPU uint8 tensor (to share over a host group).
at::Tensor nccl_unique_id() {
  ncclUniqueId id;
  check(ncclGetUniqueId(&id), "ncclGetUniqueId");
  auto t = at::empty({(int64_t)sizeof(id)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(t.data_ptr(), &id, sizeof(id));
  return t;
}

// Communicator of `nranks` ranks on the current device; returns an opaque handle.
int64_t nccl_comm_init(const at::Tensor& uid, int64_t nranks, int64_t rank) {
  TORCH_CHECK(uid.device().is_cpu() && uid.scalar_type() == at::kByte && uid.numel() == (int64_t)sizeof(ncclUniqueId),
              "nccl_comm_init: the 128-byte unique id as a CPU uint8 tensor");
  ncclUniqueId id;
  std::memcpy(&id, uid.data_ptr(), sizeof(id));
  ncclComm_t comm = nullptr;
  check(ncclCommInitRank(&comm, (int)nranks, id, (int)rank), "ncclCommInitRank");
  return static_cast<int64_t>(reinterpret_cast<intptr_t>(comm));
}

void nccl_comm_destroy(int64_t comm) {
  if (comm) check(ncclCommDestroy(as_comm(comm)), "ncclCommDestroy");
}

void nccl_send(const at::Tensor& t, int64_t peer, int64_t comm) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "nccl_send: contiguous CUDA tensor");
  c10::cuda::CUDAGuard g(t.device());
  check(ncclSend(t.data_ptr(), (size_t)t.numel(), nccl_type(t), (int)peer, as_comm(comm),
                 at::cuda::getCurrentCUDAStream().stream()),
        "ncclSend");
}

void nccl_recv(at::Tensor& t, int64_t peer, int64_t comm) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "nccl_recv: contiguous CUDA tensor");
  c10::cuda::CUDAGuard g(t.device());
  check(ncclRecv(t.data_ptr(), (size_t)t.numel(), nccl_type(t), (int)peer, as_comm(comm),
                 at::cuda::getCurrentCUDAStream().stream()),
        "ncclRecv");
}

void nccl_group_start() { check(ncclGroupStart(), "ncclGroupStart"); }
void nccl_group_end() { check(ncclGroupEnd(), "ncclGroupEnd"); }

TORCH_LIBRARY_FRAGMENT(afd_b200, m) {
  m.def("nccl_unique_id() -> Tensor");
  m.def("nccl_comm_init(Tensor uid, int nranks, int rank) -> int");
  m.def("nccl_comm_destroy(int comm) -> ()");
  m.def("nccl_send(Tensor t, int peer, int comm) -> ()");
  m.def("nccl_recv(Tensor(a!) t, int peer, int comm) -> ()");
  m.def("nccl_group_start() -> ()");
  m.def("nccl_group_end() -> ()");
}

TORCH_LIBRARY_IMPL(afd_b200, CompositeExplicitAutograd, m) {
  m.impl("nccl_unique_id", &nccl_unique_id);
  m.impl("nccl_comm_init", &nccl_comm_init);
  m.impl("nccl_comm_destroy", &nccl_comm_destroy);
  m.impl("nccl_group_start", &nccl_group_start);
  m.impl("nccl_group_end", &nccl_group_end);
}

TORCH_LIBRARY_IMPL(afd_b200, CUDA, m) {
  m.impl("nccl_send", &nccl_send);
  m.impl("nccl_recv", &nccl_recv);
}
