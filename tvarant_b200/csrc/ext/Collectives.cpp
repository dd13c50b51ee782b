// NCCL communicators for tensor-parallel use of the tvarant device (the
// reference has one device and no collectives).
//
// A communicator is created from NCCL's 128-byte unique id, exchanged by
// the caller (torch.distributed over gloo/TCPStore, or a file); handles are
// small integers so they can travel through the dispatcher as `int comm`.
// tvarant::all_reduce_(t, comm) sums a float32 tensor in place across the
// ranks of `comm` on the current stream.
#include <ATen/ATen.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include <mutex>
#include <string>
#include <vector>

#include "TvarantExt.h"

namespace tvarant {
namespace {

std::mutex g_comm_mutex;
std::vector<void*> g_comms;  // handle -> ncclComm_t (nullptr once destroyed)

void* comm_of(int64_t handle) {
  std::lock_guard<std::mutex> lock(g_comm_mutex);
  TORCH_CHECK(handle >= 0 && handle < static_cast<int64_t>(g_comms.size()) &&
                  g_comms[handle] != nullptr,
              "tvarant: unknown or destroyed communicator ", handle);
  return g_comms[handle];
}

at::Tensor& all_reduce_(at::Tensor& self, int64_t comm) {
  TORCH_CHECK(self.device().is_privateuseone(), "all_reduce_: expected a tvarant tensor");
  ops::check_fp32(self, "all_reduce_");
  TORCH_CHECK(self.is_contiguous(), "all_reduce_: tensor must be contiguous");
  c10::DeviceGuard guard(self.device());
  TVR_TRY(tvr_nccl_all_reduce(self.data_ptr(), self.data_ptr(), self.numel(), 0, 0,
                              comm_of(comm), current_stream_handle()));
  return self;
}

}  // namespace

std::string nccl_unique_id() {
  std::string id(128, '\0');
  TVR_TRY(tvr_nccl_get_unique_id(&id[0]));
  return id;
}

int64_t nccl_init(int64_t nranks, int64_t rank, const std::string& id, int64_t device,
                  int64_t max_ctas) {
  TORCH_CHECK(id.size() == 128, "nccl_init: unique id must be 128 bytes");
  void* comm = nullptr;
  TVR_TRY(tvr_nccl_comm_init_ctas(&comm, static_cast<int>(nranks), id.data(),
                                  static_cast<int>(rank), static_cast<int>(device),
                                  static_cast<int>(max_ctas)));
  std::lock_guard<std::mutex> lock(g_comm_mutex);
  g_comms.push_back(comm);
  return static_cast<int64_t>(g_comms.size() - 1);
}

void nccl_destroy(int64_t handle, bool abort) {
  void* comm = comm_of(handle);
  TVR_TRY(abort ? tvr_nccl_comm_abort(comm) : tvr_nccl_comm_destroy(comm));
  std::lock_guard<std::mutex> lock(g_comm_mutex);
  g_comms[handle] = nullptr;
}

void all_gather(const at::Tensor& src, at::Tensor& dst, int64_t comm) {
  ops::check_fp32(src, "all_gather");
  ops::check_fp32(dst, "all_gather");
  TORCH_CHECK(src.is_contiguous() && dst.is_contiguous(), "all_gather: tensors must be contiguous");
  c10::DeviceGuard guard(src.device());
  TVR_TRY(tvr_nccl_all_gather(src.data_ptr(), dst.data_ptr(), src.numel(), 0, comm_of(comm),
                              current_stream_handle()));
}

}  // namespace tvarant

TORCH_LIBRARY_IMPL(tvarant, PrivateUse1, m) {
  m.impl("all_reduce_", TORCH_FN(tvarant::all_reduce_));
}
