// Python module of the tvarant extension (_C).
//
// Exposes the same functions as the reference's csrc/Module.cpp:32-57
// (is_available, device_count, current_device, set_device, synchronize,
// backend, device, manual_seed, get_rng_state, set_rng_state) plus streams,
// memory statistics, the device status word and NCCL communicators.
// Importing the module registers the backend name; it touches no GPU, so it
// also loads on a machine without one (is_available() is then False).
#include <ATen/core/Generator.h>
#include <c10/core/Device.h>
#include <c10/core/DeviceType.h>
#include <torch/extension.h>

#include <string>

#include "TvarantExt.h"

namespace tvarant {
std::string nccl_unique_id();
int64_t nccl_init(int64_t nranks, int64_t rank, const std::string& id, int64_t device,
                  int64_t max_ctas);
void nccl_destroy(int64_t handle, bool abort);
void all_gather(const at::Tensor& src, at::Tensor& dst, int64_t comm);
}  // namespace tvarant

namespace {

int resolve(int device) { return device < 0 ? tvarant::current_device() : device; }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  c10::register_privateuse1_backend("tvarant");

  m.def("is_available", []() { return tvarant::runtime_available(); });
  m.def("device_count", []() { return tvarant::device_count(); });
  m.def("current_device", []() { return tvarant::current_device(); });
  m.def("set_device", [](int index) { tvarant::set_device(index); });
  m.def("synchronize", [](int device) { TVR_TRY(tvr_device_synchronize(resolve(device))); },
        py::arg("device") = -1);
  m.def("backend", []() { return std::string(tvr_backend_name()); });
  m.def("device", []() {
    return c10::Device(c10::DeviceType::PrivateUse1,
                       static_cast<c10::DeviceIndex>(tvarant::current_device()));
  });
  m.def("manual_seed", [](int64_t seed, int device) {
    auto gen = tvarant::default_generator(static_cast<c10::DeviceIndex>(device));
    std::lock_guard<std::mutex> lock(gen.mutex());
    gen.set_current_seed(static_cast<uint64_t>(seed));
  }, py::arg("seed"), py::arg("device") = -1);
  m.def("get_rng_state", [](int device) {
    auto gen = tvarant::default_generator(static_cast<c10::DeviceIndex>(device));
    std::lock_guard<std::mutex> lock(gen.mutex());
    return gen.get_state();
  }, py::arg("device") = -1);
  m.def("set_rng_state", [](const at::Tensor& state, int device) {
    auto gen = tvarant::default_generator(static_cast<c10::DeviceIndex>(device));
    std::lock_guard<std::mutex> lock(gen.mutex());
    gen.set_state(state);
  }, py::arg("state"), py::arg("device") = -1);

  // streams: (device, id) pairs, id 0 = default stream
  m.def("current_stream", [](int device) {
    auto s = tvarant::current_stream(static_cast<c10::DeviceIndex>(device));
    return py::make_tuple(static_cast<int>(s.device_index()), static_cast<int64_t>(s.id()));
  }, py::arg("device") = -1);
  m.def("set_stream", [](int device, int64_t id) {
    tvarant::set_current_stream(c10::Stream(
        c10::Stream::UNSAFE,
        c10::Device(c10::DeviceType::PrivateUse1, static_cast<c10::DeviceIndex>(device)), id));
  });
  m.def("stream_handle", [](int device, int64_t id) {
    return reinterpret_cast<uintptr_t>(
        tvarant::stream_handle(static_cast<c10::DeviceIndex>(resolve(device)), id));
  });
  m.def("sm_count", [](int device) {
    int v = 0;
    TVR_TRY(tvr_device_sm_count(resolve(device), &v));
    return v;
  }, py::arg("device") = -1);
  m.def("set_gemm_sm_limit", [](int device, int max_sms) {
    TVR_TRY(tvr_set_gemm_sm_limit(resolve(device), max_sms));
  });
  m.def("gemm_sm_limit", [](int device) {
    int v = 0;
    TVR_TRY(tvr_get_gemm_sm_limit(resolve(device), &v));
    return v;
  });
  m.def("current_stream_handle",
        []() { return reinterpret_cast<uintptr_t>(tvarant::current_stream_handle()); });

  m.def("memory_stats", [](int device) {
    size_t reserved = 0, in_use = 0;
    TVR_TRY(tvr_memory_stats(resolve(device), &reserved, &in_use));
    return py::make_tuple(reserved, in_use);
  }, py::arg("device") = -1);
  m.def("empty_cache", [](int device) { TVR_TRY(tvr_empty_cache(resolve(device))); },
        py::arg("device") = -1);
  m.def("get_status", [](int device) {
    int code = 0;
    TVR_TRY(tvr_get_status(resolve(device), &code));
    return code;
  }, py::arg("device") = -1);
  m.def("clear_status", [](int device) { TVR_TRY(tvr_clear_status(resolve(device))); },
        py::arg("device") = -1);

  m.def("nccl_available", []() {
    int a = 0;
    TVR_TRY(tvr_nccl_available(&a));
    return a != 0;
  });
  m.def("nccl_unique_id", []() { return py::bytes(tvarant::nccl_unique_id()); });
  m.def("nccl_init", [](int64_t nranks, int64_t rank, py::bytes id, int device, int64_t max_ctas) {
    return tvarant::nccl_init(nranks, rank, std::string(id), resolve(device), max_ctas);
  }, py::arg("nranks"), py::arg("rank"), py::arg("unique_id"), py::arg("device") = -1,
     py::arg("max_ctas") = 0);
  m.def("nccl_destroy", &tvarant::nccl_destroy, py::arg("comm"), py::arg("abort") = false);
  m.def("all_gather", [](const at::Tensor& src, at::Tensor& dst, int64_t comm) {
    tvarant::all_gather(src, dst, comm);
  });
}
