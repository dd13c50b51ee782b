// PrivateUse1 hooks of the tvarant device.
//
// Counterpart of csrc/runtime/Hooks.cpp in the reference (availability,
// device count and switching, getDeviceFromPtr, generators, storage resize),
// backed by the CUDA runtime; the pinned-memory allocator hands out
// page-locked host memory (tvr_host_alloc) so non_blocking host<->device
// copies are asynchronous.
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <c10/core/Allocator.h>
#include <c10/core/CPUAllocator.h>
#include <c10/core/Storage.h>

#include <algorithm>

#include "TvarantExt.h"

namespace tvarant {
namespace {

void free_pinned(void* p) {
  if (p != nullptr) tvr_host_free(p);
}

class PinnedAllocator final : public c10::Allocator {
 public:
  c10::DataPtr allocate(size_t nbytes) override {
    void* p = nullptr;
    if (nbytes > 0) TVR_TRY(tvr_host_alloc(&p, nbytes));
    return {p, p, &free_pinned, c10::Device(c10::DeviceType::CPU)};
  }
  c10::DeleterFnPtr raw_deleter() const override { return &free_pinned; }
  void copy_data(void* dest, const void* src, std::size_t count) const override {
    std::memcpy(dest, src, count);
  }
};

PinnedAllocator g_pinned;

struct Hooks final : public at::PrivateUse1HooksInterface {
  ~Hooks() override = default;

  bool isBuilt() const override { return true; }
  bool isAvailable() const override { return runtime_available(); }
  bool hasPrimaryContext(c10::DeviceIndex /*device_index*/) const override { return true; }
  void init() const override { runtime_available(); }

  c10::DeviceIndex deviceCount() const override {
    return static_cast<c10::DeviceIndex>(device_count());
  }
  void setCurrentDevice(c10::DeviceIndex device) const override { set_device(device); }
  c10::DeviceIndex getCurrentDevice() const override {
    return static_cast<c10::DeviceIndex>(current_device());
  }
  c10::DeviceIndex exchangeDevice(c10::DeviceIndex device) const override {
    return static_cast<c10::DeviceIndex>(exchange_device(device));
  }
  c10::DeviceIndex maybeExchangeDevice(c10::DeviceIndex device) const override {
    if (device < 0 || device >= device_count()) return getCurrentDevice();
    return exchangeDevice(device);
  }

  at::Device getDeviceFromPtr(void* data) const override {
    int dev = -1;
    TVR_TRY(tvr_pointer_device(data, &dev));
    TORCH_CHECK(dev >= 0, "Pointer is not a Tvarant allocation");
    return at::Device(at::DeviceType::PrivateUse1, static_cast<c10::DeviceIndex>(dev));
  }

  bool isPinnedPtr(const void* data) const override {
    int pinned = 0;
    return tvr_is_pinned(data, &pinned) == TVR_OK && pinned != 0;
  }
  at::Allocator* getPinnedMemoryAllocator() const override { return &g_pinned; }

  const at::Generator& getDefaultGenerator(c10::DeviceIndex device_index) const override {
    return default_generator(device_index);
  }
  at::Generator getNewGenerator(c10::DeviceIndex device_index) const override {
    return make_generator(device_index);
  }

  void resizePrivateUse1Bytes(const c10::Storage& storage, size_t newsize) const override {
    auto* impl = storage.unsafeGetStorageImpl();
    TORCH_CHECK(impl->resizable(), "Trying to resize storage that is not resizable");
    if (newsize == 0) {
      impl->set_data_ptr_noswap(allocator()->allocate(0));
      impl->set_nbytes(0);
      return;
    }
    at::DataPtr fresh = allocator()->allocate(newsize);
    const size_t keep = std::min(impl->nbytes(), newsize);
    if (keep > 0 && impl->data() != nullptr) {
      TVR_TRY(tvr_memcpy_d2d(fresh.get(), impl->data(), keep, current_stream_handle()));
    }
    impl->set_data_ptr_noswap(std::move(fresh));
    impl->set_nbytes(newsize);
  }
};

}  // namespace
}  // namespace tvarant

namespace {
static bool g_hooks_registered [[maybe_unused]] = []() {
  at::RegisterPrivateUse1HooksInterface(new tvarant::Hooks());
  return true;
}();
}  // namespace
