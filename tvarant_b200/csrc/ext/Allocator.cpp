// c10::Allocator for the tvarant device.
//
// Replaces csrc/runtime/Allocator.cpp of the reference, which forwards to
// the simulator's posix_memalign allocator.  Here allocation is
// stream-ordered: a block is taken from the device's caching pool on the
// current stream (tvr_malloc) and returned to it on that same stream when
// the storage dies (tvr_free); uses on other streams are covered by
// record_stream (Guard.cpp).
#include <c10/core/Allocator.h>
#include <c10/core/Device.h>
#include <c10/core/DeviceType.h>

#include "TvarantExt.h"

namespace tvarant {
namespace {

void delete_block(void* ptr) {
  if (ptr != nullptr) {
    // A deleter must not throw; a failed free is only reported.
    if (tvr_free(ptr) != TVR_OK) {
      TORCH_WARN("tvarant: freeing ", ptr, " failed: ", tvr_last_error());
    }
  }
}

class DeviceAllocator final : public c10::Allocator {
 public:
  c10::DataPtr allocate(size_t nbytes) override {
    const int dev = current_device();
    void* data = nullptr;
    if (nbytes > 0) {
      TVR_TRY(tvr_malloc(&data, nbytes, dev, current_stream_handle()));
    }
    return {data, data, &delete_block,
            c10::Device(c10::DeviceType::PrivateUse1, static_cast<c10::DeviceIndex>(dev))};
  }

  c10::DeleterFnPtr raw_deleter() const override { return &delete_block; }

  void copy_data(void* dest, const void* src, std::size_t count) const override {
    TVR_TRY(tvr_memcpy_d2d(dest, src, count, current_stream_handle()));
  }
};

DeviceAllocator g_allocator;

}  // namespace

c10::Allocator* allocator() { return &g_allocator; }

}  // namespace tvarant

namespace {
static c10::AllocatorRegisterer<c10::DeviceType::PrivateUse1> g_register(&tvarant::g_allocator);
}  // namespace
