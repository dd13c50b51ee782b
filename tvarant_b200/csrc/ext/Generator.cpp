// Generators of the tvarant device.
//
// As in the reference (csrc/runtime/Generator.cpp:7-33) a tvarant generator
// is a CPU Philox/MT generator tagged with the PrivateUse1 device: random
// tensors are drawn on the host and copied to the GPU, so a seeded
// torch.randn(..., device="tvarant") reproduces the CPU stream exactly.
// Unlike the reference there is one default generator per GPU.
#include <ATen/CPUGeneratorImpl.h>

#include <deque>
#include <mutex>

#include "TvarantExt.h"

namespace tvarant {
namespace {

class TvarantGenerator final : public at::CPUGeneratorImpl {
 public:
  explicit TvarantGenerator(c10::DeviceIndex device) {
    device_ = c10::Device(c10::DeviceType::PrivateUse1, device);
    key_set_ = c10::DispatchKeySet(c10::DispatchKey::PrivateUse1);
  }
};

std::once_flag g_once;
std::deque<at::Generator> g_defaults;

}  // namespace

const at::Generator& default_generator(c10::DeviceIndex device) {
  std::call_once(g_once, []() {
    const int n = device_count() > 0 ? device_count() : 1;
    for (int d = 0; d < n; ++d) {
      g_defaults.push_back(at::make_generator<TvarantGenerator>(static_cast<c10::DeviceIndex>(d)));
      g_defaults.back().seed();
    }
  });
  if (device < 0) device = static_cast<c10::DeviceIndex>(runtime_available() ? current_device() : 0);
  TORCH_CHECK(device < static_cast<c10::DeviceIndex>(g_defaults.size()),
              "tvarant generator: device index out of range: ", device);
  return g_defaults[device];
}

at::Generator make_generator(c10::DeviceIndex device) {
  if (device < 0) device = static_cast<c10::DeviceIndex>(current_device());
  return at::make_generator<TvarantGenerator>(device);
}

}  // namespace tvarant
