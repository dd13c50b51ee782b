// Devices and streams of the tvarant backend.
//
// Replaces csrc/runtime/Runtime.cpp of the reference (backend selection from
// TVARANT_BACKEND, a thread-local current device fixed to index 0,
// kDeviceCount = 1): here the device count is the number of visible GPUs,
// the current device is CUDA's per-thread current device, and each device
// has real streams — the legacy default stream plus a pool of non-blocking
// streams — with a thread-local current stream per device.
#include <array>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>

#include "TvarantExt.h"

namespace tvarant {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kPoolSize = 32;

std::once_flag g_init_once;
int g_device_count = 0;
bool g_available = false;
std::string g_init_error;

struct Pool {
  std::once_flag once;
  std::array<void*, kPoolSize> streams{};
  std::array<void*, kPoolSize> high{};
  std::atomic<unsigned> next{0};
  std::atomic<unsigned> next_high{0};
};
Pool g_pools[kMaxDevices];

// current stream id per device, per thread (0 = default stream)
thread_local std::array<c10::StreamId, kMaxDevices> t_current{};

void init_once() {
  std::call_once(g_init_once, []() {
    const char* env = std::getenv("TVARANT_BACKEND");
    if (env != nullptr && env[0] != '\0' && std::string(env) != "cuda") {
      g_init_error = std::string("TVARANT_BACKEND=") + env +
                     " is not available in this package (expected 'cuda'; the CPU simulator "
                     "and OpenCL runtimes are replaced by the B200 CUDA runtime)";
      return;
    }
    if (tvr_init() != TVR_OK) {
      g_init_error = tvr_last_error();
      return;
    }
    int n = 0;
    if (tvr_device_count(&n) == TVR_OK && n > 0) {
      g_device_count = n < kMaxDevices ? n : kMaxDevices;
      g_available = true;
    } else {
      g_init_error = "no CUDA device is visible";
    }
  });
}

// Pool stream ids: 1..kPoolSize normal priority, kPoolSize+1..2*kPoolSize high.
void create_pool(int device) {
  Pool& p = g_pools[device];
  std::call_once(p.once, [&]() {
    for (int i = 0; i < kPoolSize; ++i) {
      TVR_TRY(tvr_stream_create(&p.streams[i], device, 0));
      TVR_TRY(tvr_stream_create(&p.high[i], device, -1));
    }
  });
}

}  // namespace

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == TVR_OK, "tvarant: ", what, " failed: ", tvr_last_error());
}

bool runtime_available() {
  init_once();
  return g_available;
}

int device_count() {
  init_once();
  return g_device_count;
}

static void require_runtime() {
  init_once();
  TORCH_CHECK(g_available, "tvarant device unavailable: ", g_init_error);
}

int current_device() {
  require_runtime();
  int d = 0;
  TVR_TRY(tvr_get_device(&d));
  return d;
}

void set_device(int index) {
  require_runtime();
  TORCH_CHECK(index >= 0 && index < g_device_count, "Tvarant device index out of range: ", index,
              " (device count ", g_device_count, ")");
  TVR_TRY(tvr_set_device(index));
}

int exchange_device(int index) {
  const int prev = current_device();
  if (index != prev) set_device(index);
  return prev;
}

void* stream_handle(c10::DeviceIndex device, c10::StreamId id) {
  if (id == 0) return nullptr;
  TORCH_CHECK(device >= 0 && device < g_device_count, "bad tvarant stream device ", device);
  create_pool(device);
  Pool& p = g_pools[device];
  if (id >= 1 && id <= kPoolSize) return p.streams[id - 1];
  if (id > kPoolSize && id <= 2 * kPoolSize) return p.high[id - kPoolSize - 1];
  TORCH_CHECK(false, "unknown tvarant stream id ", id);
}

c10::Stream current_stream(c10::DeviceIndex device) {
  if (device < 0) device = static_cast<c10::DeviceIndex>(current_device());
  return c10::Stream(c10::Stream::UNSAFE, c10::Device(c10::DeviceType::PrivateUse1, device),
                     t_current[device]);
}

void set_current_stream(const c10::Stream& stream) {
  TORCH_CHECK(stream.device_type() == c10::DeviceType::PrivateUse1,
              "expected a tvarant stream, got ", stream);
  t_current[stream.device_index()] = stream.id();
}

c10::Stream stream_from_pool(c10::DeviceIndex device, bool high_priority) {
  if (device < 0) device = static_cast<c10::DeviceIndex>(current_device());
  create_pool(device);
  Pool& p = g_pools[device];
  c10::StreamId id;
  if (high_priority) {
    id = kPoolSize + 1 + static_cast<c10::StreamId>(p.next_high++ % kPoolSize);
  } else {
    id = 1 + static_cast<c10::StreamId>(p.next++ % kPoolSize);
  }
  return c10::Stream(c10::Stream::UNSAFE, c10::Device(c10::DeviceType::PrivateUse1, device), id);
}

void* current_stream_handle() {
  const int d = current_device();
  return stream_handle(static_cast<c10::DeviceIndex>(d), t_current[d]);
}

}  // namespace tvarant
