// DeviceGuardImplInterface of the tvarant device: device switching, streams
// and events.
//
// The reference's guard (csrc/runtime/Guard.cpp:10-79) reports a single
// DEFAULT stream and synchronises the whole runtime for every stream
// operation.  Here streams are real CUDA streams (Runtime.cpp) and events
// are CUDA events, so torch.Stream / torch.Event and record_stream work on
// device "tvarant".
#include <c10/core/impl/DeviceGuardImplInterface.h>

#include "TvarantExt.h"

namespace tvarant {

struct GuardImpl final : public c10::impl::DeviceGuardImplInterface {
  static constexpr c10::DeviceType static_type = c10::DeviceType::PrivateUse1;

  GuardImpl() = default;
  explicit GuardImpl(c10::DeviceType t) {
    TORCH_CHECK(t == static_type, "tvarant guard got device type ", t);
  }

  c10::DeviceType type() const override { return static_type; }

  c10::Device exchangeDevice(c10::Device d) const override {
    TORCH_CHECK(d.is_privateuseone(), "Expected tvarant device, got ", d);
    const int prev = exchange_device(d.index());
    return c10::Device(static_type, static_cast<c10::DeviceIndex>(prev));
  }

  c10::Device getDevice() const override {
    return c10::Device(static_type, static_cast<c10::DeviceIndex>(current_device()));
  }

  void setDevice(c10::Device d) const override {
    TORCH_CHECK(d.is_privateuseone(), "Expected tvarant device, got ", d);
    set_device(d.index());
  }

  void uncheckedSetDevice(c10::Device d) const noexcept override {
    if (d.is_privateuseone() && d.index() >= 0 && d.index() < device_count()) {
      tvr_set_device(d.index());
    }
  }

  c10::Stream getStream(c10::Device d) const override { return current_stream(d.index()); }

  c10::Stream getDefaultStream(c10::Device d) const override {
    return c10::Stream(c10::Stream::DEFAULT, d);
  }

  c10::Stream getNewStream(c10::Device d, int priority = 0) const override {
    return stream_from_pool(d.index(), priority < 0);
  }

  c10::Stream getStreamFromGlobalPool(c10::Device d, bool high_priority = false) const override {
    return stream_from_pool(d.index(), high_priority);
  }

  c10::Stream exchangeStream(c10::Stream s) const override {
    c10::Stream prev = current_stream(s.device_index());
    set_current_stream(s);
    return prev;
  }

  c10::DeviceIndex deviceCount() const noexcept override {
    return static_cast<c10::DeviceIndex>(device_count());
  }

  bool queryStream(const c10::Stream& s) const override {
    int done = 0;
    TVR_TRY(tvr_stream_query(stream_handle(s.device_index(), s.id()), &done));
    return done != 0;
  }

  void synchronizeStream(const c10::Stream& s) const override {
    TVR_TRY(tvr_stream_synchronize(stream_handle(s.device_index(), s.id())));
  }

  void synchronizeDevice(const c10::DeviceIndex device_index) const override {
    TVR_TRY(tvr_device_synchronize(device_index < 0 ? current_device() : device_index));
  }

  void record(void** event, const c10::Stream& s, const c10::DeviceIndex device_index,
              const c10::EventFlag flag) const override {
    TORCH_CHECK(device_index == -1 || device_index == s.device_index(),
                "event device ", device_index, " does not match stream device ",
                s.device_index());
    const int prev = exchange_device(s.device_index());
    if (*event == nullptr) {
      // as for CUDA: BACKEND_DEFAULT records timing, PYTORCH_DEFAULT does not
      TVR_TRY(tvr_event_create(event, flag == c10::EventFlag::BACKEND_DEFAULT ? 1 : 0));
    }
    TVR_TRY(tvr_event_record(*event, stream_handle(s.device_index(), s.id())));
    if (prev != s.device_index()) set_device(prev);
  }

  void block(void* event, const c10::Stream& s) const override {
    if (event == nullptr) return;
    TVR_TRY(tvr_stream_wait_event(stream_handle(s.device_index(), s.id()), event));
  }

  bool queryEvent(void* event) const override {
    if (event == nullptr) return true;
    int done = 0;
    TVR_TRY(tvr_event_query(event, &done));
    return done != 0;
  }

  void destroyEvent(void* event, const c10::DeviceIndex /*device_index*/) const noexcept override {
    if (event != nullptr) tvr_event_destroy(event);
  }

  void synchronizeEvent(void* event) const override {
    if (event != nullptr) TVR_TRY(tvr_event_synchronize(event));
  }

  double elapsedTime(void* start, void* end, const c10::DeviceIndex /*device_index*/) const override {
    TORCH_CHECK(start != nullptr && end != nullptr, "elapsedTime: both events must be recorded");
    float ms = 0.f;
    TVR_TRY(tvr_event_elapsed_ms(start, end, &ms));
    return static_cast<double>(ms);
  }

  void recordDataPtrOnStream(const c10::DataPtr& data_ptr, const c10::Stream& s) const override {
    if (data_ptr.get() == nullptr) return;
    TVR_TRY(tvr_record_stream(data_ptr.get(), stream_handle(s.device_index(), s.id())));
  }
};

}  // namespace tvarant

C10_REGISTER_GUARD_IMPL(PrivateUse1, tvarant::GuardImpl);
