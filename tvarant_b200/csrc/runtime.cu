// Device runtime of the tvarant backend: devices, stream-ordered caching
// allocation, pinned host memory, copies, streams, events and the device
// status word.
//
// Replaces the reference's runtime layer (csrc/runtime/TvarantRuntime.h:37-61,
// csrc/runtime/Runtime.cpp, csrc/runtime/CpuSimRuntime.cpp:49-240): there the
// "device" is posix_memalign'd host memory tracked in a mutex-guarded set and
// every copy is a memcpy.  Here memory comes from the CUDA stream-ordered
// pool of each device (cudaMallocAsync), configured to keep freed blocks, so
// allocation and free are queued on a stream like the kernels that use them.
#include "internal.h"

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace tvr {

namespace {

thread_local std::string t_last_error;

constexpr int kMaxDevices = 64;

std::once_flag g_init_once;
int g_init_status = TVR_OK;
std::string g_init_error;
int g_device_count = 0;
int g_sm_count[kMaxDevices] = {0};
int* g_status_words[kMaxDevices] = {nullptr};
std::once_flag g_device_once[kMaxDevices];
int g_device_init_status[kMaxDevices] = {0};

DriverApi g_driver;
bool g_driver_ok = false;

struct AllocInfo {
  int device;
  size_t nbytes;
  cudaStream_t stream;
  std::vector<cudaEvent_t> uses;  // record_stream events to wait for before free
};

std::mutex g_alloc_mutex;
std::unordered_map<void*, AllocInfo> g_allocs;
size_t g_in_use[kMaxDevices] = {0};

std::mutex g_host_mutex;
std::unordered_map<void*, size_t> g_host_allocs;

template <typename Fn>
bool resolve(const char* name, Fn* fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr) {
    return false;
  }
  *fn = reinterpret_cast<Fn>(p);
  return true;
}

void do_init() {
  cudaError_t e = cudaGetDeviceCount(&g_device_count);
  if (e != cudaSuccess) {
    g_device_count = 0;
    g_init_status = TVR_ERR_CUDA;
    g_init_error = std::string("no CUDA device: ") + cudaGetErrorString(e);
    cudaGetLastError();
    return;
  }
  if (g_device_count > kMaxDevices) g_device_count = kMaxDevices;
  for (int d = 0; d < g_device_count; ++d) {
    cudaDeviceGetAttribute(&g_sm_count[d], cudaDevAttrMultiProcessorCount, d);
  }
  bool ok = true;
  ok &= resolve("cuTensorMapEncodeTiled", &g_driver.tensorMapEncodeTiled);
  ok &= resolve("cuModuleLoadData", &g_driver.moduleLoadData);
  ok &= resolve("cuModuleGetFunction", &g_driver.moduleGetFunction);
  ok &= resolve("cuLaunchKernel", &g_driver.launchKernel);
  ok &= resolve("cuGetErrorString", &g_driver.getErrorString);
  ok &= resolve("cuCtxGetCurrent", &g_driver.ctxGetCurrent);
  g_driver_ok = ok;
}

// First use of a device on any thread: status word, pool configuration.
int init_device(int device) {
  std::call_once(g_device_once[device], [device]() {
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
      g_device_init_status[device] = TVR_ERR_CUDA;
      cudaGetLastError();
      return;
    }
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      uint64_t threshold = UINT64_MAX;  // keep freed blocks cached
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    int* status = nullptr;
    if (cudaMalloc(&status, sizeof(int)) != cudaSuccess ||
        cudaMemset(status, 0, sizeof(int)) != cudaSuccess) {
      g_device_init_status[device] = TVR_ERR_CUDA;
      cudaGetLastError();
    } else {
      g_status_words[device] = status;
    }
    cudaSetDevice(prev);
  });
  if (g_device_init_status[device] != TVR_OK) {
    return fail(g_device_init_status[device], "initialising device %d failed", device);
  }
  return TVR_OK;
}

int check_device(int device) {
  if (device < 0 || device >= g_device_count) {
    return fail(TVR_ERR_INVALID, "tvarant device index out of range: %d (device count %d)",
                device, g_device_count);
  }
  return init_device(device);
}

// RAII switch of the calling thread's current device.
struct DeviceSwitch {
  int prev = -1;
  explicit DeviceSwitch(int device) {
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    else prev = -1;
  }
  ~DeviceSwitch() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int sm_count(int device) {
  if (device >= 0 && device < kMaxDevices && g_sm_count[device] > 0) return g_sm_count[device];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  return n;
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int* device_status_ptr(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  if (init_device(device) != TVR_OK) return nullptr;
  return g_status_words[device];
}

int* device_status_ptr_if_ready(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  return g_status_words[device];
}

const DriverApi* driver() {
  std::call_once(g_init_once, do_init);
  if (!g_driver_ok) {
    fail(TVR_ERR_CUDA, "CUDA driver entry points unavailable");
    return nullptr;
  }
  return &g_driver;
}

Scratch::~Scratch() {
  if (ptr != nullptr) tvr_free(ptr);
}

int Scratch::alloc(size_t nbytes, int device, cudaStream_t s) {
  stream = s;
  return tvr_malloc(&ptr, nbytes, device, s);
}

}  // namespace tvr

using namespace tvr;

extern "C" {

const char* tvr_last_error(void) { return t_last_error.c_str(); }

int tvr_init(void) {
  std::call_once(g_init_once, do_init);
  if (g_init_status != TVR_OK) return fail(g_init_status, "%s", g_init_error.c_str());
  if (!g_driver_ok) return fail(TVR_ERR_CUDA, "CUDA driver entry points unavailable");
  return TVR_OK;
}

const char* tvr_backend_name(void) { return "cuda"; }

int tvr_device_count(int* count) {
  TVR_CHECK(count != nullptr, "tvr_device_count: null output");
  std::call_once(g_init_once, do_init);
  *count = g_device_count;
  return TVR_OK;
}

int tvr_get_device(int* device) {
  TVR_CHECK(device != nullptr, "tvr_get_device: null output");
  TVR_CUDA_TRY(cudaGetDevice(device));
  return TVR_OK;
}

int tvr_set_device(int device) {
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  TVR_CUDA_TRY(cudaSetDevice(device));
  return TVR_OK;
}

int tvr_device_sm_count(int device, int* sms) {
  TVR_CHECK(sms != nullptr, "tvr_device_sm_count: null output");
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  *sms = sm_count(device);
  return TVR_OK;
}

int tvr_device_synchronize(int device) {
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  DeviceSwitch sw(device);
  TVR_CUDA_TRY(cudaDeviceSynchronize());
  return TVR_OK;
}

int tvr_get_status(int device, int* code) {
  TVR_CHECK(code != nullptr, "tvr_get_status: null output");
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  DeviceSwitch sw(device);
  TVR_CUDA_TRY(cudaMemcpy(code, g_status_words[device], sizeof(int), cudaMemcpyDeviceToHost));
  return TVR_OK;
}

int tvr_clear_status(int device) {
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  DeviceSwitch sw(device);
  TVR_CUDA_TRY(cudaMemset(g_status_words[device], 0, sizeof(int)));
  return TVR_OK;
}

// ---- memory ----------------------------------------------------------------

int tvr_malloc(void** ptr, size_t nbytes, int device, void* stream) {
  TVR_CHECK(ptr != nullptr, "tvr_malloc: null output");
  *ptr = nullptr;
  if (nbytes == 0) return TVR_OK;
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  DeviceSwitch sw(device);
  cudaStream_t s = as_stream(stream);
  void* p = nullptr;
  cudaError_t e = cudaMallocAsync(&p, nbytes, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    // The pool may hold freed blocks that only become reusable once their
    // streams drain; synchronise and retry once before reporting OOM.
    cudaDeviceSynchronize();
    e = cudaMallocAsync(&p, nbytes, s);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(TVR_ERR_OOM, "tvarant: out of memory allocating %zu bytes on device %d (%s)",
                  nbytes, device, cudaGetErrorString(e));
    }
  }
  {
    std::lock_guard<std::mutex> lock(g_alloc_mutex);
    g_allocs[p] = AllocInfo{device, nbytes, s, {}};
    g_in_use[device] += nbytes;
  }
  *ptr = p;
  return TVR_OK;
}

int tvr_free(void* ptr) {
  if (ptr == nullptr) return TVR_OK;
  AllocInfo info;
  {
    std::lock_guard<std::mutex> lock(g_alloc_mutex);
    auto it = g_allocs.find(ptr);
    if (it == g_allocs.end()) {
      return fail(TVR_ERR_INVALID, "tvr_free: %p was not allocated by tvr_malloc", ptr);
    }
    info = std::move(it->second);
    g_allocs.erase(it);
    g_in_use[info.device] -= info.nbytes;
  }
  DeviceSwitch sw(info.device);
  for (cudaEvent_t ev : info.uses) {
    cudaStreamWaitEvent(info.stream, ev, 0);
    cudaEventDestroy(ev);
  }
  TVR_CUDA_TRY(cudaFreeAsync(ptr, info.stream));
  return TVR_OK;
}

int tvr_record_stream(void* ptr, void* stream) {
  std::lock_guard<std::mutex> lock(g_alloc_mutex);
  auto it = g_allocs.find(ptr);
  if (it == g_allocs.end()) {
    return fail(TVR_ERR_INVALID, "tvr_record_stream: %p was not allocated by tvr_malloc", ptr);
  }
  if (as_stream(stream) == it->second.stream) return TVR_OK;
  DeviceSwitch sw(it->second.device);
  cudaEvent_t ev;
  TVR_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  TVR_CUDA_TRY(cudaEventRecord(ev, as_stream(stream)));
  it->second.uses.push_back(ev);
  return TVR_OK;
}

int tvr_pointer_device(const void* ptr, int* device) {
  TVR_CHECK(device != nullptr, "tvr_pointer_device: null output");
  *device = -1;
  if (ptr == nullptr) return TVR_OK;
  {
    std::lock_guard<std::mutex> lock(g_alloc_mutex);
    auto it = g_allocs.find(const_cast<void*>(ptr));
    if (it != g_allocs.end()) {
      *device = it->second.device;
      return TVR_OK;
    }
  }
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) == cudaSuccess &&
      (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged)) {
    *device = attr.device;
  }
  cudaGetLastError();
  return TVR_OK;
}

int tvr_memory_stats(int device, size_t* reserved, size_t* in_use) {
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  cudaMemPool_t pool;
  TVR_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
  uint64_t r = 0;
  TVR_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &r));
  if (reserved) *reserved = static_cast<size_t>(r);
  if (in_use) {
    std::lock_guard<std::mutex> lock(g_alloc_mutex);
    *in_use = g_in_use[device];
  }
  return TVR_OK;
}

int tvr_empty_cache(int device) {
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  DeviceSwitch sw(device);
  TVR_CUDA_TRY(cudaDeviceSynchronize());
  cudaMemPool_t pool;
  TVR_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
  TVR_CUDA_TRY(cudaMemPoolTrimTo(pool, 0));
  return TVR_OK;
}

int tvr_host_alloc(void** ptr, size_t nbytes) {
  TVR_CHECK(ptr != nullptr, "tvr_host_alloc: null output");
  *ptr = nullptr;
  if (nbytes == 0) return TVR_OK;
  void* p = nullptr;
  cudaError_t e = cudaHostAlloc(&p, nbytes, cudaHostAllocPortable);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TVR_ERR_OOM, "tvr_host_alloc(%zu) failed: %s", nbytes, cudaGetErrorString(e));
  }
  {
    std::lock_guard<std::mutex> lock(g_host_mutex);
    g_host_allocs[p] = nbytes;
  }
  *ptr = p;
  return TVR_OK;
}

int tvr_host_free(void* ptr) {
  if (ptr == nullptr) return TVR_OK;
  {
    std::lock_guard<std::mutex> lock(g_host_mutex);
    if (g_host_allocs.erase(ptr) == 0) {
      return fail(TVR_ERR_INVALID, "tvr_host_free: %p was not allocated by tvr_host_alloc", ptr);
    }
  }
  TVR_CUDA_TRY(cudaFreeHost(ptr));
  return TVR_OK;
}

int tvr_is_pinned(const void* ptr, int* pinned) {
  TVR_CHECK(pinned != nullptr, "tvr_is_pinned: null output");
  *pinned = 0;
  if (ptr == nullptr) return TVR_OK;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) == cudaSuccess && attr.type == cudaMemoryTypeHost) {
    *pinned = 1;
  }
  cudaGetLastError();
  return TVR_OK;
}

int tvr_memcpy_h2d(void* dst, const void* src, size_t nbytes, void* stream) {
  if (nbytes == 0) return TVR_OK;
  TVR_CHECK(dst != nullptr && src != nullptr, "tvr_memcpy_h2d: null pointer");
  TVR_CUDA_TRY(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice, as_stream(stream)));
  return TVR_OK;
}

int tvr_memcpy_d2h(void* dst, const void* src, size_t nbytes, void* stream) {
  if (nbytes == 0) return TVR_OK;
  TVR_CHECK(dst != nullptr && src != nullptr, "tvr_memcpy_d2h: null pointer");
  TVR_CUDA_TRY(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, as_stream(stream)));
  return TVR_OK;
}

int tvr_memcpy_d2d(void* dst, const void* src, size_t nbytes, void* stream) {
  if (nbytes == 0 || dst == src) return TVR_OK;
  TVR_CHECK(dst != nullptr && src != nullptr, "tvr_memcpy_d2d: null pointer");
  TVR_CUDA_TRY(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
  return TVR_OK;
}

// ---- streams and events ----------------------------------------------------

int tvr_stream_create(void** stream, int device, int priority) {
  TVR_CHECK(stream != nullptr, "tvr_stream_create: null output");
  std::call_once(g_init_once, do_init);
  int rc = check_device(device);
  if (rc != TVR_OK) return rc;
  DeviceSwitch sw(device);
  int lo = 0, hi = 0;
  cudaDeviceGetStreamPriorityRange(&lo, &hi);
  int p = priority;
  if (p > lo) p = lo;
  if (p < hi) p = hi;
  cudaStream_t s;
  TVR_CUDA_TRY(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, p));
  *stream = s;
  return TVR_OK;
}

int tvr_stream_destroy(void* stream) {
  if (stream == nullptr) return TVR_OK;
  TVR_CUDA_TRY(cudaStreamDestroy(as_stream(stream)));
  return TVR_OK;
}

int tvr_stream_synchronize(void* stream) {
  TVR_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  return TVR_OK;
}

int tvr_stream_query(void* stream, int* done) {
  TVR_CHECK(done != nullptr, "tvr_stream_query: null output");
  cudaError_t e = cudaStreamQuery(as_stream(stream));
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return TVR_OK;
  }
  TVR_CUDA_TRY(e);
  *done = 1;
  return TVR_OK;
}

int tvr_stream_wait_event(void* stream, void* event) {
  TVR_CHECK(event != nullptr, "tvr_stream_wait_event: null event");
  TVR_CUDA_TRY(cudaStreamWaitEvent(as_stream(stream), reinterpret_cast<cudaEvent_t>(event), 0));
  return TVR_OK;
}

int tvr_event_create(void** event, int enable_timing) {
  TVR_CHECK(event != nullptr, "tvr_event_create: null output");
  cudaEvent_t e;
  TVR_CUDA_TRY(cudaEventCreateWithFlags(&e, enable_timing ? cudaEventDefault
                                                          : cudaEventDisableTiming));
  *event = e;
  return TVR_OK;
}

int tvr_event_destroy(void* event) {
  if (event == nullptr) return TVR_OK;
  TVR_CUDA_TRY(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event)));
  return TVR_OK;
}

int tvr_event_record(void* event, void* stream) {
  TVR_CHECK(event != nullptr, "tvr_event_record: null event");
  TVR_CUDA_TRY(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), as_stream(stream)));
  return TVR_OK;
}

int tvr_event_synchronize(void* event) {
  TVR_CHECK(event != nullptr, "tvr_event_synchronize: null event");
  TVR_CUDA_TRY(cudaEventSynchronize(reinterpret_cast<cudaEvent_t>(event)));
  return TVR_OK;
}

int tvr_event_query(void* event, int* done) {
  TVR_CHECK(event != nullptr && done != nullptr, "tvr_event_query: null argument");
  cudaError_t e = cudaEventQuery(reinterpret_cast<cudaEvent_t>(event));
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return TVR_OK;
  }
  TVR_CUDA_TRY(e);
  *done = 1;
  return TVR_OK;
}

int tvr_event_elapsed_ms(void* start, void* end, float* ms) {
  TVR_CHECK(start != nullptr && end != nullptr && ms != nullptr,
            "tvr_event_elapsed_ms: null argument");
  TVR_CUDA_TRY(cudaEventElapsedTime(ms, reinterpret_cast<cudaEvent_t>(start),
                                    reinterpret_cast<cudaEvent_t>(end)));
  return TVR_OK;
}

// ---- graphs ----------------------------------------------------------------

int tvr_graph_begin(void* stream) {
  TVR_CHECK(stream != nullptr, "tvr_graph_begin: capture needs a created stream, not the default");
  // Relaxed: the allocator's bookkeeping (events for cross-stream uses) may
  // run while the capture is open.
  TVR_CUDA_TRY(cudaStreamBeginCapture(as_stream(stream), cudaStreamCaptureModeRelaxed));
  return TVR_OK;
}

int tvr_graph_end(void* stream, void** graph) {
  TVR_CHECK(stream != nullptr && graph != nullptr, "tvr_graph_end: null argument");
  *graph = nullptr;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(as_stream(stream), &g);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (g != nullptr) cudaGraphDestroy(g);
    return fail(TVR_ERR_CUDA, "tvr_graph_end: capture failed: %s", cudaGetErrorString(e));
  }
  cudaGraphExec_t exec = nullptr;
  // Allocations a launch leaves live are released when the graph is
  // launched again, so every replay gets the same addresses.
  e = cudaGraphInstantiateWithFlags(&exec, g, cudaGraphInstantiateFlagAutoFreeOnLaunch);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TVR_ERR_CUDA, "tvr_graph_end: instantiation failed: %s", cudaGetErrorString(e));
  }
  *graph = exec;
  return TVR_OK;
}

int tvr_graph_launch(void* graph, void* stream) {
  TVR_CHECK(graph != nullptr, "tvr_graph_launch: null graph");
  TVR_CUDA_TRY(cudaGraphLaunch(reinterpret_cast<cudaGraphExec_t>(graph), as_stream(stream)));
  return TVR_OK;
}

int tvr_graph_destroy(void* graph) {
  if (graph == nullptr) return TVR_OK;
  TVR_CUDA_TRY(cudaGraphExecDestroy(reinterpret_cast<cudaGraphExec_t>(graph)));
  return TVR_OK;
}

}  // extern "C"
