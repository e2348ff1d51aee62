// runtime.cu: the device, memory, stream, graph and error calls that the reference's engine did not need (its
// kernels worked on one linear WASM memory the engine owned) and a device-memory drop-in does. Every address the
// kernels take is a device pointer from pllm_alloc (or any other CUDA allocation of the same device).
#include "pllm_common.cuh"
#include <stdarg.h>
#include <string.h>
#include <mutex>

namespace {
std::mutex g_lock;
int g_code = 0;
char g_msg[512] = {0};
// each host thread's current stream (nullptr: the legacy default stream, as torch's default stream is), so that
// threads that call the kernels concurrently on disjoint row ranges each enqueue on their own
thread_local cudaStream_t g_stream = nullptr;
int g_sms = 0;
int g_device = -1;
}  // namespace

void pllm_fail(int code, const char* fmt, ...) {
  std::lock_guard<std::mutex> guard(g_lock);
  if (g_code) return;  // the first failure is kept until it is cleared
  g_code = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof g_msg, fmt, ap);
  va_end(ap);
}

int pllm_failed() { return g_code; }
std::mutex& pllm_lookup_lock() {
  static std::mutex m;
  return m;
}
std::mutex& pllm_scratch_lock() {
  static std::mutex m;
  return m;
}
cudaStream_t pllm_stream() { return g_stream; }

int pllm_num_sms() {
  if (!g_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  return g_sms;
}

static int check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    pllm_fail(e == cudaErrorMemoryAllocation ? PLLM_ENOMEM : PLLM_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

// ---- device and errors
namespace gemvk {
int* status_word();  // gemv_tma.cu
}

PLLM_API int32_t pllm_init(int32_t device) {
  if (check(cudaSetDevice(device), "cudaSetDevice")) return -1;
  g_device = device;
  g_sms = 0;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10) {
    pllm_fail(PLLM_ECUDA, "pllm_init: device %d is sm_%d%d; this library is built for sm_100a (B200) only", device,
              major, minor);
    return -1;
  }
  if (check(cudaFree(nullptr), "context")) return -1;
  // the device status word's address, looked up here once, outside any stream capture (the kernels that report
  // through it take it at launch)
  return gemvk::status_word() ? 0 : -1;
}

PLLM_API int32_t pllm_last_error(char* buf, int32_t len) {
  std::lock_guard<std::mutex> guard(g_lock);
  if (buf && len > 0) {
    strncpy(buf, g_msg, (size_t)len - 1);
    buf[len - 1] = 0;
  }
  return g_code;
}

PLLM_API void pllm_clear_error() {
  std::lock_guard<std::mutex> guard(g_lock);
  g_code = 0;
  g_msg[0] = 0;
}

PLLM_API int32_t pllm_num_sms_of_device() { return pllm_num_sms(); }

// ---- memory
PLLM_API uint64_t pllm_alloc(uint64_t bytes) {
  void* p = nullptr;
  if (check(cudaMalloc(&p, bytes ? bytes : 1), "pllm_alloc")) return 0;
  return (uint64_t)(uintptr_t)p;
}
PLLM_API void pllm_free(uint64_t p) {
  if (p) check(cudaFree(dptr<void>(p)), "pllm_free");
}
PLLM_API uint64_t pllm_alloc_host(uint64_t bytes) {  // pinned host memory for the end-to-end copies
  void* p = nullptr;
  if (check(cudaMallocHost(&p, bytes ? bytes : 1), "pllm_alloc_host")) return 0;
  return (uint64_t)(uintptr_t)p;
}
PLLM_API void pllm_free_host(uint64_t p) {
  if (p) check(cudaFreeHost(dptr<void>(p)), "pllm_free_host");
}
// copies on the current stream (asynchronous with respect to the host unless the host memory is pageable)
PLLM_API void pllm_h2d(uint64_t dst, const void* src, uint64_t bytes) {
  check(cudaMemcpyAsync(dptr<void>(dst), src, bytes, cudaMemcpyHostToDevice, g_stream), "pllm_h2d");
}
PLLM_API void pllm_d2h(void* dst, uint64_t src, uint64_t bytes) {
  check(cudaMemcpyAsync(dst, dptr<void>(src), bytes, cudaMemcpyDeviceToHost, g_stream), "pllm_d2h");
}
PLLM_API void pllm_d2d(uint64_t dst, uint64_t src, uint64_t bytes) {
  check(cudaMemcpyAsync(dptr<void>(dst), dptr<void>(src), bytes, cudaMemcpyDeviceToDevice, g_stream), "pllm_d2d");
}
PLLM_API void pllm_memset(uint64_t dst, int32_t value, uint64_t bytes) {
  check(cudaMemsetAsync(dptr<void>(dst), value, bytes, g_stream), "pllm_memset");
}

// ---- streams
PLLM_API uint64_t pllm_stream_create() {
  cudaStream_t s = nullptr;
  if (check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "pllm_stream_create")) return 0;
  return (uint64_t)(uintptr_t)s;
}
PLLM_API void pllm_stream_destroy(uint64_t s) {
  if (s) check(cudaStreamDestroy((cudaStream_t)(uintptr_t)s), "pllm_stream_destroy");
}
// every kernel and copy after this goes on stream s (0: the legacy default stream)
PLLM_API void pllm_set_stream(uint64_t s) { g_stream = (cudaStream_t)(uintptr_t)s; }
PLLM_API uint64_t pllm_get_stream() { return (uint64_t)(uintptr_t)g_stream; }
PLLM_API int32_t pllm_sync() { return check(cudaStreamSynchronize(g_stream), "pllm_sync"); }
PLLM_API int32_t pllm_device_sync() { return check(cudaDeviceSynchronize(), "pllm_device_sync"); }

// ---- CUDA graphs: the calls between begin and end on the current stream are recorded, not run; launch replays them
PLLM_API int32_t pllm_graph_begin() {
  return check(cudaStreamBeginCapture(g_stream, cudaStreamCaptureModeThreadLocal), "pllm_graph_begin");
}
PLLM_API uint64_t pllm_graph_end() {
  cudaGraph_t graph = nullptr;
  if (check(cudaStreamEndCapture(g_stream, &graph), "pllm_graph_end")) {
    cudaGetLastError();  // an invalidated capture also leaves the thread's last error set: the next launch is not at fault
    return 0;
  }
  cudaGraphExec_t exec = nullptr;
  cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (check(e, "cudaGraphInstantiate")) return 0;
  return (uint64_t)(uintptr_t)exec;
}
PLLM_API int32_t pllm_graph_launch(uint64_t exec) {
  return check(cudaGraphLaunch((cudaGraphExec_t)(uintptr_t)exec, g_stream), "pllm_graph_launch");
}
PLLM_API void pllm_graph_destroy(uint64_t exec) {
  if (exec) check(cudaGraphExecDestroy((cudaGraphExec_t)(uintptr_t)exec), "pllm_graph_destroy");
}

// ---- events, for timing on the stream the kernels run on
PLLM_API uint64_t pllm_event_create() {
  cudaEvent_t e = nullptr;
  if (check(cudaEventCreate(&e), "pllm_event_create")) return 0;
  return (uint64_t)(uintptr_t)e;
}
PLLM_API void pllm_event_record(uint64_t e) { check(cudaEventRecord((cudaEvent_t)(uintptr_t)e, g_stream), "pllm_event_record"); }
PLLM_API float pllm_event_ms(uint64_t a, uint64_t b) {
  float ms = -1.0f;
  if (check(cudaEventSynchronize((cudaEvent_t)(uintptr_t)b), "cudaEventSynchronize")) return -1.0f;
  check(cudaEventElapsedTime(&ms, (cudaEvent_t)(uintptr_t)a, (cudaEvent_t)(uintptr_t)b), "cudaEventElapsedTime");
  return ms;
}
PLLM_API void pllm_event_destroy(uint64_t e) {
  if (e) cudaEventDestroy((cudaEvent_t)(uintptr_t)e);
}

PLLM_API const char* pllm_version() { return "pllm 0.1 (sm_100a)"; }
