// Runtime plumbing of the C ABI: errors, device/context, memory, streams, graphs and
// events. Replaces HIVE Limited's engine/cudrv.py (ctypes over libcuda).
#include <cstdlib>
#include <string>

#include "hv_internal.h"

namespace hv {

static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int cuda_fail(const char* what, cudaError_t e) {
  set_error("%s failed: %s (%d): %s", what, cudaGetErrorName(e), (int)e,
            cudaGetErrorString(e));
  return (int)e;
}

int sm_count(int* out) {
  static int cache[64];
  int dev = 0;
  HV_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && cache[dev] > 0) {
    *out = cache[dev];
    return HV_OK;
  }
  HV_CUDA(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev));
  if (dev >= 0 && dev < 64) cache[dev] = *out;
  return HV_OK;
}

}  // namespace hv

extern "C" {

int hv_version(void) { return HV_ABI_VERSION; }

int hv_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return HV_E_INVALID;
  strncpy(buf, hv::g_last_error, len - 1);
  buf[len - 1] = 0;
  return HV_OK;
}

int hv_init(void) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return hv::cuda_fail("cudaGetDeviceCount", e);
  HV_REQUIRE(n > 0, HV_E_NODEVICE, "no CUDA device is visible");
  HV_CUDA(cudaFree(nullptr));   // create the primary context on the current device
  return HV_OK;
}

int hv_device_count(int* n) {
  HV_REQUIRE(n, HV_E_INVALID, "hv_device_count: null pointer");
  HV_CUDA(cudaGetDeviceCount(n));
  return HV_OK;
}

int hv_set_device(int dev) {
  HV_CUDA(cudaSetDevice(dev));
  HV_CUDA(cudaFree(nullptr));
  return HV_OK;
}

int hv_get_device(int* dev) {
  HV_REQUIRE(dev, HV_E_INVALID, "hv_get_device: null pointer");
  HV_CUDA(cudaGetDevice(dev));
  return HV_OK;
}

int hv_device_name(int dev, char* buf, int len) {
  HV_REQUIRE(buf && len > 0, HV_E_INVALID, "hv_device_name: bad buffer");
  cudaDeviceProp p;
  HV_CUDA(cudaGetDeviceProperties(&p, dev));
  strncpy(buf, p.name, (size_t)len - 1);
  buf[len - 1] = 0;
  return HV_OK;
}

int hv_compute_capability(int dev, int* major, int* minor) {
  HV_REQUIRE(major && minor, HV_E_INVALID, "hv_compute_capability: null pointer");
  HV_CUDA(cudaDeviceGetAttribute(major, cudaDevAttrComputeCapabilityMajor, dev));
  HV_CUDA(cudaDeviceGetAttribute(minor, cudaDevAttrComputeCapabilityMinor, dev));
  return HV_OK;
}

int hv_device_attribute(int dev, int attr, int* value) {
  HV_REQUIRE(value, HV_E_INVALID, "hv_device_attribute: null pointer");
  HV_CUDA(cudaDeviceGetAttribute(value, (cudaDeviceAttr)attr, dev));
  return HV_OK;
}

int hv_driver_version(int* version) {
  HV_REQUIRE(version, HV_E_INVALID, "hv_driver_version: null pointer");
  HV_CUDA(cudaDriverGetVersion(version));
  return HV_OK;
}

int hv_mem_info(size_t* free_bytes, size_t* total_bytes) {
  HV_REQUIRE(free_bytes && total_bytes, HV_E_INVALID, "hv_mem_info: null pointer");
  HV_CUDA(cudaMemGetInfo(free_bytes, total_bytes));
  return HV_OK;
}

int hv_synchronize(void) {
  HV_CUDA(cudaDeviceSynchronize());
  return HV_OK;
}

int hv_alloc(void** ptr, size_t nbytes) {
  HV_REQUIRE(ptr, HV_E_INVALID, "hv_alloc: null pointer");
  size_t n = (nbytes + 255) & ~size_t(255);
  if (n == 0) n = 256;
  HV_CUDA(cudaMalloc(ptr, n));
  return HV_OK;
}

int hv_free(void* ptr) {
  HV_CUDA(cudaFree(ptr));
  return HV_OK;
}

int hv_upload(void* dst, const void* src, size_t nbytes) {
  HV_CUDA(cudaMemcpy(dst, src, nbytes, cudaMemcpyHostToDevice));
  return HV_OK;
}

int hv_download(void* dst, const void* src, size_t nbytes) {
  HV_CUDA(cudaMemcpy(dst, src, nbytes, cudaMemcpyDeviceToHost));
  return HV_OK;
}

int hv_memset(void* ptr, int value, size_t nbytes) {
  HV_CUDA(cudaMemset(ptr, value, nbytes));
  return HV_OK;
}

int hv_host_alloc(void** ptr, size_t nbytes) {
  HV_REQUIRE(ptr, HV_E_INVALID, "hv_host_alloc: null pointer");
  HV_CUDA(cudaHostAlloc(ptr, nbytes ? nbytes : 16, cudaHostAllocDefault));
  return HV_OK;
}

int hv_host_free(void* ptr) {
  HV_CUDA(cudaFreeHost(ptr));
  return HV_OK;
}

int hv_upload_async(void* dst, const void* src, size_t nbytes, void* stream) {
  HV_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
  return HV_OK;
}

int hv_download_async(void* dst, const void* src, size_t nbytes, void* stream) {
  HV_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  return HV_OK;
}

int hv_copy_async(void* dst, const void* src, size_t nbytes, void* stream) {
  HV_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  return HV_OK;
}

int hv_ipc_handle(const void* dev_ptr, void* handle_out) {
  HV_REQUIRE(dev_ptr && handle_out, HV_E_INVALID, "hv_ipc_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == HV_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  HV_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
  memcpy(handle_out, &h, sizeof(h));
  return HV_OK;
}

int hv_ipc_open(const void* handle, void** dev_ptr) {
  HV_REQUIRE(handle && dev_ptr, HV_E_INVALID, "hv_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  HV_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return HV_OK;
}

int hv_ipc_close(void* dev_ptr) {
  HV_REQUIRE(dev_ptr, HV_E_INVALID, "hv_ipc_close: null pointer");
  HV_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return HV_OK;
}

int hv_stream_create(void** stream) {
  HV_REQUIRE(stream, HV_E_INVALID, "hv_stream_create: null pointer");
  cudaStream_t s;
  HV_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return HV_OK;
}

int hv_stream_destroy(void* stream) {
  HV_CUDA(cudaStreamDestroy((cudaStream_t)stream));
  return HV_OK;
}

int hv_stream_synchronize(void* stream) {
  HV_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  return HV_OK;
}

int hv_capture_begin(void* stream) {
  HV_REQUIRE(stream, HV_E_INVALID, "hv_capture_begin: capture needs a created stream");
  HV_CUDA(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeGlobal));
  return HV_OK;
}

int hv_capture_end(void* stream, void** graph) {
  HV_REQUIRE(graph, HV_E_INVALID, "hv_capture_end: null pointer");
  cudaGraph_t g = nullptr;
  HV_CUDA(cudaStreamEndCapture((cudaStream_t)stream, &g));
  *graph = g;
  return HV_OK;
}

int hv_graph_instantiate(void* graph, void** exec) {
  HV_REQUIRE(graph && exec, HV_E_INVALID, "hv_graph_instantiate: null pointer");
  cudaGraphExec_t e = nullptr;
  HV_CUDA(cudaGraphInstantiate(&e, (cudaGraph_t)graph, 0));
  *exec = e;
  return HV_OK;
}

int hv_graph_launch(void* exec, void* stream) {
  HV_CUDA(cudaGraphLaunch((cudaGraphExec_t)exec, (cudaStream_t)stream));
  return HV_OK;
}

int hv_graph_destroy(void* graph, void* exec) {
  if (exec) HV_CUDA(cudaGraphExecDestroy((cudaGraphExec_t)exec));
  if (graph) HV_CUDA(cudaGraphDestroy((cudaGraph_t)graph));
  return HV_OK;
}

int hv_event_create(void** event) {
  HV_REQUIRE(event, HV_E_INVALID, "hv_event_create: null pointer");
  cudaEvent_t e;
  HV_CUDA(cudaEventCreate(&e));
  *event = e;
  return HV_OK;
}

int hv_event_destroy(void* event) {
  HV_CUDA(cudaEventDestroy((cudaEvent_t)event));
  return HV_OK;
}

int hv_event_record(void* event, void* stream) {
  HV_CUDA(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
  return HV_OK;
}

int hv_event_elapsed_ms(void* start, void* end, float* ms) {
  HV_REQUIRE(ms, HV_E_INVALID, "hv_event_elapsed_ms: null pointer");
  HV_CUDA(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return HV_OK;
}

}  // extern "C"
