// Library core: error text, device status word, memory and stream entry
// points of the C ABI (include/templit_cuda.h).
#include "tl_common.cuh"

#include <cstdlib>
#include <cstring>

#include <cstdio>
#include <cstring>

namespace tl {

static thread_local std::string g_last_error;

int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return TL_OK;
  return fail(TL_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

static thread_local uint64_t g_kernel_launches = 0;

int launch_status(const char *what) {
  ++g_kernel_launches;
  return check_cuda(cudaGetLastError(), what);
}

// One status word per device that loads the library.
__device__ uint32_t g_status_flags;

uint32_t *device_status_ptr() {
  static uint32_t *cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cached[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_flags) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<uint32_t *>(p);
  }
  return cached[dev];
}

// Moves the status word into a mailbox and clears it, in stream order.
__global__ void status_take_kernel(uint32_t *status, uint32_t *mailbox) {
  pdl_enter();
  *mailbox = *status;
  *status = 0;
}

__device__ uint32_t g_status_mailbox;

bool pdl_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("TL_PDL");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  return on;
}

}  // namespace tl

using namespace tl;

extern "C" {

int tl_version(void) { return 1; }

const char *tl_last_error(void) { return g_last_error.c_str(); }

int tl_device_init(int device) {
  int rc = check_cuda(cudaSetDevice(device), "cudaSetDevice");
  if (rc) return rc;
  return check_cuda(cudaFree(nullptr), "context init");
}

int tl_device_status(uint32_t *flags, void *stream) {
  if (!flags) return fail(TL_ERR_INVALID, "tl_device_status: null flags");
  int rc = check_cuda(cudaStreamSynchronize(as_stream(stream)), "stream sync");
  if (rc) return rc;
  rc = check_cuda(cudaMemcpyFromSymbol(flags, g_status_flags, sizeof(uint32_t)),
                  "read status");
  if (rc) return rc;
  if (*flags) {
    const uint32_t zero = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_status_flags, &zero, sizeof(uint32_t)),
                    "clear status");
  }
  return rc;
}

int tl_device_status_enqueue(uint32_t *host_flags, void *stream) {
  if (!host_flags) return fail(TL_ERR_INVALID, "tl_device_status_enqueue: null flags");
  uint32_t *status = device_status_ptr();
  uint32_t *mailbox = nullptr;
  int rc = check_cuda(cudaGetSymbolAddress(reinterpret_cast<void **>(&mailbox), g_status_mailbox),
                      "status mailbox");
  if (rc) return rc;
  if (!status) return fail(TL_ERR_CUDA, "tl_device_status_enqueue: no status word");
  cudaStream_t s = as_stream(stream);
  launch_pdl(status_take_kernel, 1, 1, 0, s, status, mailbox);
  rc = launch_status("tl_device_status_enqueue");
  if (rc) return rc;
  return check_cuda(cudaMemcpyAsync(host_flags, mailbox, sizeof(uint32_t),
                                    cudaMemcpyDeviceToHost, s),
                    "status copy");
}

int tl_malloc(void **ptr, size_t bytes) {
  if (!ptr) return fail(TL_ERR_INVALID, "tl_malloc: null out pointer");
  *ptr = nullptr;
  if (bytes == 0) return TL_OK;
  return check_cuda(cudaMalloc(ptr, bytes), "cudaMalloc");
}

int tl_free(void *ptr) {
  if (!ptr) return TL_OK;
  return check_cuda(cudaFree(ptr), "cudaFree");
}

int tl_host_alloc(void **ptr, size_t bytes) {
  if (!ptr) return fail(TL_ERR_INVALID, "tl_host_alloc: null out pointer");
  *ptr = nullptr;
  if (bytes == 0) return TL_OK;
  return check_cuda(cudaMallocHost(ptr, bytes), "cudaMallocHost");
}

int tl_host_free(void *ptr) {
  if (!ptr) return TL_OK;
  return check_cuda(cudaFreeHost(ptr), "cudaFreeHost");
}

int tl_stream_create(void **stream) {
  if (!stream) return fail(TL_ERR_INVALID, "tl_stream_create: null out pointer");
  cudaStream_t s = nullptr;
  int rc = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking),
                      "cudaStreamCreate");
  *stream = s;
  return rc;
}

int tl_stream_destroy(void *stream) {
  if (!stream) return TL_OK;
  return check_cuda(cudaStreamDestroy(as_stream(stream)), "cudaStreamDestroy");
}

int tl_stream_sync(void *stream) {
  return check_cuda(cudaStreamSynchronize(as_stream(stream)), "cudaStreamSynchronize");
}

int tl_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream) {
  if (bytes == 0) return TL_OK;
  if (!dst || !src) return fail(TL_ERR_INVALID, "tl_memcpy_h2d: null pointer");
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice,
                                    as_stream(stream)),
                    "cudaMemcpyAsync H2D");
}

int tl_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream) {
  if (bytes == 0) return TL_OK;
  if (!dst || !src) return fail(TL_ERR_INVALID, "tl_memcpy_d2h: null pointer");
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost,
                                    as_stream(stream)),
                    "cudaMemcpyAsync D2H");
}

int tl_event_create(void **event) {
  if (!event) return fail(TL_ERR_INVALID, "tl_event_create: null out pointer");
  cudaEvent_t e = nullptr;
  int rc = check_cuda(cudaEventCreate(&e), "cudaEventCreate");
  *event = e;
  return rc;
}

int tl_event_destroy(void *event) {
  if (!event) return TL_OK;
  return check_cuda(cudaEventDestroy(static_cast<cudaEvent_t>(event)), "cudaEventDestroy");
}

int tl_event_record(void *event, void *stream) {
  if (!event) return fail(TL_ERR_INVALID, "tl_event_record: null event");
  return check_cuda(cudaEventRecord(static_cast<cudaEvent_t>(event), as_stream(stream)),
                    "cudaEventRecord");
}

int tl_event_elapsed_ms(float *ms, void *start, void *end) {
  if (!ms || !start || !end) return fail(TL_ERR_INVALID, "tl_event_elapsed_ms: null pointer");
  int rc = check_cuda(cudaEventSynchronize(static_cast<cudaEvent_t>(end)), "cudaEventSynchronize");
  if (rc) return rc;
  return check_cuda(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start),
                                         static_cast<cudaEvent_t>(end)),
                    "cudaEventElapsedTime");
}

int tl_event_query(void *event, int *done) {
  if (!event || !done) return fail(TL_ERR_INVALID, "tl_event_query: null pointer");
  const cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(event));
  if (e == cudaErrorNotReady) {
    *done = 0;
    return TL_OK;
  }
  *done = 1;
  return check_cuda(e, "cudaEventQuery");
}

int tl_graph_capture_begin(void *stream) {
  if (!stream) return fail(TL_ERR_INVALID, "tl_graph_capture_begin: legacy stream cannot capture");
  return check_cuda(cudaStreamBeginCapture(as_stream(stream), cudaStreamCaptureModeThreadLocal),
                    "cudaStreamBeginCapture");
}

int tl_graph_capture_end(void *stream, void **graph_exec) {
  if (!graph_exec) return fail(TL_ERR_INVALID, "tl_graph_capture_end: null out pointer");
  *graph_exec = nullptr;
  cudaGraph_t graph = nullptr;
  int rc = check_cuda(cudaStreamEndCapture(as_stream(stream), &graph), "cudaStreamEndCapture");
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  cudaGraphExec_t exec = nullptr;
  rc = check_cuda(cudaGraphInstantiate(&exec, graph, 0), "cudaGraphInstantiate");
  cudaGraphDestroy(graph);
  if (rc) return rc;
  *graph_exec = exec;
  return TL_OK;
}

int tl_graph_launch(void *graph_exec, void *stream) {
  if (!graph_exec) return fail(TL_ERR_INVALID, "tl_graph_launch: null graph");
  return check_cuda(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), as_stream(stream)),
                    "cudaGraphLaunch");
}

int tl_graph_destroy(void *graph_exec) {
  if (!graph_exec) return TL_OK;
  return check_cuda(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)),
                    "cudaGraphExecDestroy");
}

uint64_t tl_kernel_launches(void) { return g_kernel_launches; }

int tl_memcpy_d2d(void *dst, const void *src, size_t bytes, void *stream) {
  if (bytes == 0 || dst == src) return TL_OK;
  if (!dst || !src) return fail(TL_ERR_INVALID, "tl_memcpy_d2d: null pointer");
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice,
                                    as_stream(stream)),
                    "cudaMemcpyAsync D2D");
}

}  // extern "C"
