// Library plumbing: error text, device queries, stream capture / graph replay.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace cb {

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

int sm_count() {
  static thread_local int cached_device = -1;
  static thread_local int cached_count = 0;
  int device = 0;
  cudaGetDevice(&device);
  if (device != cached_device) {
    cudaDeviceGetAttribute(&cached_count, cudaDevAttrMultiProcessorCount, device);
    cached_device = device;
  }
  return cached_count > 0 ? cached_count : 148;
}

}  // namespace cb

extern "C" {

int cb_abi_version(void) { return 1; }

const char* cb_last_error(void) { return cb::g_error; }

int cb_sm_count(int* count) {
  *count = cb::sm_count();
  return CB_OK;
}

int cb_stream_create(cb_stream_t* stream) {
  cudaStream_t s;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    cb::set_error("cudaStreamCreate: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  *stream = s;
  return CB_OK;
}

int cb_stream_destroy(cb_stream_t stream) {
  cudaError_t e = cudaStreamDestroy(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cb::set_error("cudaStreamDestroy: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

int cb_capture_begin(cb_stream_t stream) {
  cudaError_t e = cudaStreamBeginCapture(static_cast<cudaStream_t>(stream),
                                         cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) {
    cb::set_error("cudaStreamBeginCapture: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

int cb_capture_end(cb_stream_t stream, void** graph_exec) {
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &graph);
  if (e != cudaSuccess) {
    cb::set_error("cudaStreamEndCapture: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiateWithFlags(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    cb::set_error("cudaGraphInstantiate: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  *graph_exec = exec;
  return CB_OK;
}

int cb_graph_launch(void* graph_exec, cb_stream_t stream) {
  cudaError_t e = cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec),
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cb::set_error("cudaGraphLaunch: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

int cb_graph_destroy(void* graph_exec) {
  cudaError_t e = cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec));
  if (e != cudaSuccess) {
    cb::set_error("cudaGraphExecDestroy: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

}  // extern "C"
