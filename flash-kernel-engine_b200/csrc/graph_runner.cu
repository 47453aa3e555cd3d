// CUDA graph runner (capture once, replay per decode step) and its C ABI.
// The capture/instantiate/launch sequence follows the reference's
// src/cuda_graph_runner.cu:14-55; errors are reported instead of exiting.
#include <stdexcept>
#include <string>

#include "../../include/cuda_graph_runner.h"
#include "../../include/flash_engine_c.h"

namespace flash_engine {
namespace graph {

namespace {
void throw_if(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("CUDAGraphRunner: ") + what + ": " +
                             cudaGetErrorString(e));
}
}  // namespace

CUDAGraphRunner::CUDAGraphRunner() : graph_(nullptr), instance_(nullptr), instantiated_(false) {}

CUDAGraphRunner::~CUDAGraphRunner() { reset(); }

void CUDAGraphRunner::capture(std::function<void(cudaStream_t)> record_func,
                              cudaStream_t stream) {
  reset();
  throw_if(cudaStreamBeginCapture(stream, cudaStreamCaptureModeGlobal), "begin capture");
  try {
    record_func(stream);
  } catch (...) {
    cudaStreamEndCapture(stream, &graph_);
    reset();
    throw;
  }
  throw_if(cudaStreamEndCapture(stream, &graph_), "end capture");
  throw_if(cudaGraphInstantiate(&instance_, graph_, nullptr, nullptr, 0), "instantiate");
  instantiated_ = true;
}

void CUDAGraphRunner::launch(cudaStream_t stream) {
  if (!instantiated_) throw std::runtime_error("CUDAGraphRunner: Cannot launch uncaptured graph.");
  throw_if(cudaGraphLaunch(instance_, stream), "launch");
}

void CUDAGraphRunner::reset() {
  if (instance_) {
    cudaGraphExecDestroy(instance_);
    instance_ = nullptr;
  }
  if (graph_) {
    cudaGraphDestroy(graph_);
    graph_ = nullptr;
  }
  instantiated_ = false;
}

}  // namespace graph
}  // namespace flash_engine

extern "C" {

int fe_graph_capture(fe_record_fn record, void* user, void* stream, void** graph_out) {
  if (!record || !graph_out) return static_cast<int>(cudaErrorInvalidValue);
  *graph_out = nullptr;
  auto* g = new flash_engine::graph::CUDAGraphRunner();
  try {
    g->capture([&](cudaStream_t s) { record(reinterpret_cast<void*>(s), user); },
               reinterpret_cast<cudaStream_t>(stream));
  } catch (const std::exception&) {
    delete g;
    cudaError_t e = cudaGetLastError();
    return static_cast<int>(e == cudaSuccess ? cudaErrorStreamCaptureInvalidated : e);
  }
  *graph_out = g;
  return 0;
}

int fe_graph_launch(void* graph, void* stream) {
  if (!graph) return static_cast<int>(cudaErrorInvalidValue);
  try {
    static_cast<flash_engine::graph::CUDAGraphRunner*>(graph)->launch(
        reinterpret_cast<cudaStream_t>(stream));
  } catch (const std::exception&) {
    cudaError_t e = cudaGetLastError();
    return static_cast<int>(e == cudaSuccess ? cudaErrorInvalidResourceHandle : e);
  }
  return 0;
}

void fe_graph_destroy(void* graph) {
  delete static_cast<flash_engine::graph::CUDAGraphRunner*>(graph);
}

}  // extern "C"
