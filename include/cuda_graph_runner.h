// CUDA graph capture / replay of a decode step -- drop-in for the reference's
// include/cuda_graph_runner.h:10-35 (same class, same methods). Implemented in
// libflash_engine_b200.so (csrc/graph_runner.cu). Difference: CUDA errors raise
// std::runtime_error with the error string instead of exiting the process
// (the reference's CUDA_CHECK calls exit()).
#pragma once

#include <cuda_runtime.h>

#include <functional>

namespace flash_engine {
namespace graph {

class CUDAGraphRunner {
 public:
  CUDAGraphRunner();
  ~CUDAGraphRunner();
  CUDAGraphRunner(const CUDAGraphRunner&) = delete;
  CUDAGraphRunner& operator=(const CUDAGraphRunner&) = delete;

  // Records everything record_func enqueues on `stream` (global capture mode) and
  // instantiates the graph. Any previous graph is released first.
  void capture(std::function<void(cudaStream_t)> record_func, cudaStream_t stream = nullptr);
  // Replays the instantiated graph on `stream`.
  void launch(cudaStream_t stream = nullptr);
  bool is_captured() const { return instantiated_; }
  void reset();

 private:
  cudaGraph_t graph_;
  cudaGraphExec_t instance_;
  bool instantiated_;
};

}  // namespace graph
}  // namespace flash_engine
