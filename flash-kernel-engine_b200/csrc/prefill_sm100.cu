// tcgen05 FA2 prefill (placeholder until the kernel lands).
#include "prefill.h"

namespace fe {
namespace prefill {

cudaError_t launch_prefill(const void*, const void*, const void*, void*, int, int, int, int, int,
                           int, float, bool, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace prefill
}  // namespace fe
