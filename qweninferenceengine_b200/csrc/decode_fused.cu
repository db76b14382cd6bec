// decode_fused.cu -- the fused decode step (placeholder until the persistent
// kernel lands): reports that the fused path is unavailable.
#include "engine.h"
#include "status.h"

namespace qwen {

int fused_scratch_bytes(int, int, int, size_t* bytes) {
  *bytes = 0;
  return set_error(QWEN_ERR_STATE, "fused decode path not built in this library");
}
int enqueue_fused_step(const FusedStepArgs&, cudaStream_t) {
  return set_error(QWEN_ERR_STATE, "fused decode path not built in this library");
}

}  // namespace qwen
