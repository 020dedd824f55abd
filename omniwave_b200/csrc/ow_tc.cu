// Tensor-core (tcgen05) BiGEMM path for bf16/f16 compute.  Placeholder until
// the sm_100a kernels land: reports every shape as unsupported so calls take
// the CUDA-core path.
#include "ow_common.cuh"
#include "ow_internal.h"

namespace ow {

bool tc_supported(const ow_bigemm_args_t*, const Prob&, const char** why) {
  if (why) *why = "tensor-core path not built";
  return false;
}

int tc_forward(const ow_bigemm_args_t*, const Prob&, void*, Carver&) {
  set_error("tensor-core path not built");
  return OW_ERR_UNSUPPORTED;
}

int tc_backward(const ow_bigemm_args_t*, const ow_bigemm_grads_t*, const Prob&, void*, Carver&) {
  set_error("tensor-core path not built");
  return OW_ERR_UNSUPPORTED;
}

}  // namespace ow
