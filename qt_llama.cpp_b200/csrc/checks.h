// checks.h — argument checks shared by the C-ABI entry points (internal), so
// that every entry point that takes the same shapes accepts the same ones.
#pragma once
#include <stdint.h>

#include "../../include/mrml_moe.h"
#include "kernels.h"

namespace mrml {

// Router shapes and pointers (mrml_moe_router, mrml_moe_router_noalloc,
// the router half of mrml_moe_forward).
inline int check_router_args(const float* W, const float* x, const float* logits, const int32_t* ids,
                             const float* probs, int H, int E, int K, int T) {
  if (H <= 0 || E <= 0 || K <= 0 || T < 0) return MRML_ERR_INVALID_ARGUMENT;
  if (K > E) return MRML_ERR_INVALID_ARGUMENT;
  if (E > kMaxExperts || K > kMaxTopK) return MRML_ERR_UNSUPPORTED;
  if (T > 0 && (!W || !x || !logits || !ids || !probs)) return MRML_ERR_INVALID_ARGUMENT;
  return MRML_OK;
}

}  // namespace mrml
