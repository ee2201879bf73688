#include "exec/nvls.h"

namespace nb {

bool nvls_supported(const int*, int) { return false; }

bool nvls_ensure(const int*, int, size_t, std::string* why) {
  if (why) *why = "NVLS not built";
  return false;
}

cudaError_t nvls_launch(const PlanOp&, const Plan&, const Binding&, const Policy&, cudaStream_t,
                        int) {
  return cudaErrorNotSupported;
}

unsigned nvls_status(const int*, int) { return 0; }

}  // namespace nb
