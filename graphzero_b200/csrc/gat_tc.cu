// bf16 tensor-core GAT forward (placeholder until the tcgen05 kernel lands).
#include "gz_internal.h"

namespace gz {
size_t gat_tc_packed_bytes(int) { return 0; }
cudaError_t launch_gat_tc_pack(int, const float*, void*, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_gat_tc(int, const void*, const float*, const int8_t*, const int8_t*, int, float*, float*,
                          cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace gz
