// tcgen05 (sm_100a) Atlas scan -- placeholder until the fused kernels land.
#include "common.cuh"
#include "scan_internal.h"

namespace atlas {
namespace tc {
bool supported(const AtlasScanParams&, const char** why) {
  *why = "not built yet";
  return false;
}
size_t saved_bytes(const AtlasScanParams&) { return 0; }
size_t workspace_bytes(const AtlasScanParams&) { return 0; }
cudaError_t launch_fwd(const FwdArgs&, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_bwd(const BwdArgs&, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace tc
}  // namespace atlas
