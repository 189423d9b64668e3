// atlas_scan_fwd_noalloc: the tensor-path forward scan for callers that may not
// allocate device memory.  The scratch the forward kernel needs (per-chain
// progress counters, one carry slot per chain and per-cluster factor rows) lives in a fixed array in
// this file instead of a caller-provided workspace.
#include <mutex>
#include <string>

#include "common.cuh"
#include "scan_internal.h"

namespace {

constexpr size_t kChainSlotBytes = 4ull * 64 * 256 * sizeof(float);    // W1, S1, W2, S2 of one (b, h)
constexpr size_t kFlagBytes = 256;                                       // counters, padded
constexpr size_t kFactorBytes = 2ull * 64 * 256 * sizeof(float);       // per cluster: both CTAs' row factors
// at most one cluster per chain, so 16 chains need at most 16 clusters: 6 MiB + 256 B
constexpr size_t kScratchBytes = kFlagBytes + ATLAS_NOALLOC_MAX_CHAINS * (kChainSlotBytes + kFactorBytes);

// Device-resident scratch shared by every call on a device.  In host code this
// name is only a handle: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_addr[64] = {};  // device address of g_noalloc_scratch, per device ordinal

// Once per device, with that device current: look up the scratch address.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return atlas::report_error(ATLAS_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return atlas::report_error(ATLAS_ERR_UNSUPPORTED, "device ordinal >= 64");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return atlas::report_error(ATLAS_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) failed");
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return ATLAS_OK;
}

}  // namespace

extern "C" int atlas_scan_fwd_noalloc(const AtlasScanParams* p, const void* q, const void* k, const void* v,
                                      const float* alpha, const float* eta, const float* theta,
                                      const float* gamma, const float* W1_in, const float* W2_in,
                                      const float* S1_in, const float* S2_in, void* y, float* W1_out,
                                      float* W2_out, float* S1_out, float* S2_out, void* stream) {
  atlas::clear_error();
  // argument checks shared with the other entry points (sets the error string)
  const int rc0 = atlas::check_scan_params(p);
  if (rc0) return rc0;
  const char* why = "";
  if (!atlas::tc::supported(*p, &why)) {
    std::string m = std::string("tensor path (no-alloc forward): ") + why;
    return atlas::report_error(ATLAS_ERR_UNSUPPORTED, m.c_str());
  }
  if (p->precision != ATLAS_PREC_TENSOR)
    return atlas::report_error(ATLAS_ERR_UNSUPPORTED, "atlas_scan_fwd_noalloc supports ATLAS_PREC_TENSOR only");
  if ((long)p->B * p->H > ATLAS_NOALLOC_MAX_CHAINS)
    return atlas::report_error(ATLAS_ERR_INVALID_ARGUMENT,
                               "atlas_scan_fwd_noalloc: B*H exceeds ATLAS_NOALLOC_MAX_CHAINS (16)");
  if (!q || !k || !v || !alpha || !eta || !theta || !y)
    return atlas::report_error(ATLAS_ERR_INVALID_ARGUMENT, "q, k, v, alpha, eta, theta and y must be non-NULL");
  if ((W1_in || W2_in || S1_in || S2_in) && !(W1_in && W2_in && S1_in && S2_in))
    return atlas::report_error(ATLAS_ERR_INVALID_ARGUMENT, "state_in must be all NULL or all non-NULL");
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  atlas::FwdArgs a;
  a.p = *p;
  a.q = q; a.k = k; a.v = v;
  a.alpha = alpha; a.eta = eta; a.theta = theta; a.gamma = gamma;
  a.W1_in = W1_in; a.W2_in = W2_in; a.S1_in = S1_in; a.S2_in = S2_in;
  a.y = y;
  a.W1_out = W1_out; a.W2_out = W2_out; a.S1_out = S1_out; a.S2_out = S2_out;
  a.saved = nullptr;  // carries go through the fixed scratch
  a.ws = scratch;     // the launcher clears the counters at its start (stream-ordered memset)
  a.status = atlas::device_status_ptr();
  cudaError_t e = atlas::tc::launch_fwd(a, (cudaStream_t)stream);
  if (e != cudaSuccess) return atlas::report_error(ATLAS_ERR_CUDA, cudaGetErrorString(e));
  return ATLAS_OK;
}
