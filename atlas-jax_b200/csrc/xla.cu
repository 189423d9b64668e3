// XLA custom-call adapters of the scan (include/atlas_scan.h, atlas_xla_*).
//
// They use XLA's status-returning custom-call signature (api_version 2):
//   void fn(cudaStream_t stream, void** buffers, const char* opaque, size_t opaque_len,
//           XlaCustomCallStatus* status)
// which needs no XLA header: the buffers are the operands followed by the results
// in the order documented in the header, and `opaque` is the packed AtlasScanParams
// (the custom call's backend_config).  They replace the jax.custom_vjp pair
// fused_chunk_scan_kernel (atlas_jax/kernels/fused_chunk.py:321-379, called at
// atlas_jax/memory_layer.py:535-541) and, one level up, the scan of
// AtlasMemoryLayer.__call__ (memory_layer.py:635-718).
//
// Errors: XLA's XlaCustomCallStatusSetFailure is referenced weakly.  Inside a
// process where XLA exports it, a failing call reports its message there; otherwise
// (and always) the message is also left in atlas_last_error_string() of the calling
// thread.
#include <cstring>

#include "atlas_scan.h"
#include "scan_internal.h"

extern "C" void XlaCustomCallStatusSetFailure(void* status, const char* message, size_t message_len)
    __attribute__((weak));

namespace {

int unpack(const char* opaque, size_t len, AtlasScanParams* p) {
  if (!opaque || len != sizeof(AtlasScanParams))
    return atlas::report_error(ATLAS_ERR_INVALID_ARGUMENT, "atlas_xla: opaque must be one packed AtlasScanParams");
  std::memcpy(p, opaque, sizeof(*p));
  return ATLAS_OK;
}

void finish(int rc, void* status) {
  if (rc == ATLAS_OK || !status || !XlaCustomCallStatusSetFailure) return;
  const char* m = atlas_last_error_string();
  XlaCustomCallStatusSetFailure(status, m, std::strlen(m));
}

}  // namespace

extern "C" {

size_t atlas_xla_opaque_bytes(void) { return sizeof(AtlasScanParams); }

void atlas_xla_fwd(void* stream, void** b, const char* opaque, size_t opaque_len, void* status) {
  atlas::clear_error();
  AtlasScanParams p;
  int rc = unpack(opaque, opaque_len, &p);
  if (rc == ATLAS_OK && !b) rc = atlas::report_error(ATLAS_ERR_INVALID_ARGUMENT, "atlas_xla_fwd: buffers is NULL");
  if (rc == ATLAS_OK) {
    const size_t ws = atlas_scan_workspace_bytes(&p);
    rc = atlas_scan_fwd(&p, b[0], b[1], b[2], (const float*)b[3], (const float*)b[4], (const float*)b[5],
                        (const float*)b[6], (const float*)b[7], (const float*)b[8], (const float*)b[9],
                        (const float*)b[10], b[11], (float*)b[12], (float*)b[13], (float*)b[14], (float*)b[15],
                        b[16], b[17], ws, stream);
  }
  finish(rc, status);
}

void atlas_xla_bwd(void* stream, void** b, const char* opaque, size_t opaque_len, void* status) {
  atlas::clear_error();
  AtlasScanParams p;
  int rc = unpack(opaque, opaque_len, &p);
  if (rc == ATLAS_OK && !b) rc = atlas::report_error(ATLAS_ERR_INVALID_ARGUMENT, "atlas_xla_bwd: buffers is NULL");
  if (rc == ATLAS_OK) {
    const size_t ws = atlas_scan_workspace_bytes(&p);
    rc = atlas_scan_bwd(&p, b[0], b[1], b[2], (const float*)b[3], (const float*)b[4], (const float*)b[5],
                        (const float*)b[6], b[7], b[8], (const float*)b[9], (const float*)b[10],
                        (const float*)b[11], (const float*)b[12], b[13], b[14], b[15], (float*)b[16],
                        (float*)b[17], (float*)b[18], (float*)b[19], (float*)b[20], (float*)b[21], (float*)b[22],
                        (float*)b[23], b[24], ws, stream);
  }
  finish(rc, status);
}

// Opaque of atlas_xla_polar_express: the problem and its options, packed.
struct AtlasXlaPEOpaque {
  int64_t batch;
  int32_t rows, cols, ns_steps, precision;
  float eps_in_sqrt;
  int32_t pad;
};

size_t atlas_xla_pe_opaque_bytes(void) { return sizeof(AtlasXlaPEOpaque); }

void atlas_xla_polar_express(void* stream, void** b, const char* opaque, size_t opaque_len, void* status) {
  atlas::clear_error();
  int rc = ATLAS_OK;
  AtlasXlaPEOpaque o;
  if (!opaque || opaque_len != sizeof(o) || !b)
    rc = atlas::report_error(ATLAS_ERR_INVALID_ARGUMENT,
                             "atlas_xla_polar_express: opaque must be one packed AtlasXlaPEOpaque");
  if (rc == ATLAS_OK) {
    std::memcpy(&o, opaque, sizeof(o));
    const size_t ws = atlas_polar_express_workspace_bytes(o.batch, o.rows, o.cols, o.ns_steps, o.precision);
    rc = atlas_polar_express_batched((const float*)b[0], (float*)b[1], o.batch, o.rows, o.cols, o.ns_steps,
                                     o.eps_in_sqrt, o.precision, b[2], ws, stream);
  }
  finish(rc, status);
}

}  // extern "C"
