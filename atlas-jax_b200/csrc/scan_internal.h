// Internal launch interface shared by the ABI layer and the kernel files.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#include <mutex>

#include "atlas_scan.h"

namespace atlas {

struct FwdArgs {
  AtlasScanParams p;
  const void *q, *k, *v;
  const float *alpha, *eta, *theta, *gamma;
  const float *W1_in, *W2_in, *S1_in, *S2_in;  // may be null (LM init)
  void* y;
  float *W1_out, *W2_out, *S1_out, *S2_out;
  void* saved;  // may be null
  void* ws;
  int* status;  // device status word
};

struct BwdArgs {
  AtlasScanParams p;
  const void *q, *k, *v;
  const float *alpha, *eta, *theta, *gamma;
  const void* saved;
  const void* dy;
  const float *dW1_out, *dW2_out, *dS1_out, *dS2_out;  // may be null
  void *dq, *dk, *dv;
  float *dalpha, *deta, *dtheta, *dgamma;
  float *dW1_in, *dW2_in, *dS1_in, *dS2_in;
  void* ws;
  int* status;
};

// A host-side value computed once per device ordinal (occupancy-derived grid sizes
// and the like), thread-safe.  Ordinals >= 64 compute it on every call.
struct DeviceCache {
  std::mutex mu;
  int v[64];
  DeviceCache() {
    for (int& x : v) x = -1;
  }
  template <class F>
  int get(F compute) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return compute();
    std::lock_guard<std::mutex> lk(mu);
    if (v[dev] < 0) v[dev] = compute();
    return v[dev];
  }
};

__host__ __device__ inline int n_chunks(const AtlasScanParams& p) { return (p.T + p.chunk - 1) / p.chunk; }

// Linear memory (memory_layer.py:468-494) on the float64 path: forward (bwd = 0) or
// forward recompute + VJP (bwd = 1), one CTA per chain.
struct LinArgs {
  AtlasScanParams p;
  const void *q, *k, *v, *dy;
  const float *alpha, *eta, *theta, *gamma;
  const float *M_in, *S_in, *dM_out, *dS_out;
  void* y;
  float *M_out, *S_out;
  void *dq, *dk, *dv;
  float *dalpha, *deta, *dtheta, *dgamma, *dM_in, *dS_in;
  void* ws;
  int bwd;
};

namespace exact {
size_t lin_workspace_bytes(const AtlasScanParams& p);
cudaError_t lin_launch(const LinArgs& a, cudaStream_t s);
size_t saved_bytes(const AtlasScanParams& p);
size_t workspace_bytes(const AtlasScanParams& p);
cudaError_t launch_fwd(const FwdArgs& a, cudaStream_t s);
cudaError_t launch_bwd(const BwdArgs& a, cudaStream_t s);
cudaError_t launch_pe(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps,
                      void* ws, cudaStream_t s);
size_t pe_workspace_bytes(int64_t batch, int rows, int cols, int steps);
}  // namespace exact

int* device_status_ptr();  // address of the status word on the current device
// Test hooks for the bounded inter-cluster waits (set through
// atlas_debug_set_wait_hooks): the ordering-flag threshold is raised by
// flag_bias (0 in normal use) and the wait gives up after spin_limit polls.
struct WaitHooks {
  int flag_bias;
  int spin_limit;
};
WaitHooks wait_hooks();
int report_error(int code, const char* msg);  // sets atlas_last_error_string(), returns code
void clear_error();                           // atlas_last_error_string() -> ""
int check_scan_params(const AtlasScanParams* p);  // the entry points' parameter checks (sets the message)

// tcgen05 batched Polar Express for large matrices (Muon), pe_tc.cu
namespace tcpe {
size_t workspace_bytes(int64_t batch, int rows, int cols);
cudaError_t launch(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps, void* ws,
                   cudaStream_t s);
}  // namespace tcpe

// Polar Express of D = 128 matrices (E = 256 or 512) on 2-CTA clusters, matrix kept on
// chip across the steps (pe_cluster.cu); tcpe::launch dispatches to it.
namespace pecl {
bool usable(int rows, int cols);
cudaError_t launch(const float* S, float* Y, int64_t batch, int rows, int cols, int steps, float eps,
                   cudaStream_t s);
}  // namespace pecl

// Polar Express of 64 x 256 matrices, two per CTA in flight, on chip across the steps
// (pe_cta.cu); tcpe::launch dispatches to it.
namespace pecta {
bool usable(int rows, int cols);
cudaError_t launch(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps,
                   cudaStream_t s);
}  // namespace pecta

// Shape-generic tensor-path forward (scan_gen.cu): deep memory of any D in
// {32, 64, 128, 256} / E / chunk, and linear memory (memory_layer.py:468-494).
enum { KIND_DEEP = 0, KIND_LINEAR = 1 };
namespace gen {
bool supported(const AtlasScanParams& p, int kind, const char** why);
size_t workspace_bytes(const AtlasScanParams& p, int kind);
cudaError_t launch_fwd(const FwdArgs& a, int kind, cudaStream_t s);
}  // namespace gen

namespace tc {
bool supported(const AtlasScanParams& p, const char** why);      // forward and backward
bool supported_fwd(const AtlasScanParams& p, const char** why);  // forward (also chunk <= 128)
size_t saved_bytes(const AtlasScanParams& p);
size_t workspace_bytes(const AtlasScanParams& p);
cudaError_t launch_fwd(const FwdArgs& a, cudaStream_t s);
cudaError_t launch_bwd(const BwdArgs& a, cudaStream_t s);
}  // namespace tc

}  // namespace atlas
