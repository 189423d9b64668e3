// C ABI entry points (include/atlas_scan.h): argument checks, dispatch to the
// exact or the tcgen05 implementation, error reporting.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"
#include "scan_internal.h"
#include "atlas_selftest.h"

namespace atlas {
__device__ int g_status = 0;

int* device_status_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
  return (int*)p;
}
// test hooks of the bounded waits (atlas_debug_set_wait_hooks), read at every launch
static std::atomic<int> g_flag_bias{0}, g_spin_limit{50000000};
WaitHooks wait_hooks() { return WaitHooks{g_flag_bias.load(), g_spin_limit.load()}; }
void set_wait_hooks(int bias, int limit) {
  g_flag_bias.store(bias);
  g_spin_limit.store(limit > 0 ? limit : 50000000);
}
}  // namespace atlas

namespace {
thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

// Which tensor-path implementation serves a valid TENSOR / TENSOR_BATCHED problem.
enum Impl { IMPL_EXACT, IMPL_FUSED, IMPL_BATCHED };
Impl impl_of(const AtlasScanParams& p) {
  if (p.precision == ATLAS_PREC_EXACT) return IMPL_EXACT;
  const char* why = "";
  if (p.precision == ATLAS_PREC_TENSOR && atlas::tc::supported_fwd(p, &why)) return IMPL_FUSED;
  return IMPL_BATCHED;
}

// A forward-only ATLAS_PREC_TENSOR call (saved == NULL) with few chains runs the batched
// forward: the fused kernels run one chain per 2-CTA cluster, so with fewer chains than
// about half the clusters most SMs idle, while the batched forward spreads every chunk's
// tokens over the whole GPU.  Calls that keep `saved` for a backward stay on the fused path,
// whose carries the backward reads.
atlas::DeviceCache g_sms;  // multiprocessors per device

bool few_chains(const AtlasScanParams& p) {
  const char* why = "";
  const int sms = g_sms.get([] {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        n <= 0)
      n = 148;
    return n;
  });
  return (long)p.B * p.H * 4 <= (long)sms &&
         atlas::gen::supported(p, atlas::KIND_DEEP, &why);
}

// dir: 0 = forward (and the size queries), 1 = backward
int check_params(const AtlasScanParams* p, int dir = 0) {
  if (!p) return fail(ATLAS_ERR_INVALID_ARGUMENT, "params is NULL");
  if (p->abi_version != ATLAS_ABI_VERSION)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "abi_version %d != library %d", p->abi_version, ATLAS_ABI_VERSION);
  if (p->B <= 0 || p->T <= 0 || p->H <= 0 || p->D <= 0 || p->E <= 0 || p->chunk <= 0)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "B, T, H, D, E and chunk must be positive");
  if (p->omega < 1) return fail(ATLAS_ERR_INVALID_ARGUMENT, "omega must be >= 1");
  if (p->ns_steps < 0 || p->ns_steps > 5) return fail(ATLAS_ERR_INVALID_ARGUMENT, "ns_steps must be in 0..5");
  if (p->act_dtype != ATLAS_F32 && p->act_dtype != ATLAS_BF16)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "act_dtype must be ATLAS_F32 or ATLAS_BF16");
  if (p->precision != ATLAS_PREC_EXACT && p->precision != ATLAS_PREC_TENSOR &&
      p->precision != ATLAS_PREC_TENSOR_BATCHED)
    return fail(ATLAS_ERR_INVALID_ARGUMENT,
                "precision must be ATLAS_PREC_EXACT, ATLAS_PREC_TENSOR or ATLAS_PREC_TENSOR_BATCHED");
  if (p->precision != ATLAS_PREC_EXACT) {
    const char* why = "";
    const bool fused = p->precision == ATLAS_PREC_TENSOR &&
                       (dir == 1 ? atlas::tc::supported(*p, &why) : atlas::tc::supported_fwd(*p, &why));
    if (dir == 1 && !fused)
      return fail(ATLAS_ERR_UNSUPPORTED,
                  "tensor path: the backward needs D=64, E=256, chunk<=64 and ATLAS_PREC_TENSOR (%s); "
                  "ATLAS_PREC_EXACT covers other shapes",
                  p->precision == ATLAS_PREC_TENSOR ? why : "batched forward has no backward");
    const char* why2 = "";
    if (!fused && !atlas::gen::supported(*p, atlas::KIND_DEEP, &why2))
      return fail(ATLAS_ERR_UNSUPPORTED, "tensor path: %s", why2);
  }
  return ATLAS_OK;
}

int cuda_result(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(ATLAS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ATLAS_OK;
}
}  // namespace

int atlas::report_error(int code, const char* msg) { return fail(code, "%s", msg); }
void atlas::clear_error() { g_err.clear(); }
int atlas::check_scan_params(const AtlasScanParams* p) { return check_params(p); }

extern "C" {

int atlas_abi_version(void) { return ATLAS_ABI_VERSION; }

const char* atlas_last_error_string(void) { return g_err.c_str(); }

size_t atlas_scan_saved_bytes(const AtlasScanParams* p) {
  if (check_params(p) != ATLAS_OK) return 0;
  switch (impl_of(*p)) {
    case IMPL_EXACT: return atlas::exact::saved_bytes(*p);
    case IMPL_FUSED: return atlas::tc::saved_bytes(*p);
    default: return 256;  // the batched forward keeps no carries (it has no backward)
  }
}

size_t atlas_scan_workspace_bytes(const AtlasScanParams* p) {
  if (check_params(p) != ATLAS_OK) return 0;
  switch (impl_of(*p)) {
    case IMPL_EXACT: return atlas::exact::workspace_bytes(*p);
    case IMPL_FUSED:  // also sized for the batched forward that forward-only calls with few chains take
      return few_chains(*p) ? std::max(atlas::tc::workspace_bytes(*p), atlas::gen::workspace_bytes(*p, atlas::KIND_DEEP))
                            : atlas::tc::workspace_bytes(*p);
    default: return atlas::gen::workspace_bytes(*p, atlas::KIND_DEEP);
  }
}

int atlas_scan_fwd(const AtlasScanParams* p, const void* q, const void* k, const void* v, const float* alpha,
                   const float* eta, const float* theta, const float* gamma, const float* W1_in,
                   const float* W2_in, const float* S1_in, const float* S2_in, void* y, float* W1_out,
                   float* W2_out, float* S1_out, float* S2_out, void* saved, void* workspace,
                   size_t workspace_bytes, void* stream) {
  g_err.clear();
  int rc = check_params(p);
  if (rc) return rc;
  if (!q || !k || !v || !alpha || !eta || !theta || !y)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "q, k, v, alpha, eta, theta and y must be non-NULL");
  if ((W1_in || W2_in || S1_in || S2_in) && !(W1_in && W2_in && S1_in && S2_in))
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "state_in must be all NULL or all non-NULL");
  size_t need = atlas_scan_workspace_bytes(p);
  if (need && (!workspace || workspace_bytes < need))
    return fail(ATLAS_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  atlas::FwdArgs a;
  a.p = *p;
  a.q = q; a.k = k; a.v = v;
  a.alpha = alpha; a.eta = eta; a.theta = theta; a.gamma = gamma;
  a.W1_in = W1_in; a.W2_in = W2_in; a.S1_in = S1_in; a.S2_in = S2_in;
  a.y = y;
  a.W1_out = W1_out; a.W2_out = W2_out; a.S1_out = S1_out; a.S2_out = S2_out;
  a.saved = saved;
  a.ws = workspace;
  a.status = atlas::device_status_ptr();
  cudaStream_t s = (cudaStream_t)stream;
  Impl im = impl_of(*p);
  if (im == IMPL_FUSED && !saved && few_chains(*p)) im = IMPL_BATCHED;
  cudaError_t e = im == IMPL_EXACT   ? atlas::exact::launch_fwd(a, s)
                  : im == IMPL_FUSED ? atlas::tc::launch_fwd(a, s)
                                     : atlas::gen::launch_fwd(a, atlas::KIND_DEEP, s);
  return cuda_result(e, "atlas_scan_fwd launch");
}

int atlas_scan_bwd(const AtlasScanParams* p, const void* q, const void* k, const void* v, const float* alpha,
                   const float* eta, const float* theta, const float* gamma, const void* saved, const void* dy,
                   const float* dW1_out, const float* dW2_out, const float* dS1_out, const float* dS2_out,
                   void* dq, void* dk, void* dv, float* dalpha, float* deta, float* dtheta, float* dgamma,
                   float* dW1_in, float* dW2_in, float* dS1_in, float* dS2_in, void* workspace,
                   size_t workspace_bytes, void* stream) {
  g_err.clear();
  int rc = check_params(p, 1);
  if (rc) return rc;
  if (!q || !k || !v || !alpha || !eta || !theta || !saved || !dy || !dq || !dk || !dv)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "q, k, v, gates, saved, dy, dq, dk, dv must be non-NULL");
  size_t need = atlas_scan_workspace_bytes(p);
  if (need && (!workspace || workspace_bytes < need))
    return fail(ATLAS_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  atlas::BwdArgs a;
  a.p = *p;
  a.q = q; a.k = k; a.v = v;
  a.alpha = alpha; a.eta = eta; a.theta = theta; a.gamma = gamma;
  a.saved = saved; a.dy = dy;
  a.dW1_out = dW1_out; a.dW2_out = dW2_out; a.dS1_out = dS1_out; a.dS2_out = dS2_out;
  a.dq = dq; a.dk = dk; a.dv = dv;
  a.dalpha = dalpha; a.deta = deta; a.dtheta = dtheta; a.dgamma = dgamma;
  a.dW1_in = dW1_in; a.dW2_in = dW2_in; a.dS1_in = dS1_in; a.dS2_in = dS2_in;
  a.ws = workspace;
  a.status = atlas::device_status_ptr();
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = p->precision == ATLAS_PREC_EXACT ? atlas::exact::launch_bwd(a, s) : atlas::tc::launch_bwd(a, s);
  return cuda_result(e, "atlas_scan_bwd launch");
}

}  // extern "C"

namespace {
int linear_check(const AtlasScanParams* p, size_t* need) {
  *need = 0;
  int rc = check_params(p);
  if (rc) return rc;
  if (p->precision == ATLAS_PREC_EXACT) {
    *need = atlas::exact::lin_workspace_bytes(*p);
    return ATLAS_OK;
  }
  const char* why = "";
  if (!atlas::gen::supported(*p, atlas::KIND_LINEAR, &why)) return fail(ATLAS_ERR_UNSUPPORTED, "linear memory: %s", why);
  *need = atlas::gen::workspace_bytes(*p, atlas::KIND_LINEAR);
  return ATLAS_OK;
}
}  // namespace

extern "C" {

size_t atlas_linear_scan_workspace_bytes(const AtlasScanParams* p) {
  size_t need = 0;
  linear_check(p, &need);
  return need;
}

int atlas_linear_scan_fwd(const AtlasScanParams* p, const void* q, const void* k, const void* v,
                          const float* alpha, const float* eta, const float* theta, const float* gamma,
                          const float* M_in, const float* S_in, void* y, float* M_out, float* S_out,
                          void* workspace, size_t workspace_bytes, void* stream) {
  g_err.clear();
  size_t need = 0;
  int rc = linear_check(p, &need);
  if (rc) return rc;
  if (!q || !k || !v || !alpha || !eta || !theta || !y)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "q, k, v, alpha, eta, theta and y must be non-NULL");
  if ((M_in == nullptr) != (S_in == nullptr))
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "M_in and S_in must be both NULL or both non-NULL");
  if (!workspace || workspace_bytes < need)
    return fail(ATLAS_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  atlas::FwdArgs a{};
  a.p = *p;
  a.q = q; a.k = k; a.v = v;
  a.alpha = alpha; a.eta = eta; a.theta = theta; a.gamma = gamma;
  a.W1_in = M_in; a.S1_in = S_in;
  a.y = y;
  a.W1_out = M_out; a.S1_out = S_out;
  a.ws = workspace;
  a.status = atlas::device_status_ptr();
  if (p->precision == ATLAS_PREC_EXACT) {
    atlas::LinArgs la{};
    la.p = *p;
    la.q = q; la.k = k; la.v = v;
    la.alpha = alpha; la.eta = eta; la.theta = theta; la.gamma = gamma;
    la.M_in = M_in; la.S_in = S_in;
    la.y = y; la.M_out = M_out; la.S_out = S_out;
    la.ws = workspace;
    la.bwd = 0;
    return cuda_result(atlas::exact::lin_launch(la, (cudaStream_t)stream), "atlas_linear_scan_fwd launch (exact)");
  }
  return cuda_result(atlas::gen::launch_fwd(a, atlas::KIND_LINEAR, (cudaStream_t)stream),
                     "atlas_linear_scan_fwd launch");
}

int atlas_linear_scan_bwd(const AtlasScanParams* p, const void* q, const void* k, const void* v,
                          const float* alpha, const float* eta, const float* theta, const float* gamma,
                          const float* M_in, const float* S_in, const void* dy, const float* dM_out,
                          const float* dS_out, void* dq, void* dk, void* dv, float* dalpha, float* deta,
                          float* dtheta, float* dgamma, float* dM_in, float* dS_in, void* workspace,
                          size_t workspace_bytes, void* stream) {
  g_err.clear();
  if (p && p->precision != ATLAS_PREC_EXACT)
    return fail(ATLAS_ERR_UNSUPPORTED, "the linear-memory backward runs on ATLAS_PREC_EXACT");
  size_t need = 0;
  int rc = linear_check(p, &need);
  if (rc) return rc;
  if (!q || !k || !v || !alpha || !eta || !theta || !dq || !dk || !dv || !dalpha || !deta || !dtheta)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "inputs, dq, dk, dv and the gate gradients must be non-NULL");
  if ((M_in == nullptr) != (S_in == nullptr))
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "M_in and S_in must be both NULL or both non-NULL");
  if (!workspace || workspace_bytes < need)
    return fail(ATLAS_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  atlas::LinArgs la{};
  la.p = *p;
  la.q = q; la.k = k; la.v = v; la.dy = dy;
  la.alpha = alpha; la.eta = eta; la.theta = theta; la.gamma = gamma;
  la.M_in = M_in; la.S_in = S_in; la.dM_out = dM_out; la.dS_out = dS_out;
  la.dq = dq; la.dk = dk; la.dv = dv;
  la.dalpha = dalpha; la.deta = deta; la.dtheta = dtheta; la.dgamma = dgamma;
  la.dM_in = dM_in; la.dS_in = dS_in;
  la.ws = workspace;
  la.bwd = 1;
  return cuda_result(atlas::exact::lin_launch(la, (cudaStream_t)stream), "atlas_linear_scan_bwd launch");
}

size_t atlas_polar_express_workspace_bytes(int64_t batch, int32_t rows, int32_t cols, int32_t ns_steps,
                                           int32_t precision) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  if (precision == ATLAS_PREC_TENSOR) return atlas::tcpe::workspace_bytes(batch, rows, cols);
  return atlas::exact::pe_workspace_bytes(batch, rows, cols, ns_steps);
}

int atlas_polar_express_batched(const float* X, float* Y, int64_t batch, int32_t rows, int32_t cols,
                                int32_t ns_steps, float eps_in_sqrt, int32_t precision, void* workspace,
                                size_t workspace_bytes, void* stream) {
  g_err.clear();
  if (!X || !Y) return fail(ATLAS_ERR_INVALID_ARGUMENT, "X and Y must be non-NULL");
  if (batch <= 0 || rows <= 0 || cols <= 0) return fail(ATLAS_ERR_INVALID_ARGUMENT, "empty problem");
  if (ns_steps < 0 || ns_steps > 5) return fail(ATLAS_ERR_INVALID_ARGUMENT, "ns_steps must be in 0..5");
  if (precision != ATLAS_PREC_EXACT && precision != ATLAS_PREC_TENSOR)
    return fail(ATLAS_ERR_INVALID_ARGUMENT, "precision must be ATLAS_PREC_EXACT or ATLAS_PREC_TENSOR");
  size_t need = atlas_polar_express_workspace_bytes(batch, rows, cols, ns_steps, precision);
  if (!workspace || workspace_bytes < need)
    return fail(ATLAS_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (precision == ATLAS_PREC_TENSOR)
    return cuda_result(atlas::tcpe::launch(X, Y, batch, rows, cols, ns_steps, eps_in_sqrt, workspace,
                                           (cudaStream_t)stream),
                       "atlas_polar_express_batched launch (tensor)");
  return cuda_result(atlas::exact::launch_pe(X, Y, batch, rows, cols, ns_steps, eps_in_sqrt, workspace,
                                             (cudaStream_t)stream),
                     "atlas_polar_express_batched launch");
}

int atlas_debug_set_wait_hooks(int32_t flag_bias, int32_t spin_limit) {
  atlas::set_wait_hooks(flag_bias, spin_limit);
  return ATLAS_OK;
}

int atlas_scan_status(void) {
  int h = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&h, atlas::g_status, sizeof(int));
  if (e != cudaSuccess) return fail(ATLAS_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
  cudaMemcpyToSymbol(atlas::g_status, &zero, sizeof(int));
  if (h) fail(h, "device-side wait expired");
  return h;
}

}  // extern "C"
