/*
 * atlas_scan.h -- C ABI of the B200 (sm_100a) Atlas chunked deep-memory scan.
 *
 * This boundary replaces the whole scan of AtlasMemoryLayer.__call__ in
 * rkstgr/atlas-jax (atlas_jax/memory_layer.py:635-718: initial state, padding,
 * lax.scan over jax.checkpoint(chunk_body), un-chunking) together with the
 * inner fused-kernel boundary it dispatches to (fused_chunk_scan_kernel,
 * memory_layer.py:535-541 -> atlas_jax/kernels/fused_chunk.py:321-379, a
 * jax.custom_vjp whose backward is JAX recompute + vjp, fused_chunk.py:366-376).
 * A jax.ffi / XLA custom-call registration binds these entry points one-to-one
 * (the atlas_xla_* adapters below).
 *
 * Conventions
 *  - All buffers are caller-owned DEVICE pointers; no entry point allocates.
 *  - Activations q, k, v, y, dy, dq, dk, dv: row-major (B, T, H, D) in
 *    params->act_dtype (ATLAS_F32 or ATLAS_BF16).
 *  - Gates alpha, eta, theta, gamma and their gradients: (B, T, H) float32, already
 *    activated (sigmoid, eta times max_lr), memory_layer.py:627-633.  gamma may be
 *    NULL (treated as all ones; the reference passes zeros when omega <= 1, which
 *    the window-1 aggregation never reads).
 *  - Memory state (carry), always float32, the reference's naming
 *    (memory_layer.py:106-115): W1, S1 are (B, H, D, E); W2, S2 are (B, H, E, D).
 *  - T need not be a multiple of chunk: padding follows memory_layer.py:649-660
 *    (pad tokens have q=k=v=0, alpha=1, eta=theta=gamma=0), so the final S is 0
 *    when T % chunk != 0, exactly as in the reference.
 *  - stream is a cudaStream_t passed as void*.  Calls are stream-ordered and
 *    asynchronous; a returned ATLAS_OK means "launched".  Device-side failures
 *    (bounded waits that expired) are reported in the status word that
 *    atlas_scan_status() reads after the stream is synchronised.
 *  - Thread safety: any thread may call any entry point.  The error message is
 *    thread-local.  Process-wide state: per-device caches of launch sizes (filled
 *    once under a mutex), the wait-limit test hooks (atomics), and one device
 *    status word per GPU, shared by every stream and thread on that GPU: a
 *    bounded wait that expires in any call sets it, and atlas_scan_status()
 *    reads and clears it for everyone.
 *  - The tensor-path kernels are persistent: a cluster that finishes a (chain,
 *    chunk) item takes the next one from a ticket counter, and waits until the
 *    chain's neighbouring chunk is done.  That chunk always holds a smaller ticket,
 *    taken by a cluster that is already running, so the scan makes progress with
 *    any number of resident clusters: kernels running concurrently on the same GPU
 *    only slow it down.
 */
#ifndef ATLAS_SCAN_H_
#define ATLAS_SCAN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ATLAS_ABI_VERSION 1

/* status codes */
enum {
  ATLAS_OK = 0,
  ATLAS_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, mismatched version */
  ATLAS_ERR_UNSUPPORTED = 2,      /* valid but not implemented for this precision/shape */
  ATLAS_ERR_CUDA = 3,             /* a CUDA runtime call failed */
  ATLAS_ERR_DEVICE_TIMEOUT = 4,   /* a bounded device-side wait expired */
  ATLAS_ERR_WORKSPACE = 5         /* workspace smaller than atlas_scan_workspace_bytes() */
};

/* element types */
enum { ATLAS_F32 = 0, ATLAS_BF16 = 1 };

/* arithmetic used inside the scan */
enum {
  /* float64 CUDA-core arithmetic: reproduces the reference's math well below its
   * own float32 rounding noise.  For parity runs and small shapes. */
  ATLAS_PREC_EXACT = 0,
  /* tcgen05 tensor cores, every Polar Express product on split fp16 operands
   * (hi + lo of a power-of-two multiple of the value, float32 accumulation),
   * float32 carries: as accurate as the reference's float32 arithmetic.  The
   * production path: the fused kernels for D=64, E=256, chunk <= 64 (forward and
   * backward) and 64 < chunk <= 128 (forward only); other shapes run the batched
   * forward below (forward only).  A forward call without saved carries (saved ==
   * NULL, so no backward follows) whose B*H is at most a quarter of the SM count also
   * runs the batched forward: the fused kernels keep one chain per 2-CTA cluster and
   * would leave most SMs idle.  The two paths agree to float32 rounding, not bit for bit. */
  ATLAS_PREC_TENSOR = 1,
  /* Token-parallel batched forward on the tensor cores for any D in {32, 64, 128,
   * 256}, E <= 2048, chunk <= 4096: the chunk's momenta first, then one batched
   * Polar Express of all its matrices (atlas_polar_express_batched's GEMMs), then the
   * memory recurrence and read-out.  Forward only (atlas_scan_bwd refuses it). */
  ATLAS_PREC_TENSOR_BATCHED = 2
};

typedef struct AtlasScanParams {
  int32_t abi_version;      /* must be ATLAS_ABI_VERSION */
  int32_t B, T, H, D, E;    /* batch, sequence, heads, head_dim, memory hidden (E = memory_expand*D) */
  int32_t chunk;            /* config.chunk_size   (config.py:14) */
  int32_t omega;            /* config.omega_window (config.py:17) */
  int32_t ns_steps;         /* config.ns_steps     (config.py:16), 1..5 */
  int32_t pe_ste;           /* config.pe_ste       (config.py:21) */
  int32_t stop_grad_chunks; /* config.stop_grad_chunks (config.py:29) */
  int32_t act_dtype;        /* ATLAS_F32 or ATLAS_BF16 */
  int32_t precision;        /* ATLAS_PREC_EXACT or ATLAS_PREC_TENSOR */
} AtlasScanParams;

/* ABI version of the loaded library. */
int atlas_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* atlas_last_error_string(void);

/* Bytes of the `saved` buffer atlas_scan_fwd fills for atlas_scan_bwd: the
 * float32 carry entering every chunk (the reference recomputes each chunk from
 * its checkpointed carry, memory_layer.py:675). */
size_t atlas_scan_saved_bytes(const AtlasScanParams* p);

/* Bytes of scratch memory the forward / backward need. */
size_t atlas_scan_workspace_bytes(const AtlasScanParams* p);

/* Forward scan.  Replaces memory_layer.py:635-718 (scan part of the layer).
 * state_in may be NULL: the LM-path initial state W1=0, W2=[I;0], S=0 is used
 * (atlas_jax/model.py:251-264).  saved may be NULL when no backward follows. */
int atlas_scan_fwd(const AtlasScanParams* p,
                   const void* q, const void* k, const void* v,
                   const float* alpha, const float* eta, const float* theta, const float* gamma,
                   const float* W1_in, const float* W2_in, const float* S1_in, const float* S2_in,
                   void* y,
                   float* W1_out, float* W2_out, float* S1_out, float* S2_out,
                   void* saved, void* workspace, size_t workspace_bytes, void* stream);

/* Backward scan: the VJP of atlas_scan_fwd, which the reference obtains from
 * JAX autodiff of the checkpointed lax.scan (memory_layer.py:675, 711).
 * dW1_out..dS2_out are the cotangents of the final state (each may be NULL =
 * zero).  dW1_in..dS2_in receive the cotangents of the initial state.
 * `saved` must come from the atlas_scan_fwd call with the same inputs. */
int atlas_scan_bwd(const AtlasScanParams* p,
                   const void* q, const void* k, const void* v,
                   const float* alpha, const float* eta, const float* theta, const float* gamma,
                   const void* saved, const void* dy,
                   const float* dW1_out, const float* dW2_out, const float* dS1_out, const float* dS2_out,
                   void* dq, void* dk, void* dv,
                   float* dalpha, float* deta, float* dtheta, float* dgamma,
                   float* dW1_in, float* dW2_in, float* dS1_in, float* dS2_in,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Forward scan that allocates nothing and takes no workspace, for callers that
 * cannot call cudaMalloc (for example code running inside an allocator or an
 * inference runtime that forbids device allocations after start-up).  It has no
 * counterpart in the reference.  Same arguments and semantics as atlas_scan_fwd
 * without `saved` and `workspace`; tensor path only (params->precision must be
 * ATLAS_PREC_TENSOR).  Its scratch is a fixed 6 MiB array inside the library,
 * enough for B*H <= ATLAS_NOALLOC_MAX_CHAINS; larger problems are rejected with
 * ATLAS_ERR_INVALID_ARGUMENT.  Every GPU that loads the library keeps that array
 * until the process exits.  The first call on a device looks up the array's
 * device address; make that first call before any stream capture.  All calls
 * share the array, so calls whose executions overlap on the GPU (different
 * streams, no ordering between them) race and corrupt each other's results. */
#define ATLAS_NOALLOC_MAX_CHAINS 16
int atlas_scan_fwd_noalloc(const AtlasScanParams* p,
                           const void* q, const void* k, const void* v,
                           const float* alpha, const float* eta, const float* theta, const float* gamma,
                           const float* W1_in, const float* W2_in, const float* S1_in, const float* S2_in,
                           void* y,
                           float* W1_out, float* W2_out, float* S1_out, float* S2_out, void* stream);

/* Linear-memory variant of the scan (AtlasMemoryLayer with deep_memory=False,
 * atlas_jax/memory_layer.py:468-494): memory M (D x D), momentum S, pred = M k,
 * u = (2/D) (pred - v) k^T, Omega window, S_t = theta S_{t-1} - eta G_t,
 * M_t = alpha M_{t-1} + PE(S_t) (square Polar Express), y_t = M_t q_t (no residual).
 * params->E is ignored.  ATLAS_PREC_TENSOR / ATLAS_PREC_TENSOR_BATCHED run the
 * batched tensor-core forward; ATLAS_PREC_EXACT runs float64 on CUDA cores, one CTA
 * per chain (and is the precision of the backward below).  M_in / S_in (B, H, D, D)
 * float32 may both be NULL (zeros, the reference's linear initial state
 * memory_layer.py:138-140).  The workspace size depends on params->precision. */
size_t atlas_linear_scan_workspace_bytes(const AtlasScanParams* p);
int atlas_linear_scan_fwd(const AtlasScanParams* p, const void* q, const void* k, const void* v,
                          const float* alpha, const float* eta, const float* theta, const float* gamma,
                          const float* M_in, const float* S_in, void* y, float* M_out, float* S_out,
                          void* workspace, size_t workspace_bytes, void* stream);

/* VJP of atlas_linear_scan_fwd (JAX autodiff of memory_layer.py:468-494 under the
 * scan driver 649-718): recomputes the forward from (M_in, S_in) and returns dq, dk,
 * dv (act_dtype), the gate gradients (B, T, H) float32 (dgamma may be NULL) and the
 * initial-state cotangents dM_in, dS_in (may be NULL).  dy, dM_out, dS_out NULL mean
 * zero cotangents.  params->precision must be ATLAS_PREC_EXACT; the workspace is
 * atlas_linear_scan_workspace_bytes() of the same params. */
int atlas_linear_scan_bwd(const AtlasScanParams* p, const void* q, const void* k, const void* v,
                          const float* alpha, const float* eta, const float* theta, const float* gamma,
                          const float* M_in, const float* S_in, const void* dy, const float* dM_out,
                          const float* dS_out, void* dq, void* dk, void* dv, float* dalpha, float* deta,
                          float* dtheta, float* dgamma, float* dM_in, float* dS_in, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Batched Polar Express on float32 (batch, rows, cols) matrices, out-of-place.
 * Replaces fused_polar_express (atlas_jax/kernels/triton_pe.py:26-69, same math
 * as memory_layer.py:43-71) and the Muon orthogonalisation call site
 * (atlas_jax/optim.py:68-83, which omits the 1e-12 inside the square root:
 * pass eps_in_sqrt = 0 for that behaviour, 1e-12 for the memory layer's).
 * precision: ATLAS_PREC_EXACT runs float64 on CUDA cores, one CTA per matrix (small
 * matrices, parity checks); ATLAS_PREC_TENSOR runs each Newton-Schulz step as three
 * batched tcgen05 GEMMs on split fp16 operands (large matrices such as
 * Muon's stacked parameter gradients). */
int atlas_polar_express_batched(const float* X, float* Y, int64_t batch, int32_t rows, int32_t cols,
                                int32_t ns_steps, float eps_in_sqrt, int32_t precision,
                                void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes atlas_polar_express_batched needs for this problem. */
size_t atlas_polar_express_workspace_bytes(int64_t batch, int32_t rows, int32_t cols, int32_t ns_steps,
                                           int32_t precision);

/* XLA custom-call adapters (status-returning legacy signature, api_version 2):
 *   void fn(cudaStream_t stream, void** buffers, const char* opaque, size_t opaque_len,
 *           XlaCustomCallStatus* status)
 * `opaque` is one packed AtlasScanParams (atlas_xla_opaque_bytes() bytes).  They are
 * the jax.ffi registration targets that replace the custom-VJP pair
 * fused_chunk_scan_kernel (atlas_jax/kernels/fused_chunk.py:321-379, called at
 * atlas_jax/memory_layer.py:535-541) with the whole scan (memory_layer.py:635-718).
 * Failures go to XlaCustomCallStatusSetFailure when the process exports it and to
 * atlas_last_error_string() of the calling thread.
 *
 * atlas_xla_fwd buffers (operands, then results):
 *   0 q  1 k  2 v  3 alpha  4 eta  5 theta  6 gamma  7 W1_in  8 W2_in  9 S1_in  10 S2_in
 *   11 y  12 W1_out  13 W2_out  14 S1_out  15 S2_out  16 saved  17 workspace
 * atlas_xla_bwd buffers:
 *   0 q  1 k  2 v  3 alpha  4 eta  5 theta  6 gamma  7 saved  8 dy
 *   9 dW1_out  10 dW2_out  11 dS1_out  12 dS2_out
 *   13 dq  14 dk  15 dv  16 dalpha  17 deta  18 dtheta  19 dgamma
 *   20 dW1_in  21 dW2_in  22 dS1_in  23 dS2_in  24 workspace
 * Every buffer is present (gamma all ones when unused, the initial state explicit,
 * zero final-state cotangents); saved / workspace have atlas_scan_saved_bytes() /
 * atlas_scan_workspace_bytes() bytes. */
size_t atlas_xla_opaque_bytes(void);
void atlas_xla_fwd(void* stream, void** buffers, const char* opaque, size_t opaque_len, void* status);
void atlas_xla_bwd(void* stream, void** buffers, const char* opaque, size_t opaque_len, void* status);

/* XLA adapter of atlas_polar_express_batched, the target that replaces the Muon
 * orthogonalisation of atlas_jax/optim.py:68-83.  Buffers: 0 X, 1 Y, 2 workspace
 * (atlas_polar_express_workspace_bytes()).  `opaque` is the packed struct
 *   { int64 batch; int32 rows, cols, ns_steps, precision; float eps_in_sqrt; int32 pad; }
 * of atlas_xla_pe_opaque_bytes() bytes. */
size_t atlas_xla_pe_opaque_bytes(void);
void atlas_xla_polar_express(void* stream, void** buffers, const char* opaque, size_t opaque_len, void* status);

/* Reads and clears the device status word of the calling device after the
 * caller synchronised the stream (ATLAS_OK or ATLAS_ERR_DEVICE_TIMEOUT). */
int atlas_scan_status(void);

#ifdef __cplusplus
}
#endif

#endif /* ATLAS_SCAN_H_ */
