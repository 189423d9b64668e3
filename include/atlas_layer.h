/*
 * atlas_layer.h -- C ABI of the fused prologue and epilogue around the Atlas scan.
 *
 * They replace the per-layer elementwise ops that AtlasMemoryLayer.__call__ runs
 * before and after the scan (rkstgr/atlas-jax, atlas_jax/memory_layer.py):
 *   prologue  606-633: ShortConv of the q/k/v projections (memory_layer.py:303-329),
 *             rms_norm (211-216) and the polynomial feature map (455-462) of q and
 *             k, and the sigmoid gates alpha, eta * max_lr, theta, gamma, plus the
 *             retrieve gate's sigmoid (720-722);
 *   epilogue  720-722: y * sigmoid(retrieve) before c_proj.
 * The projections themselves (x @ [c_q; c_k; c_v; gate_*; retrieve_gate]^T and
 * c_proj) are plain GEMMs and stay with the caller's GEMM library: the prologue
 * reads their one concatenated output, so the layer makes one GEMM, one prologue
 * launch and one scan call where the reference makes ~20 XLA ops with HBM
 * round trips between them.
 *
 * Layout.  x's projection "proj" is row-major (B*T, NP), NP = 3*H*D + G*H (rows
 * proj_stride >= NP elements apart, extra columns ignored), in act_dtype, with columns
 *   [ q (H*D) | k (H*D) | v (H*D) | alpha (H) | eta (H) | theta (H) | gamma (H, if has_gamma)
 *     | retrieve (H, if has_retrieve) ]
 * (G = 3 + has_gamma + has_retrieve).  The pre-activation gate columns do not
 * include the gate biases; gate_bias holds them, (G-has_retrieve) x H float32, in
 * the same gate order (the retrieve gate has no bias, memory_layer.py:455-456).
 * conv_w is (3, K, H*D) float32, tap-major: the q, k, v convolutions' (dim, 1, K)
 * reference weights stacked and transposed, so one tap of consecutive channels is
 * contiguous; conv_b (3, H*D), poly (poly_degree) float32.
 * Outputs: q, k, v (B, T, H, D) in act_dtype; alpha, eta, theta, gamma, retrieve
 * (B, T, H) float32, activated.  Pointers of absent gates may be NULL.
 *
 * Arithmetic is float32 throughout; act_dtype outputs are rounded once at the end.
 * Conventions (status codes, thread-local error string, stream as void*) are those
 * of atlas_scan.h.
 */
#ifndef ATLAS_LAYER_H_
#define ATLAS_LAYER_H_

#include <stddef.h>
#include <stdint.h>

#include "atlas_scan.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int32_t abi_version; /* ATLAS_ABI_VERSION */
  int32_t B, T, H, D;
  int32_t conv_kernel;  /* ShortConv kernel size K (config.conv_kernel), 1..8 */
  int32_t poly_degree;  /* 0 = plain rms_norm of q and k; else 1..4 */
  int32_t has_gamma;    /* omega_window > 1 */
  int32_t has_retrieve; /* n_head > 1 */
  int32_t act_dtype;    /* ATLAS_F32 or ATLAS_BF16: proj, q, k, v, dproj, dq, dk, dv */
  int32_t proj_stride;  /* elements between rows of proj / dproj (0 = NP); a multiple of 8
                         * (bf16) or 4 (f32) lets the kernels move 16 bytes per lane */
  float max_lr;         /* eta = sigmoid(.) * max_lr */
} AtlasLayerParams;

/* Bytes of workspace atlas_layer_prologue_bwd needs (0 on invalid params). */
size_t atlas_layer_prologue_workspace_bytes(const AtlasLayerParams* p);

/* Forward prologue.  Replaces memory_layer.py:606-633 after the projections. */
int atlas_layer_prologue_fwd(const AtlasLayerParams* p, const void* proj, const float* conv_w,
                             const float* conv_b, const float* poly, const float* gate_bias, void* q, void* k,
                             void* v, float* alpha, float* eta, float* theta, float* gamma, float* retrieve,
                             void* stream);

/* VJP of atlas_layer_prologue_fwd.  Inputs: the forward's inputs and the cotangents of
 * its outputs (dgamma / dretrieve may be NULL when absent; NULL cotangents count as
 * zero).  Outputs: dproj (B*T, NP) in act_dtype (absent gates' columns are written 0),
 * and the parameter gradients dconv_w (3, K, H*D), dconv_b (3, H*D), dpoly
 * (poly_degree), dgate_bias (G - has_retrieve, H), all float32 and OVERWRITTEN. */
int atlas_layer_prologue_bwd(const AtlasLayerParams* p, const void* proj, const float* conv_w,
                             const float* conv_b, const float* poly, const float* gate_bias, const void* dq,
                             const void* dk, const void* dv, const float* dalpha, const float* deta,
                             const float* dtheta, const float* dgamma, const float* dretrieve, void* dproj,
                             float* dconv_w, float* dconv_b, float* dpoly, float* dgate_bias, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Epilogue: yg = y * retrieve[..., None], y and yg (B, T, H, D) act_dtype, retrieve
 * (B, T, H) float32 activated.  Replaces memory_layer.py:720-722. */
int atlas_layer_retrieve_fwd(const AtlasLayerParams* p, const void* y, const float* retrieve, void* yg,
                             void* stream);

/* VJP: dy = dyg * retrieve, dretrieve = sum_d dyg * y (float32). */
int atlas_layer_retrieve_bwd(const AtlasLayerParams* p, const void* y, const float* retrieve, const void* dyg,
                             void* dy, float* dretrieve, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ATLAS_LAYER_H_ */
