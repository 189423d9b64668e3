/*
 * atlas_swa.h -- C ABI of the banded (sliding-window) causal attention of the MAG
 * hybrid (rkstgr/atlas-jax, atlas_jax/model.py:77-135, used by
 * atlas_jax/mag_transformer.py:22-80).
 *
 * Replaces the attention core of SlidingWindowAttention.__call__ (model.py:117-133):
 * RoPE on q and k (model.py:49-75, 117-121: inv_freq = 10000^(-2i/D), halves
 * rotated), scores q.k / sqrt(D), mask key <= query and query - key <= window
 * (model.py:126-130), float32 softmax, and the weighted sum of v.  The reference
 * materialises the dense T x T score matrix; these kernels visit only the band
 * (window + 1 keys per query) in 128 x 128 tiles on the tcgen05 tensor cores with an
 * online softmax, so memory is O(T).  rms_norm, to_qkv and to_out stay with the
 * caller (plain GEMMs).
 *
 * Layout: q, k, v, o and their gradients are (B, T, H, D) bfloat16, row-major, q and k
 * BEFORE RoPE (the raw projections); lse is (B, H, T) float32 (log-sum-exp of each
 * query's scaled scores, saved by the forward for the backward).  D = 64.
 * Arithmetic: bf16 operands, float32 accumulation and softmax; the probabilities
 * are rounded to bf16 before the value product (the reference rounds them to the
 * activation dtype too, model.py:131).
 * Conventions (status codes, thread-local error string, stream as void*) are those
 * of atlas_scan.h.
 */
#ifndef ATLAS_SWA_H_
#define ATLAS_SWA_H_

#include <stddef.h>
#include <stdint.h>

#include "atlas_scan.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int32_t abi_version; /* ATLAS_ABI_VERSION */
  int32_t B, T, H, D;  /* D must be 64 */
  int32_t window;      /* keys with 0 <= query - key <= window attend (config.window_size) */
  int32_t rope;        /* 1: apply RoPE to q and k inside the kernels (the reference); 0: q, k as given */
} AtlasSwaParams;

/* Workspace of both calls: the rotated q and k (bf16) and B*H*T float32 (the
 * per-query dO.o sums of the backward). */
size_t atlas_swa_workspace_bytes(const AtlasSwaParams* p);

/* Forward: o (B,T,H,D) bf16 and lse (B,H,T) float32. */
int atlas_swa_fwd(const AtlasSwaParams* p, const void* q, const void* k, const void* v, void* o, float* lse,
                  void* workspace, size_t workspace_bytes, void* stream);

/* VJP: dq, dk (with respect to the pre-RoPE q, k), dv, all (B,T,H,D) bf16. */
int atlas_swa_bwd(const AtlasSwaParams* p, const void* q, const void* k, const void* v, const void* o,
                  const float* lse, const void* dout, void* dq, void* dk, void* dv, void* workspace,
                  size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ATLAS_SWA_H_ */
