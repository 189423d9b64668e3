/*
 * atlas_selftest.h -- diagnostic entry point of libatlas_scan.so (not part of
 * the reference's interface; used by the GPU tests to validate the tcgen05
 * operand layouts the scan kernels rely on).
 */
#ifndef ATLAS_SELFTEST_H_
#define ATLAS_SELFTEST_H_
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* D (M x N, float32) = A (M x K) @ B (K x N) computed by one CTA with
 * tcgen05.mma kind::f16 (operands rounded to bf16, float32 accumulation).
 * M in {64, 128}; N a multiple of 16 in [16, 256]; K a multiple of 16 <= 256.
 * a_mn_major / b_mn_major choose the shared-memory operand orientation.
 * All pointers are device pointers; returns 0 on success. */
int atlas_selftest_tc_gemm(const float* A, const float* B, float* D, int32_t M, int32_t N, int32_t K,
                           int32_t a_mn_major, int32_t b_mn_major, void* stream);

/* Failure-detection test hook for the bounded device-side waits of the tensor
 * path: every chunk-ordering wait requires its counter to exceed the normal
 * threshold by `flag_bias` (a value nothing ever reaches when > 0) and gives up
 * after `spin_limit` polls (<= 0 restores the default).  A forward or backward
 * launched with flag_bias > 0 therefore reports ATLAS_ERR_DEVICE_TIMEOUT through
 * atlas_scan_status() instead of hanging.  Affects later launches from this
 * process; reset with (0, 0). */
int atlas_debug_set_wait_hooks(int32_t flag_bias, int32_t spin_limit);

#ifdef __cplusplus
}
#endif
#endif
