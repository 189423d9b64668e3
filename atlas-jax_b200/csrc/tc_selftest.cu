// One-CTA tcgen05 GEMM used only to validate descriptor and TMEM layouts.
#include <cuda_bf16.h>

#include "atlas_selftest.h"
#include "tc_ops.cuh"

namespace atlas {
namespace {
using namespace tcx;

__global__ void selftest_gemm(const float* A, const float* B, float* D, int M, int N, int K, int amn, int bmn) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  uint8_t* sA = sm;                    // A tile
  uint8_t* sB = sm + M * K * 2;        // B tile
  // A: K-major tile rows=m cols=k ; MN-major tile rows=k cols=m
  for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
    int m = i / K, k = i % K;
    uint32_t off = amn ? cm_off(k, m, M) : cm_off(m, k, K);
    *(__nv_bfloat16*)(sA + off) = __float2bfloat16_rn(A[i]);
  }
  for (int i = threadIdx.x; i < K * N; i += blockDim.x) {
    int k = i / N, n = i % N;
    uint32_t off = bmn ? cm_off(k, n, N) : cm_off(n, k, K);
    *(__nv_bfloat16*)(sB + off) = __float2bfloat16_rn(B[i]);
  }
  fence_async_smem();
  if (threadIdx.x < 32) {
    tmem_alloc(&tbase, 256);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  fence_before();
  __syncthreads();
  fence_after();
  uint32_t tm = tbase;
  if (threadIdx.x < 32) {  // one warp issues (elected lane)
    uint32_t id = idesc_bf16(M, N, amn, bmn);
    for (int kb = 0; kb < K / 16; ++kb) {
      // advance two core matrices along K
      uint32_t aoff = amn ? (uint32_t)(kb * 2) * (M * 16) : (uint32_t)kb * 256;
      uint32_t boff = bmn ? (uint32_t)(kb * 2) * (N * 16) : (uint32_t)kb * 256;
      uint64_t da = amn ? desc_mnmajor(smem_u32(sA) + aoff, M) : desc_kmajor(smem_u32(sA) + aoff, K);
      uint64_t db = bmn ? desc_mnmajor(smem_u32(sB) + boff, N) : desc_kmajor(smem_u32(sB) + boff, K);
      mma_kf16(tm, da, db, id, kb > 0);
    }
    mma_commit(&bar);
  }
  __syncwarp();
  bool ok = mbar_wait(&bar, 0);
  fence_after();
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  // row held by this thread's lane
  int lane = w * 32 + l;
  int row = (M == 128) ? lane : ((l < 16) ? (w * 16 + l) : -1);
  for (int c0 = 0; c0 < N; c0 += 16) {
    float v[16];
    tmem_ld16(tm + ((uint32_t)(w * 32) << 16) + c0, v);
    tmem_wait_ld();
    if (row >= 0 && ok)
      for (int j = 0; j < 16; ++j) D[row * N + c0 + j] = v[j];
  }
  fence_before();
  __syncthreads();
  if (threadIdx.x < 32) tmem_dealloc(tm, 256);
}
}  // namespace
}  // namespace atlas

extern "C" int atlas_selftest_tc_gemm(const float* A, const float* B, float* D, int32_t M, int32_t N, int32_t K,
                                      int32_t a_mn_major, int32_t b_mn_major, void* stream) {
  if ((M != 64 && M != 128) || N < 16 || N > 256 || N % 16 || K < 16 || K > 256 || K % 16) return 1;
  size_t smem = (size_t)(M * K + K * N) * 2;
  cudaFuncSetAttribute(atlas::selftest_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  atlas::selftest_gemm<<<1, 128, smem, (cudaStream_t)stream>>>(A, B, D, M, N, K, a_mn_major, b_mn_major);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

