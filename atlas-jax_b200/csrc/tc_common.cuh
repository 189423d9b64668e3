// Shared pieces of the tcgen05 scan kernels (forward and backward).
#pragma once
#include <cuda_bf16.h>

#include "common.cuh"
#include "tc_ops.cuh"

namespace atlas {
namespace tc {
using namespace tcx;

constexpr int D = 64;
constexpr int E = 256;
constexpr int NT = 256;      // 8 warps: warp w -> TMEM lane quadrant w % 4, column half w / 4
constexpr int MAXCS = 64;
constexpr int DE = D * E;
constexpr int XT_BYTES = E * D * 2;  // bf16 E x D tile
constexpr int AT_BYTES = D * D * 2;  // bf16 D x D tile
constexpr int TMEM_COLS = 256;
// TMEM column map
constexpr uint32_t TM_X = 0;      // X~ update: rows 0-127 in cols [0,64), rows 128-255 in [64,128)
constexpr uint32_t TM_GRAM = 128; // Gram A (M=64 layout)
constexpr uint32_t TM_A2 = 192;   // A*A    (M=64 layout)

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_remote_f32(const float* local_addr, uint32_t rank, float v) {
  uint32_t la = smem_u32(local_addr), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Split 8 consecutive float32 values into bf16 hi and lo parts and store them
// as one 16-byte core-matrix row segment in each tile.
__device__ __forceinline__ void store_split8(uint8_t* th, uint8_t* tl, uint32_t off, const float* v) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * k]);
    __nv_bfloat16 h1 = __float2bfloat16_rn(v[2 * k + 1]);
    __nv_bfloat16 l0 = __float2bfloat16_rn(v[2 * k] - __bfloat162float(h0));
    __nv_bfloat16 l1 = __float2bfloat16_rn(v[2 * k + 1] - __bfloat162float(h1));
    h[k] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
    l[k] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
  }
  *(uint4*)(th + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *(uint4*)(tl + off) = make_uint4(l[0], l[1], l[2], l[3]);
}
// 32 consecutive columns [c0, c0+32) of row r of a tile with C columns.
__device__ __forceinline__ void store_split32(uint8_t* th, uint8_t* tl, int r, int c0, int C, const float* v) {
#pragma unroll
  for (int k = 0; k < 4; ++k) store_split8(th, tl, cm_off(r, c0 + 8 * k, C), v + 8 * k);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + 16, v + 16);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  return s;
}

// Reduce-scatter of 32 per-lane values over a warp: afterwards lane l holds the
// warp-wide sum of element l in v[0].
__device__ __forceinline__ float warp_reduce_scatter32(float* v) {
  const int l = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool up = (l & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      float send = up ? v[k] : v[k + s];
      float keep = up ? v[k + s] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// Three-term split product into TMEM column `tmd`:
//   D (+)= Ah*Bh + Ah*Bl + Al*Bh   (M x 64, contraction length K)
// Operand tiles have 64 columns (core-matrix tiles of C = 64).  amn / bmn pick
// the MN-major view (rows = K index) instead of the K-major view (rows = M/N).
// a_off is a byte offset into the A tiles (selects the 128-row half for M = 128).
__device__ __forceinline__ void mma3(uint32_t tmd, const uint8_t* ah, const uint8_t* al, bool amn,
                                     const uint8_t* bh, const uint8_t* bl, bool bmn, int M, int K,
                                     uint32_t a_off, bool accumulate) {
  const uint32_t id = idesc_bf16(M, 64, amn, bmn);
  const uint8_t* ta[3] = {ah, ah, al};
  const uint8_t* tb[3] = {bh, bl, bh};
  for (int t = 0; t < 3; ++t)
    for (int ks = 0; ks < K / 16; ++ks) {
      uint32_t aa = smem_u32(ta[t]) + a_off + (amn ? ks * 2048 : ks * 256);
      uint32_t bb = smem_u32(tb[t]) + (bmn ? ks * 2048 : ks * 256);
      uint64_t da = amn ? desc_mnmajor(aa, 64) : desc_kmajor(aa, 64);
      uint64_t db = bmn ? desc_mnmajor(bb, 64) : desc_kmajor(bb, 64);
      mma_bf16(tmd, da, db, id, (accumulate || t || ks) ? 1u : 0u);
    }
}

// All threads of the CTA: publish freshly written operand tiles to the tensor
// core, let thread 0 issue, wait for the commit.  When an earlier wait expired
// (*bad != 0) the work is skipped but the control flow is kept.
template <typename F>
__device__ __forceinline__ bool mma_sync_run(uint64_t* bar, volatile int* bad, uint32_t& phase, F issue) {
  fence_async_smem();
  fence_before();
  __syncthreads();
  if (*bad) return false;
  if (threadIdx.x == 0) {
    fence_after();
    issue();
    mma_commit(bar);
  }
  bool ok = mbar_wait(bar, phase);
  phase ^= 1;
  fence_after();
  return ok;
}

}  // namespace tc
}  // namespace atlas
