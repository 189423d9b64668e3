// Polar Express of 64 x 256 matrices (the head_dim-64 memory matrices, memory_layer.py:43-71),
// one matrix per in-flight slot with the whole iteration on chip.
//
// The fused scan kernels spend most of each token on exactly this problem, interleaved
// with the momentum and read-out recurrences; here a persistent grid of single CTAs does
// nothing else.  Each CTA keeps two matrices in flight (the fused kernels' slot machinery,
// tc_common.cuh: stacked fp16 hi / lo operand tiles, a producer warp issuing every
// tcgen05.mma, eight epilogue warps handing tiles to it through mbarriers), reads each
// input once from HBM and writes each result once.  The batched GEMMs this replaces move
// every step's operands through HBM (about 64 KB per matrix and product).
//
// Used by atlas_polar_express_batched (ATLAS_PREC_TENSOR) for 64 x 256 / 256 x 64 stacks,
// and so by the batched forward scan at head_dim 64 (scan_gen.cu).  Numerics are the fused
// kernels': every product on split fp16 operands, float32 accumulation in TMEM.
#include <algorithm>

#include "common.cuh"
#include "scan_internal.h"
#include "tc_common.cuh"

namespace atlas {
namespace pecta {
using namespace tc;

struct __align__(1024) Smem {
  uint8_t slot[2][NS_TILE_BYTES];  // per in-flight matrix: stacked X~, stacked A, B' hi / lo
  float red[8];
  uint64_t done[2];   // MMAs of slot s complete
  uint64_t ready[2];  // slot s operand tiles published by the 8 epilogue warps
  uint32_t tmem;
  int bad;
};

// X~ (E x D) element (e, d..d+3) of matrix z in the caller's layout: tall (E x D) is X~
// itself, wide (D x E) its transpose.
__device__ __forceinline__ float4 ld4(const float* M, int e, int d, bool tall) {
  if (tall) return *(const float4*)&M[(size_t)e * D + d];
  return make_float4(M[(size_t)d * E + e], M[(size_t)(d + 1) * E + e], M[(size_t)(d + 2) * E + e],
                     M[(size_t)(d + 3) * E + e]);
}
__device__ __forceinline__ void st4(float* M, int e, int d, bool tall, float4 v) {
  if (tall) {
    *(float4*)&M[(size_t)e * D + d] = v;
  } else {
    M[(size_t)d * E + e] = v.x;
    M[(size_t)(d + 1) * E + e] = v.y;
    M[(size_t)(d + 2) * E + e] = v.z;
    M[(size_t)(d + 3) * E + e] = v.w;
  }
}

// 8 epilogue warps + 1 producer warp.  The CTA takes matrix pairs (2p, 2p + 1),
// p = blockIdx.x, blockIdx.x + gridDim.x, ...; both roles walk the same sequence.
__global__ void __launch_bounds__(NT + 32, 1)
    pe_kernel(const float* X, float* Y, int64_t batch, int tall, int steps, float eps, int* status) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int qd = w & 3, ch = w >> 2;
  const int e0 = 32 * qd + l, e1 = e0 + 128, dc = 32 * ch;
  const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
  if (w == 0) {
    tmem_alloc(&s.tmem, TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.done[0], 1);
    mbar_init(&s.done[1], 1);
    mbar_init(&s.ready[0], 8);
    mbar_init(&s.ready[1], 8);
    fence_mbar_init();
    s.bad = 0;
  }
  fence_before();
  __syncthreads();
  fence_after();
  PESlot sl[2];
  for (int j = 0; j < 2; ++j) {
    uint8_t* b = s.slot[j];
    sl[j].Xh = b;
    sl[j].Xl = b + XLO;
    sl[j].Ah = b + 2 * XT_BYTES;
    sl[j].Al = sl[j].Ah + XLO;
    sl[j].Bh = sl[j].Ah + 2 * AT_BYTES;
    sl[j].Bl = sl[j].Bh + AT_BYTES;
    sl[j].bar = &s.done[j];
    sl[j].tm = s.tmem + 256u * j;
    sl[j].phase = 0;
    sl[j].ns = nullptr;
    sl[j].save_last = 0;
  }
  PEBars B;
  B.ready[0] = &s.ready[0];
  B.ready[1] = &s.ready[1];
  B.done[0] = &s.done[0];
  B.done[1] = &s.done[1];
  B.ready_phase[0] = B.ready_phase[1] = B.done_phase[0] = B.done_phase[1] = 0;
  const int64_t npairs = (batch + 1) / 2;
  const size_t DEs = (size_t)DE;

  if (w == 8) {  // ---- producer warp ----
    for (int64_t p = blockIdx.x; p < npairs; p += gridDim.x) {
      const int n = (int)std::min<int64_t>(2, batch - 2 * p);
      const int64_t pn = p + gridDim.x;  // the next pair's inputs into L2 while this one runs
      if (pn < npairs && l < (int)std::min<int64_t>(2, batch - 2 * pn)) {
        const float* Xn = X + (2 * pn + l) * DEs;
        if (tall) {
          bulk_prefetch_l2(Xn, DE * sizeof(float));
        } else {
          for (int d = 0; d < D; ++d) bulk_prefetch_l2(Xn + (size_t)d * E, E * sizeof(float));
        }
      }
      if (steps > 0 && !pe_produce(sl, B, n, steps, &s.bad) && !s.bad) {
        set_status(status, ATLAS_ERR_DEVICE_TIMEOUT);
        s.bad = 1;
      }
    }
  } else {  // ---- 8 epilogue warps ----
    for (int64_t p = blockIdx.x; p < npairs; p += gridDim.x) {
      const int n = (int)std::min<int64_t>(2, batch - 2 * p);
      for (int j = 0; j < n; ++j) {
        const float* Xz = X + (2 * p + j) * DEs;
        float v[2][32];
        float ss = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 t = ld4(Xz, h ? e1 : e0, dc + 4 * q4, tall);
            v[h][4 * q4] = t.x;
            v[h][4 * q4 + 1] = t.y;
            v[h][4 * q4 + 2] = t.z;
            v[h][4 * q4 + 3] = t.w;
            ss = fmaf(t.x, t.x, fmaf(t.y, t.y, fmaf(t.z, t.z, fmaf(t.w, t.w, ss))));
          }
        ss = block_sum_epi(ss, s.red);
        // X = S / (1.01 sqrt(sum S^2 + eps) + 1e-6)  (memory_layer.py:55-56)
        const float inv = 1.0f / (sqrtf(ss + eps) * 1.01f + 1e-6f);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) v[h][jj] *= inv;
        if (steps == 0) {
          float* Yz = Y + (2 * p + j) * DEs;
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4)
              st4(Yz, h ? e1 : e0, dc + 4 * q4, tall,
                  make_float4(v[h][4 * q4], v[h][4 * q4 + 1], v[h][4 * q4 + 2], v[h][4 * q4 + 3]));
        } else {
          store_stk<32>(sl[j].Xh, e0, dc, v[0]);
          store_stk<32>(sl[j].Xh, e1, dc, v[1]);
        }
      }
      if (steps == 0) continue;
      if (!pe_consume(sl, B, n, steps, &s.bad) && !s.bad) {
        set_status(status, ATLAS_ERR_DEVICE_TIMEOUT);
        s.bad = 1;
      }
      for (int j = 0; j < n; ++j) {
        float* Yz = Y + (2 * p + j) * DEs;
        float x0[32], x1[32];
        tmem_ld32(sl[j].tm + lane_off + TM_X + dc, x0);
        tmem_ld32(sl[j].tm + lane_off + TM_X + 64 + dc, x1);
        tmem_wait_ld();
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {  // TMEM holds KSPLIT^2 X_steps
          st4(Yz, e0, dc + 4 * q4, tall,
              make_float4(x0[4 * q4] * KUNSC2, x0[4 * q4 + 1] * KUNSC2, x0[4 * q4 + 2] * KUNSC2,
                          x0[4 * q4 + 3] * KUNSC2));
          st4(Yz, e1, dc + 4 * q4, tall,
              make_float4(x1[4 * q4] * KUNSC2, x1[4 * q4 + 1] * KUNSC2, x1[4 * q4 + 2] * KUNSC2,
                          x1[4 * q4 + 3] * KUNSC2));
        }
      }
      fence_before();
      epi_sync();  // every TMEM read of this pair precedes the next pair's MMAs
    }
  }
  fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(s.tmem, TMEM_COLS);
}

bool usable(int rows, int cols) { return std::min(rows, cols) == D && std::max(rows, cols) == E; }

static DeviceCache g_blocks;  // resident CTAs per device

cudaError_t launch(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps,
                   cudaStream_t st) {
  if (batch <= 0) return cudaSuccess;
  const size_t smem = sizeof(Smem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(pe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int nb = g_blocks.get([&] {
    int dev = 0, sms = 148, per = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, pe_kernel, NT + 32, smem) != cudaSuccess || per < 1)
      per = 1;
    return sms * per;
  });
  const int64_t npairs = (batch + 1) / 2;
  const int grid = (int)std::min<int64_t>(npairs, nb);
  pe_kernel<<<grid, NT + 32, smem, st>>>(X, Y, batch, (int)(rows > cols), steps, eps, device_status_ptr());
  return cudaGetLastError();
}

}  // namespace pecta
}  // namespace atlas
