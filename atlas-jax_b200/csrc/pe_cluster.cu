// Polar Express of head_dim-128 matrices on a 2-CTA cluster that keeps the matrix on chip
// for all Newton-Schulz steps (memory_layer.py:43-71; optim.py:68-83 for the Muon shapes).
//
// One cluster orthogonalises one D x E matrix at a time (D = 128, E = 256 or 512; tall
// inputs are handled as their transpose, as the reference does).  The matrix is held in
// the "tile" orientation X~ = X^T (E x D): CTA rank r keeps the E/2 rows
// [r E/2, (r+1) E/2) as fp16 hi / lo splits of KX * X~ in shared memory (128 KB at
// E = 512), so S is read from HBM once and the result written once, instead of every
// step's operands making an HBM round trip through the batched GEMMs.
//
// Per step (a, b, c = POLAR_EXPRESS_COEFFS[step]):
//   1. Gram: each CTA forms its partial X~_r^T X~_r (M = N = 128, K = E/2) on tcgen05
//      (hi*hi + hi*lo + lo*hi, float32 TMEM accumulator).
//   2. DSMEM reduction: CTA r owns the 64 columns [64 r, 64 r + 64) of A = X~^T X~.  The
//      warps holding the other half send it to the peer's receive buffer; after a cluster
//      barrier the owning warps add the peer's half, keep their A entries in registers
//      and write the split of A into both CTAs' A tiles.
//   3. A A for the owned 64 columns only (M = 128, N = 64, K = 128).
//   4. B' = a I + b A + c A A for the owned columns, split into both CTAs' B' tiles (the
//      a X term rides in B', as in the fused D = 64 scan).
//   5. X~' = X~ B'^T for the CTA's own rows (M = 128 per half, N = 128, K = 128); the
//      epilogue splits it back into the X~ tiles, or writes the result after the last step.
// Three cluster barriers per step order the DSMEM traffic; one warp issues the MMAs.
//
// Numerics are the batched path's: every product on split fp16 operands (~22 significant
// bits), float32 accumulation, power-of-two operand scales (KX = 512 for X~, whose
// entries are ~E^-1/2 D^-1/2 after the Frobenius normalisation; KB = 256 for A and B').
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "scan_internal.h"
#include "tc_ops.cuh"

namespace atlas {
namespace pecl {
using namespace tcx;

constexpr int D = 128;
constexpr int NT = 256;       // 8 warps: warp w -> TMEM lane quadrant w % 4, column half w / 4
constexpr int MAXR = 256;     // rows of X~ per CTA (E <= 512)
constexpr float KX = 512.f;   // operand scale of X~
constexpr float KB = 256.f;   // operand scale of A and B'
constexpr uint32_t TM_G = 0;     // partial Gram (128 cols)
constexpr uint32_t TM_A2 = 128;  // A A, owned columns (64 cols)
constexpr uint32_t TM_X = 256;   // X~ B'^T, 128 cols per 128-row half

struct __align__(128) Smem {
  uint8_t Xh[MAXR * D * 2], Xl[MAXR * D * 2];  // split of KX X~ (core-matrix tiles, 128 columns)
  uint8_t Ah[D * D * 2], Al[D * D * 2];        // split of KB A, then of KB B'
  float recv[D * 64];                          // the peer's partial Gram, owned columns (swizzled)
  uint64_t bar, bar2;  // MMA completion: every group; the second 128-row half of X~ B'^T
  double red[8];
  double peer_ss;  // the peer's sum of squares
  uint32_t tmem;
  int bad;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// generic-proxy writes into any CTA of the cluster -> visible to the tensor cores
__device__ __forceinline__ void fence_async_cluster() {
  asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
}
__device__ __forceinline__ uint32_t peer_addr(const void* local, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
  return ra;
}
__device__ __forceinline__ void st_peer_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Splits 8 consecutive values (times scale) into fp16 hi / lo 16-byte row segments.
__device__ __forceinline__ void split8(const float* v, float scale, uint4& h, uint4& l) {
  uint32_t hh[4], ll[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float y0 = v[2 * k] * scale, y1 = v[2 * k + 1] * scale;
    const __half2 hv = __floats2half2_rn(y0, y1);
    const float2 hf = __half22float2(hv);
    const __half2 lv = __floats2half2_rn(y0 - hf.x, y1 - hf.y);
    hh[k] = *reinterpret_cast<const uint32_t*>(&hv);
    ll[k] = *reinterpret_cast<const uint32_t*>(&lv);
  }
  h = make_uint4(hh[0], hh[1], hh[2], hh[3]);
  l = make_uint4(ll[0], ll[1], ll[2], ll[3]);
}

// receive buffer: row d of 64 floats as 16 float4 chunks, chunk index XOR (d & 15)
__device__ __forceinline__ int recv_idx(int d, int j4) { return d * 64 + ((j4 ^ (d & 15)) << 2); }

// Three-term split product into TMEM: D (+)= Ah*Bh + Ah*Bl + Al*Bh over K in steps of 16.
// da_h / da_l / db_h / db_l are the operand descriptors, sa / sb their per-16-of-K steps.
__device__ __forceinline__ void mma_split(uint32_t tmd, uint64_t dah, uint64_t dal, uint64_t dbh, uint64_t dbl,
                                          uint64_t sa, uint64_t sb, int ksteps, uint32_t idesc) {
  const uint64_t ta[3] = {dah, dah, dal}, tb[3] = {dbh, dbl, dbh};
#pragma unroll
  for (int t = 0; t < 3; ++t)
    for (int ks = 0; ks < ksteps; ++ks) mma_kf16(tmd, ta[t] + ks * sa, tb[t] + ks * sb, idesc, (t || ks) ? 1u : 0u);
}

// Element (row e of X~, columns d..d+3) of the input / output in the caller's layout:
// tall (E x D) holds X~ itself, wide (D x E) its transpose.
__device__ __forceinline__ float4 ld4(const float* S, int e, int d, bool tall, int E) {
  if (tall) return *(const float4*)&S[(size_t)e * D + d];
  return make_float4(S[(size_t)d * E + e], S[(size_t)(d + 1) * E + e], S[(size_t)(d + 2) * E + e],
                     S[(size_t)(d + 3) * E + e]);
}
__device__ __forceinline__ void st4(float* Y, int e, int d, bool tall, int E, float4 v) {
  if (tall) {
    *(float4*)&Y[(size_t)e * D + d] = v;
  } else {
    Y[(size_t)d * E + e] = v.x;
    Y[(size_t)(d + 1) * E + e] = v.y;
    Y[(size_t)(d + 2) * E + e] = v.z;
    Y[(size_t)(d + 3) * E + e] = v.w;
  }
}

// All threads: wait for the MMAs committed to s.bar (bounded; a timeout marks the
// CTA bad, records ATLAS_ERR_DEVICE_TIMEOUT and skips every later wait and MMA).
__device__ __forceinline__ void wait_mma(Smem& s, uint64_t* bar, uint32_t& phase, int* status) {
  if (!s.bad && !mbar_wait(bar, phase)) {
    s.bad = 1;
    set_status(status, ATLAS_ERR_DEVICE_TIMEOUT);
  }
  phase ^= 1;
  fence_after();
}

__global__ void __launch_bounds__(NT, 1)
    pe_kernel(const float* S, float* Y, int64_t batch, int E, int tall, int steps, float eps, int* status) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, qd = w & 3, ch = w >> 2;
  const uint32_t rank = cluster_rank(), peer = rank ^ 1;
  const int ER = E / 2, MH = ER / 128;
  const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
  const int dA = 32 * qd + l;             // row of the D x D products this thread reads
  const bool own = ch == (int)rank;       // this thread's 64 columns of A are owned by this CTA
  const int64_t ncl = gridDim.x >> 1;
  const size_t DE = (size_t)D * E;
  if (w == 0) {
    tmem_alloc(&s.tmem, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.bar, 1);
    mbar_init(&s.bar2, 1);
    fence_mbar_init();
    s.bad = 0;
  }
  fence_before();
  __syncthreads();
  fence_after();
  cluster_sync();  // both CTAs initialised before any DSMEM traffic
  const uint32_t tm = s.tmem;
  uint32_t phase = 0, phase2 = 0;
  const uint32_t r_recv = peer_addr(s.recv, peer), r_Ah = peer_addr(s.Ah, peer), r_Al = peer_addr(s.Al, peer);
  const uint32_t r_ss = peer_addr(&s.peer_ss, peer);

  for (int64_t z = blockIdx.x >> 1; z < batch; z += ncl) {
    const float* Sz = S + z * DE;
    float* Yz = Y + z * DE;
    if (w == 7 && z + ncl < batch) {  // the next matrix's rows of this CTA into L2
      const float* Sn = S + (z + ncl) * DE;
      if (tall) {
        const uint32_t part = (uint32_t)ER * D * 4 / 32;
        bulk_prefetch_l2((const uint8_t*)(Sn + (size_t)rank * ER * D) + l * part, part);
      } else {
        for (int d = l; d < D; d += 32) bulk_prefetch_l2(Sn + (size_t)d * E + (size_t)rank * ER, ER * 4);
      }
    }
    // ---- Frobenius normalisation: X = S / (1.01 sqrt(sum S^2 + eps) + 1e-6) ----
    float ssf = 0.f;
    for (int h = 0; h < MH; ++h) {
      const int e = (int)rank * ER + 128 * h + dA;
#pragma unroll 4
      for (int j = 0; j < 64; j += 4) {
        const float4 v = ld4(Sz, e, 64 * ch + j, tall, E);
        ssf = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ssf))));
      }
    }
    double ss = ssf;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (l == 0) s.red[w] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) tot += s.red[i];
    if (tid == 0) asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(r_ss), "d"(tot) : "memory");
    cluster_sync();
    const double all = tot + s.peer_ss;  // the same sum on both CTAs (addition commutes)
    const float inv = (float)(1.0 / (sqrt(all + (double)eps) * 1.01 + 1e-6));
    for (int h = 0; h < MH; ++h) {
      const int r = 128 * h + dA, e = (int)rank * ER + r;
#pragma unroll 2
      for (int j = 0; j < 64; j += 8) {
        const float4 v0 = ld4(Sz, e, 64 * ch + j, tall, E), v1 = ld4(Sz, e, 64 * ch + j + 4, tall, E);
        float x[8] = {v0.x * inv, v0.y * inv, v0.z * inv, v0.w * inv, v1.x * inv, v1.y * inv, v1.z * inv, v1.w * inv};
        if (steps == 0) {
          st4(Yz, e, 64 * ch + j, tall, E, make_float4(x[0], x[1], x[2], x[3]));
          st4(Yz, e, 64 * ch + j + 4, tall, E, make_float4(x[4], x[5], x[6], x[7]));
        } else {
          uint4 hv, lv;
          split8(x, KX, hv, lv);
          const uint32_t off = cm_off(r, 64 * ch + j, D);
          *(uint4*)(s.Xh + off) = hv;
          *(uint4*)(s.Xl + off) = lv;
        }
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();

    for (int st = 0; st < steps; ++st) {
      const float ca = (float)kPE[st][0], cb = (float)kPE[st][1], cc = (float)kPE[st][2];
      // ---- 1. partial Gram X~_r^T X~_r (both operands MN-major views of the X~ tiles) ----
      if (w == 0 && !s.bad) {
        fence_after();
        const uint64_t xh = desc_mnmajor(smem_u32(s.Xh), D), xl = desc_mnmajor(smem_u32(s.Xl), D);
        mma_split(tm + TM_G, xh, xl, xh, xl, 256, 256, ER / 16, idesc_f16(128, 128, true, true));
        mma_commit(&s.bar);
      }
      wait_mma(s, &s.bar, phase, status);
      // ---- 2. reduce over the cluster; this CTA owns columns [64 rank, 64 rank + 64) ----
      float g[64];
      tmem_ld16(tm + lane_off + TM_G + 64 * ch, g);
      tmem_ld16(tm + lane_off + TM_G + 64 * ch + 16, g + 16);
      tmem_ld16(tm + lane_off + TM_G + 64 * ch + 32, g + 32);
      tmem_ld16(tm + lane_off + TM_G + 64 * ch + 48, g + 48);
      tmem_wait_ld();
      if (!own) {
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4)
          st_peer_v4(r_recv + 4u * recv_idx(dA, j4),
                     make_uint4(__float_as_uint(g[4 * j4]), __float_as_uint(g[4 * j4 + 1]),
                                __float_as_uint(g[4 * j4 + 2]), __float_as_uint(g[4 * j4 + 3])));
      }
      cluster_sync();
      float Av[64];  // A[dA][64 rank + j] (owning threads)
      if (own) {
        constexpr float un = 1.f / (KX * KX);
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4) {
          const float4 rv = *(const float4*)&s.recv[recv_idx(dA, j4)];
          Av[4 * j4] = (g[4 * j4] + rv.x) * un;
          Av[4 * j4 + 1] = (g[4 * j4 + 1] + rv.y) * un;
          Av[4 * j4 + 2] = (g[4 * j4 + 2] + rv.z) * un;
          Av[4 * j4 + 3] = (g[4 * j4 + 3] + rv.w) * un;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          uint4 hv, lv;
          split8(Av + 8 * k, KB, hv, lv);
          const uint32_t off = cm_off(dA, 64 * (int)rank + 8 * k, D);
          *(uint4*)(s.Ah + off) = hv;
          *(uint4*)(s.Al + off) = lv;
          st_peer_v4(r_Ah + off, hv);
          st_peer_v4(r_Al + off, lv);
        }
      }
      fence_async_cluster();
      fence_before();
      cluster_sync();
      // ---- 3. A A for the owned columns (A symmetric: its rows are the K-major B operand) ----
      if (w == 0 && !s.bad) {
        fence_after();
        const uint32_t ah = smem_u32(s.Ah), al = smem_u32(s.Al), boff = 16384u * rank;
        mma_split(tm + TM_A2, desc_kmajor(ah, D), desc_kmajor(al, D), desc_kmajor(ah + boff, D),
                  desc_kmajor(al + boff, D), 16, 16, D / 16, idesc_f16(128, 64, false, false));
        mma_commit(&s.bar);
      }
      wait_mma(s, &s.bar, phase, status);
      cluster_sync();  // both CTAs' A A products have read the A tiles
      // ---- 4. B' = a I + b A + c A A for the owned columns, into both CTAs' tiles ----
      if (own) {
        tmem_ld16(tm + lane_off + TM_A2, g);
        tmem_ld16(tm + lane_off + TM_A2 + 16, g + 16);
        tmem_ld16(tm + lane_off + TM_A2 + 32, g + 32);
        tmem_ld16(tm + lane_off + TM_A2 + 48, g + 48);
        tmem_wait_ld();
        constexpr float un = 1.f / (KB * KB);
#pragma unroll
        for (int j = 0; j < 64; ++j)
          g[j] = fmaf(cc * un, g[j], cb * Av[j]) + (dA == 64 * (int)rank + j ? ca : 0.f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          uint4 hv, lv;
          split8(g + 8 * k, KB, hv, lv);
          const uint32_t off = cm_off(dA, 64 * (int)rank + 8 * k, D);
          *(uint4*)(s.Ah + off) = hv;
          *(uint4*)(s.Al + off) = lv;
          st_peer_v4(r_Ah + off, hv);
          st_peer_v4(r_Al + off, lv);
        }
      }
      fence_async_cluster();
      fence_before();
      cluster_sync();
      // ---- 5. X~' = X~ B'^T for this CTA's rows ----
      if (w == 0 && !s.bad) {
        fence_after();
        const uint32_t bh = smem_u32(s.Ah), bl = smem_u32(s.Al);
        for (int h = 0; h < MH; ++h) {  // one commit per half: half 0's epilogue overlaps half 1's MMAs
          const uint32_t xo = 32768u * h;
          mma_split(tm + TM_X + 128 * h, desc_kmajor(smem_u32(s.Xh) + xo, D), desc_kmajor(smem_u32(s.Xl) + xo, D),
                    desc_kmajor(bh, D), desc_kmajor(bl, D), 16, 16, D / 16, idesc_f16(128, 128, false, false));
          mma_commit(h ? &s.bar2 : &s.bar);
        }
      }
      const bool last = st + 1 == steps;
      for (int h = 0; h < MH; ++h) {
        if (h)
          wait_mma(s, &s.bar2, phase2, status);
        else
          wait_mma(s, &s.bar, phase, status);
        const int r = 128 * h + dA, e = (int)rank * ER + r;
        const uint32_t ta = tm + lane_off + TM_X + 128 * h + 64 * ch;
        tmem_ld16(ta, g);
        tmem_ld16(ta + 16, g + 16);
        tmem_ld16(ta + 32, g + 32);
        tmem_ld16(ta + 48, g + 48);
        tmem_wait_ld();
        if (last) {  // TMEM holds KX KB X~'
          constexpr float un = 1.f / (KX * KB);
#pragma unroll
          for (int j = 0; j < 64; j += 4)
            st4(Yz, e, 64 * ch + j, tall, E, make_float4(g[j] * un, g[j + 1] * un, g[j + 2] * un, g[j + 3] * un));
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            uint4 hv, lv;
            split8(g + 8 * k, 1.f / KB, hv, lv);
            const uint32_t off = cm_off(r, 64 * ch + 8 * k, D);
            *(uint4*)(s.Xh + off) = hv;
            *(uint4*)(s.Xl + off) = lv;
          }
        }
      }
      fence_async_smem();
      fence_before();
      __syncthreads();
    }
    cluster_sync();  // the peer is done with this matrix's DSMEM slots
  }
  fence_before();
  __syncthreads();
  cluster_sync();
  if (w == 0) tmem_dealloc(s.tmem, 512);
}

bool usable(int rows, int cols) {
  const int d = std::min(rows, cols), e = std::max(rows, cols);
  return d == D && (e == 256 || e == 512);
}

static DeviceCache g_max_clusters;

cudaError_t launch(const float* S, float* Y, int64_t batch, int rows, int cols, int steps, float eps,
                   cudaStream_t st) {
  if (batch <= 0) return cudaSuccess;
  const int E = std::max(rows, cols);
  const size_t smem = sizeof(Smem) + 128;
  cudaError_t e = cudaFuncSetAttribute(pe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int maxc = g_max_clusters.get([&] {
    int n = 0;
    cfg.gridDim = dim3(2);
    if (cudaOccupancyMaxActiveClusters(&n, pe_kernel, &cfg) != cudaSuccess || n <= 0) n = 1;
    return n;
  });
  cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(batch, maxc)));
  return cudaLaunchKernelEx(&cfg, pe_kernel, S, Y, batch, E, (int)(rows > cols), steps, eps, device_status_ptr());
}

}  // namespace pecl
}  // namespace atlas
