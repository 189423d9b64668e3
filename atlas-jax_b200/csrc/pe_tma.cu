// TMA-fed tcgen05 GEMM for the batched Polar Express of large matrices (the Muon
// stacks of atlas_jax/optim.py:56-108, iteration of memory_layer.py:43-71).
//
// Every operand is pre-split once, by the epilogue that produces it, into fp16 hi / lo
// parts of a power-of-two multiple of its value, stored K-major as [batch][part][rows][K].
// The main loop then moves no float32 data and does no conversion work: a TMA warp
// loads both parts of a 128 x 64 A tile and a BN x 64 B tile per stage (one
// cp.async.bulk.tensor each, 128-byte swizzle, no multicast), an MMA warp issues the
// three split terms hi*hi + hi*lo + lo*hi as M=128 x N=BN x K=16 tcgen05 MMAs into a
// float32 TMEM accumulator, and eight epilogue warps (two per TMEM lane quadrant, one
// column half each) turn the accumulator into alpha * acc + beta * addend, written as
// float32 and / or as the next product's split operand (row-major or transposed).  The
// kernel is persistent (one CTA per SM walking the output tiles) with two TMEM
// accumulators, so one tile's epilogue overlaps the next tile's MMAs.  Every wait is
// bounded and records ATLAS_ERR_DEVICE_TIMEOUT instead of hanging.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "pe_tma.h"
#include "tc_ops.cuh"

namespace atlas {
namespace pet2 {
using namespace tcx;

constexpr int BM = 128, TK = 64, NTH = 320;  // warps 0-7 epilogue, 8 TMA, 9 MMA
constexpr int NEPI = 8;

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 2 : 3;
  static constexpr int A_BYTES = 2 * BM * TK * 2;  // hi + lo, 128 B per row
  static constexpr int B_BYTES = 2 * BN * TK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(2 * BN <= 512, "two accumulators must fit TMEM");
};

// SM100 shared-memory descriptor of a K-major operand in the 128-byte swizzled
// layout TMA writes: rows of 128 bytes (64 fp16 of K), 8-row atoms of 1024 bytes.
// Stepping K by 16 inside the atom adds 32 bytes to the start address.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;              // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;              // version
  d |= (uint64_t)2 << 61;              // layout: SWIZZLE_128B
  return d;
}

// MN-major operand as TMA writes it for a (64 n x TK k x 2 parts) box per 64-column chunk:
// each k row is 128 bytes of n, 8-row atoms of 1024 bytes; chunk j of a part at
// j * 2 * TK * 128 bytes (leading byte offset), next 8 k rows at 1024 (stride byte offset).
__device__ __forceinline__ uint64_t desc_sw128_mn(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((2 * TK * 128) >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_load3(void* sdst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(sdst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Writes fp16 hi / lo parts of so * v for 8 consecutive values into a split array.
__device__ __forceinline__ void split8_g(__half* hi, __half* lo, const float* v, float so) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float y0 = v[2 * k] * so, y1 = v[2 * k + 1] * so;
    const __half2 hv = __floats2half2_rn(y0, y1);
    const float2 hf = __half22float2(hv);
    const __half2 lv = __floats2half2_rn(y0 - hf.x, y1 - hf.y);
    h[k] = *reinterpret_cast<const uint32_t*>(&hv);
    l[k] = *reinterpret_cast<const uint32_t*>(&lv);
  }
  *(uint4*)hi = make_uint4(h[0], h[1], h[2], h[3]);
  *(uint4*)lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void split_pair(float y, __half* hi, __half* lo) {
  const __half h = __float2half_rn(y);
  *hi = h;
  *lo = __float2half_rn(y - __half2float(h));
}

// Epilogue of the packed mode for the TMEM row of packed row R (batch entry R / D,
// row R % D).  Diagonal products (g.diag): only the row's own D x D block (columns
// D (R % 128 / D) ..) is kept: alpha acc + beta Dm as float32 [z][D][D] (Cf), as a packed
// split [part][batch D][D] (Cs), and / or as a packed split of row length 128 with
// the block at columns D (z % P) and zeros elsewhere (Cpad: the block-diagonal A operand
// of the row product).  Row product: alpha acc + beta (split addend Ds) over N = E
// columns, written as the packed split (Cs), or as float32 rows (Cf, wide) / columns
// (CfT, tall) of the caller's matrices.
template <int BN>
__device__ __forceinline__ void packed_epilogue(const EpiArgs& g, uint32_t tacc, int R, int n0, int half,
                                                int batch) {
  const int D = g.M, P = g.pack;
  const int z = R / D, r = R % D;
  const bool live = z < batch;
  const size_t rows = (size_t)batch * D;
  if (g.diag) {
    const int blk = (R % BM) / D;  // this row's diagonal block within the tile
    // column chunks of 32 that hold the block (D >= 32: uniform across the warp)
#pragma unroll 1
    for (int cb = 0; cb < BN / 32; ++cb) {
      if (cb / 2 != half) continue;  // column half of this warp
      const int c0 = 32 * cb;
      if (c0 < blk * D || c0 >= blk * D + D) continue;  // warp-uniform (32 rows share blk)
      float v[32];
      tmem_ld16(tacc + c0, v);
      tmem_ld16(tacc + c0 + 16, v + 16);
      tmem_wait_ld();
      if (!live) continue;
      const int cc = c0 - blk * D;  // column within the D x D block
      const size_t o = (size_t)z * D * D + (size_t)r * D + cc;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        v[j] = fmaf(g.alpha, v[j], g.Dm ? g.beta * g.Dm[o + j] : 0.f) + (r == cc + j ? g.diag_add : 0.f);
      if (g.Cf) {
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          *(float4*)(g.Cf + o + 4 * j4) = make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
      }
      if (g.Cs) {
        __half* hp = g.Cs + (size_t)R * D + cc;
#pragma unroll
        for (int k8 = 0; k8 < 4; ++k8) split8_g(hp + 8 * k8, hp + rows * D + 8 * k8, v + 8 * k8, g.so);
      }
      if (g.Cpad) {
        __half* hp = g.Cpad + (size_t)R * BM;
        const size_t lo = rows * BM;
#pragma unroll
        for (int k8 = 0; k8 < 4; ++k8) split8_g(hp + (z % P) * D + cc + 8 * k8, hp + lo + (z % P) * D + cc + 8 * k8,
                                               v + 8 * k8, g.so);
        if (cc == 0) {  // zeros outside the block (this thread's row)
          const uint4 zero = make_uint4(0, 0, 0, 0);
          for (int c = 0; c < BM; c += 8)
            if (c < (z % P) * D || c >= (z % P) * D + D) {
              *(uint4*)(hp + c) = zero;
              *(uint4*)(hp + lo + c) = zero;
            }
        }
      }
    }
    return;
  }
  const int E = g.N;
#pragma unroll 1
  for (int cb = half * (BN / 64); cb < (half + 1) * (BN / 64); ++cb) {
    const int nb = n0 + 32 * cb;
    if (nb >= E) break;  // warp-uniform
    float v[32];
    tmem_ld16(tacc + 32 * cb, v);
    tmem_ld16(tacc + 32 * cb + 16, v + 16);
    tmem_wait_ld();
    if (!live) continue;
    const bool full32 = nb + 32 <= E;
    const size_t o = (size_t)R * E + nb;
    if (g.Ds) {
      const float bs = g.beta * g.dscale_inv;
      if (full32 && (E & 7) == 0) {
#pragma unroll
        for (int k8 = 0; k8 < 4; ++k8) {
          const uint4 h4 = *(const uint4*)(g.Ds + o + 8 * k8), l4 = *(const uint4*)(g.Ds + rows * E + o + 8 * k8);
          const uint32_t hw[4] = {h4.x, h4.y, h4.z, h4.w}, lw[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hw[q]));
            const float2 lf = __half22float2(*reinterpret_cast<const __half2*>(&lw[q]));
            v[8 * k8 + 2 * q] = fmaf(g.alpha, v[8 * k8 + 2 * q], bs * (hf.x + lf.x));
            v[8 * k8 + 2 * q + 1] = fmaf(g.alpha, v[8 * k8 + 2 * q + 1], bs * (hf.y + lf.y));
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = fmaf(g.alpha, v[j],
                      nb + j < E ? bs * (__half2float(g.Ds[o + j]) + __half2float(g.Ds[rows * E + o + j])) : 0.f);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= g.alpha;
    }
    if (g.Cs) {
      __half* hp = g.Cs + o;
      if (full32 && (E & 7) == 0) {
#pragma unroll
        for (int k8 = 0; k8 < 4; ++k8) split8_g(hp + 8 * k8, hp + rows * E + 8 * k8, v + 8 * k8, g.so);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (nb + j < E) split_pair(v[j] * g.so, hp + j, hp + rows * E + j);
      }
    }
    if (g.Cf) {
      if (full32 && (E & 3) == 0) {
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          *(float4*)(g.Cf + o + 4 * j4) = make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (nb + j < E) g.Cf[o + j] = v[j];
      }
    }
    if (g.CfT) {  // tall caller matrices: Y[z] is E x D
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (nb + j < E) g.CfT[(size_t)z * D * E + (size_t)(nb + j) * D + r] = v[j];
    }
  }
}

// Persistent: each CTA walks output tiles (batch entry, n tile, m tile) with stride
// gridDim.x.  Two TMEM accumulators (2 * BN columns) let the epilogue of one tile run
// while the MMAs of the next accumulate.
template <int BN, bool BMN>
__global__ void __launch_bounds__(NTH, 1) gemm_kernel(const __grid_constant__ CUtensorMap mapA,
                                                        const __grid_constant__ CUtensorMap mapB, const EpiArgs g,
                                                        int z0, int nz) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* bad = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int t = threadIdx.x, w = t >> 5, lane = t & 31;
  const int nk = (g.K + TK - 1) / TK;
  // Packed mode (g.pack = P matrices of D = 128 / P rows per 128-row tile): tile t of
  // the diagonal products covers matrices [tP, tP + P) on both operands; tile (t, n) of
  // the row product reads A rows [128 t, 128 t + 128) and B's K rows from the same offset.
  const int tiles_m = g.pack ? (nz + g.pack - 1) / g.pack : (g.M + BM - 1) / BM;
  const int tiles_n = g.pack && g.diag ? 1 : (g.N + BN - 1) / BN;
  const int ntiles = g.pack ? tiles_m * tiles_n : tiles_m * tiles_n * nz;
  // m0: A row coordinate; n0: B row (K-major) or column (MN-major) coordinate; kb: B's
  // K coordinate base (MN-major); c2: third coordinate of both maps; z: batch entry
  auto tile_coords = [&](int tile, int& m0, int& n0, int& z, int& kb, int& c2) {
    if (g.pack) {
      const int tm_ = tile % tiles_m;
      m0 = BM * tm_;
      n0 = g.diag ? m0 : (tile / tiles_m) * BN;
      kb = g.diag ? 0 : m0;
      c2 = 0;
      z = tm_ * g.pack;
      return;
    }
    m0 = (tile % tiles_m) * BM;
    const int r = tile / tiles_m;
    n0 = (r % tiles_n) * BN;
    z = z0 + r / tiles_n;
    kb = 0;
    c2 = 2 * z;
  };

  if (w == 0) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  if (t == 32) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], NEPI);  // one arrival per epilogue warp
    }
    *bad = 0;
    fence_mbar_init();
  }
  if (t == 64) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapB) : "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = *tmem_slot;

  if (w == NEPI) {  // TMA producer
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*bad; tile += gridDim.x) {
        int m0, n0, z, kb, c2;
        tile_coords(tile, m0, n0, z, kb, c2);
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % C::STAGES;
          if (it >= C::STAGES && !mbar_wait(&empty[s], ((it / C::STAGES) - 1) & 1)) {
            set_status(g.status, ATLAS_ERR_DEVICE_TIMEOUT);
            *bad = 1;
            break;
          }
          uint8_t* sa = base + s * C::STAGE_BYTES;
          mbar_expect_tx(&full[s], (uint32_t)C::STAGE_BYTES);
          tma_load3(sa, &mapA, i * TK, m0, c2, &full[s]);
          if (BMN) {  // 64-column chunks [j][part][k][64 n]
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load3(sa + C::A_BYTES + j * (2 * TK * 128), &mapB, n0 + 64 * j, kb + i * TK, c2, &full[s]);
          } else {
            tma_load3(sa + C::A_BYTES, &mapB, i * TK, n0, c2, &full[s]);
          }
        }
      }
    }
  } else if (w == NEPI + 1) {  // MMA issuer (whole warp; one elected lane issues)
    const uint32_t idesc = idesc_f16(BM, BN, false, BMN);
    int it = 0, lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++lt) {
      const int a = lt & 1;
      if (lt >= 2 && !mbar_wait(&acc_empty[a], ((lt >> 1) - 1) & 1)) ok = false;
      fence_after();
      const uint32_t acc = tm + (uint32_t)(a * BN);
      for (int i = 0; i < nk && ok; ++i, ++it) {
        const int s = it % C::STAGES;
        if (!mbar_wait(&full[s], (it / C::STAGES) & 1)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t sa = smem_u32(base + s * C::STAGE_BYTES);
        const uint32_t sb = sa + C::A_BYTES;
        const uint64_t da[2] = {desc_sw128(sa), desc_sw128(sa + BM * 128)};
        const uint64_t db[2] = {BMN ? desc_sw128_mn(sb) : desc_sw128(sb),
                                BMN ? desc_sw128_mn(sb + TK * 128) : desc_sw128(sb + BN * 128)};
        constexpr uint64_t bstep = BMN ? (16 * 128) >> 4 : 2;  // K = 16: 16 rows (MN-major) or 32 bytes
        const int ta[3] = {0, 0, 1}, tb[3] = {0, 1, 0};  // hi*hi, hi*lo, lo*hi
#pragma unroll
        for (int term = 0; term < 3; ++term)
#pragma unroll
          for (int ks = 0; ks < TK / 16; ++ks)
            mma_kf16(acc, da[ta[term]] + 2 * ks, db[tb[term]] + bstep * ks, idesc, (i || term || ks) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(&acc_full[a]);
    }
    if (!ok && lane == 0) {
      set_status(g.status, ATLAS_ERR_DEVICE_TIMEOUT);
      *bad = 1;
    }
  } else {  // epilogue warps 0-7: TMEM lane quadrant w % 4 = rows m0 + 32 (w % 4) .. +31, column half w / 4
    const size_t MN = (size_t)g.M * g.N;
    int lt = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++lt) {
      int m0, n0, z, kb, c2;
      tile_coords(tile, m0, n0, z, kb, c2);
      const int a = lt & 1;
      const bool ok = mbar_wait(&acc_full[a], (lt >> 1) & 1) && !*bad;
      fence_after();
      if (!ok) {
        if (lane == 0) {
          set_status(g.status, ATLAS_ERR_DEVICE_TIMEOUT);
          *bad = 1;
        }
        break;
      }
      const int qd = w & 3, half = w >> 2;
      if (g.pack) {
        packed_epilogue<BN>(g, tm + (uint32_t)(a * BN) + ((uint32_t)(32 * qd) << 16), m0 + 32 * qd + lane, n0,
                            half, nz);
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[a]);
        continue;
      }
      const int m = m0 + 32 * qd + lane;
      const bool mrow = m < g.M;
      const size_t zz = (size_t)z;
      const float* Dm = g.Dm ? g.Dm + zz * g.sD : nullptr;
      float* Cf = g.Cf ? g.Cf + zz * g.sC : nullptr;
      float* CfT = g.CfT ? g.CfT + zz * MN : nullptr;
      __half* sh = g.Cs ? g.Cs + zz * 2 * MN : nullptr;
      __half* th = g.Ct ? g.Ct + zz * 2 * MN : nullptr;
      const uint32_t tacc = tm + (uint32_t)(a * BN) + ((uint32_t)(32 * qd) << 16);
#pragma unroll 1
      for (int cb = half * (BN / 64); cb < (half + 1) * (BN / 64); ++cb) {
        const int nb = n0 + 32 * cb;
        if (nb >= g.N) break;  // warp-uniform
        float v[32];
        tmem_ld16(tacc + 32 * cb, v);
        tmem_ld16(tacc + 32 * cb + 16, v + 16);
        tmem_wait_ld();
        if (!mrow) continue;
        const bool full32 = nb + 32 <= g.N;
        if (Dm) {
          const float* dp = Dm + (size_t)m * g.ldd + nb;
          if (full32 && (g.ldd & 3) == 0) {
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 d = *(const float4*)(dp + 4 * j4);
              v[4 * j4 + 0] = fmaf(g.alpha, v[4 * j4 + 0], g.beta * d.x);
              v[4 * j4 + 1] = fmaf(g.alpha, v[4 * j4 + 1], g.beta * d.y);
              v[4 * j4 + 2] = fmaf(g.alpha, v[4 * j4 + 2], g.beta * d.z);
              v[4 * j4 + 3] = fmaf(g.alpha, v[4 * j4 + 3], g.beta * d.w);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaf(g.alpha, v[j], nb + j < g.N ? g.beta * dp[j] : 0.f);
          }
        } else if (g.Ds) {
          const __half* dh = g.Ds + zz * 2 * MN + (size_t)m * g.N + nb;
          if (full32 && (g.N & 7) == 0) {
#pragma unroll
            for (int k8 = 0; k8 < 4; ++k8) {
              const uint4 h4 = *(const uint4*)(dh + 8 * k8), l4 = *(const uint4*)(dh + MN + 8 * k8);
              const uint32_t hw[4] = {h4.x, h4.y, h4.z, h4.w}, lw[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hw[q]));
                const float2 lf = __half22float2(*reinterpret_cast<const __half2*>(&lw[q]));
                const float bs = g.beta * g.dscale_inv;
                v[8 * k8 + 2 * q] = fmaf(g.alpha, v[8 * k8 + 2 * q], bs * (hf.x + lf.x));
                v[8 * k8 + 2 * q + 1] = fmaf(g.alpha, v[8 * k8 + 2 * q + 1], bs * (hf.y + lf.y));
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              v[j] = fmaf(g.alpha, v[j],
                          nb + j < g.N ? g.beta * g.dscale_inv * (__half2float(dh[j]) + __half2float(dh[MN + j])) : 0.f);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= g.alpha;
        }
        if (Cf) {
          float* cp = Cf + (size_t)m * g.ldc + nb;
          if (full32 && (g.ldc & 3) == 0) {
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4)
              *(float4*)(cp + 4 * j4) = make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < g.N) cp[j] = v[j];
          }
        }
        if (CfT) {  // [N][M], column m: lanes write consecutive m
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < g.N) CfT[(size_t)(nb + j) * g.M + m] = v[j];
        }
        if (sh) {  // [part][M][N], row m
          __half* hp = sh + (size_t)m * g.N + nb;
          if (full32 && (g.N & 7) == 0) {
#pragma unroll
            for (int k8 = 0; k8 < 4; ++k8) split8_g(hp + 8 * k8, hp + MN + 8 * k8, v + 8 * k8, g.so);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < g.N) {
                const float y = v[j] * g.so;
                const __half h = __float2half_rn(y);
                hp[j] = h;
                hp[MN + j] = __float2half_rn(y - __half2float(h));
              }
          }
        }
        if (th) {  // [part][N][M], column m
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < g.N) {
              const float y = v[j] * g.so;
              const __half h = __float2half_rn(y);
              const size_t o = (size_t)(nb + j) * g.M + m;
              th[o] = h;
              th[MN + o] = __float2half_rn(y - __half2float(h));
            }
        }
      }
      // accumulator a is free for the tile after next
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }
  fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tm, 2 * BN);
}

constexpr int NPART = 64;  // partial sums of squares per matrix

__global__ void __launch_bounds__(256) sumsq_kernel(const float* S, double* part, size_t n, int vec) {
  __shared__ double red[8];
  const float* s = S + (size_t)blockIdx.y * n;
  double acc = 0;
  if (vec) {
    for (size_t i = ((size_t)blockIdx.x * 256 + threadIdx.x) * 4; i < n; i += (size_t)gridDim.x * 1024) {
      const float4 x = *(const float4*)(s + i);
      acc += (double)x.x * x.x + (double)x.y * x.y + (double)x.z * x.z + (double)x.w * x.w;
    }
  } else {
    for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (size_t)gridDim.x * 256)
      acc += (double)s[i] * s[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    part[(size_t)blockIdx.y * NPART + blockIdx.x] = tot;
  }
}

__device__ __forceinline__ void split1(__half* o, size_t lo_off, float y) {
  const __half h = __float2half_rn(y);
  o[0] = h;
  o[lo_off] = __float2half_rn(y - __half2float(h));
}

// One 32 x 32 tile (wide rows d, columns e) per block, through shared memory so every
// read and write is coalesced.
__global__ void __launch_bounds__(256) norm_split_kernel(const float* S, float* Xf, __half* Xs, __half* Xt,
                                                         const double* part, int D, int E, int tall, float eps,
                                                         float sx, int64_t packed_z0, int64_t packed_batch) {
  __shared__ float tile[32][33];
  __shared__ float s_inv;
  const size_t DE = (size_t)D * E;
  const size_t z = blockIdx.z;
  const float* s = S + z * DE;
  if (threadIdx.x == 0) {
    double tot = 0;
    for (int i = 0; i < NPART; ++i) tot += part[z * NPART + i];
    s_inv = (float)(1.0 / (sqrt(tot + (double)eps) * 1.01 + 1e-6));
  }
  const int e0 = blockIdx.x * 32, d0 = blockIdx.y * 32, tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (tall) {  // S is E x D
      const int e = e0 + ty + 8 * k, d = d0 + tx;
      tile[tx][ty + 8 * k] = (e < E && d < D) ? s[(size_t)e * D + d] : 0.f;
    } else {  // S is D x E
      const int d = d0 + ty + 8 * k, e = e0 + tx;
      tile[ty + 8 * k][tx] = (e < E && d < D) ? s[(size_t)d * E + e] : 0.f;
    }
  }
  __syncthreads();
  const float inv = s_inv;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = d0 + ty + 8 * k, e = e0 + tx;
    if (d < D && e < E) {
      const float x = tile[ty + 8 * k][tx] * inv;
      if (Xf) Xf[z * DE + (size_t)d * E + e] = x;
      if (packed_batch)  // [part][batch * D][E]
        split1(Xs + (packed_z0 + z) * DE + (size_t)d * E + e, (size_t)packed_batch * DE, x * sx);
      else
        split1(Xs + z * 2 * DE + (size_t)d * E + e, DE, x * sx);
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = e0 + ty + 8 * k, d = d0 + tx;
    if (Xt && d < D && e < E) split1(Xt + z * 2 * DE + (size_t)e * D + d, DE, tile[tx][ty + 8 * k] * inv * sx);
  }
}

cudaError_t normalize_split(const float* S, float* Xf, __half* Xs, __half* Xt, double* part, int64_t batch, int rows,
                            int cols, float eps, float sx, cudaStream_t st, bool packed) {
  const int D = rows < cols ? rows : cols, E = rows < cols ? cols : rows;
  const size_t DE = (size_t)D * E;
  const int vec = (reinterpret_cast<uintptr_t>(S) & 15) == 0 && DE % 4 == 0;
  for (int64_t z0 = 0; z0 < batch; z0 += 65535) {
    const int nz = (int)std::min<int64_t>(65535, batch - z0);
    sumsq_kernel<<<dim3(NPART, nz), 256, 0, st>>>(S + z0 * DE, part + z0 * NPART, DE, vec);
    norm_split_kernel<<<dim3((E + 31) / 32, (D + 31) / 32, nz), 256, 0, st>>>(
        S + z0 * DE, Xf ? Xf + z0 * DE : nullptr, packed ? Xs : Xs + z0 * 2 * DE, Xt ? Xt + z0 * 2 * DE : nullptr,
        part + z0 * NPART, D, E, rows > cols, eps, sx, z0, packed ? batch : 0);
  }
  return cudaGetLastError();
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map of a split operand [batch][part][rows][K] (fp16): box of 64 K x box_rows
// rows x both parts, 128-byte swizzle, out-of-range elements read as zero.
static bool make_map(CUtensorMap* map, const __half* base, int64_t batch, int rows, int K, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)(2 * batch)};
  const cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)rows * K * 2};
  const cuuint32_t box[3] = {(cuuint32_t)TK, (cuuint32_t)box_rows, 2};
  const cuuint32_t es[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of a split operand stored [batch][part][K][cols] (MN-major use): box of
// 64 columns x TK K rows x both parts.
static bool make_map_mn(CUtensorMap* map, const __half* base, int64_t batch, int cols, int K) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)K, (cuuint64_t)(2 * batch)};
  const cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)cols * K * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)TK, 2};
  const cuuint32_t es[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool BMN>
static cudaError_t gemm_bn(const __half* As, const __half* Bs, const EpiArgs& g, int64_t batch, cudaStream_t s) {
  CUtensorMap ma, mb;
  const size_t smem = Cfg<BN>::SMEM;
  cudaError_t e =
      cudaFuncSetAttribute(gemm_kernel<BN, BMN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (g.pack) {  // packed arrays: [part][batch * rows][K]
    if (batch * g.M >= ((int64_t)1 << 31)) return cudaErrorInvalidValue;
    const int rows = (int)(batch * g.M);
    if (!make_map(&ma, As, 1, rows, g.K, BM) ||
        !(g.diag ? make_map(&mb, Bs, 1, rows, g.K, BN) : make_map_mn(&mb, Bs, 1, g.N, rows)))
      return cudaErrorInvalidValue;
    const int64_t tiles = ((batch + g.pack - 1) / g.pack) * (g.diag ? 1 : (g.N + BN - 1) / BN);
    gemm_kernel<BN, BMN><<<(int)std::min<int64_t>(tiles, sms), NTH, smem, s>>>(ma, mb, g, 0, (int)batch);
    return cudaGetLastError();
  }
  if (!make_map(&ma, As, batch, g.M, g.K, BM) ||
      !(BMN ? make_map_mn(&mb, Bs, batch, g.N, g.K) : make_map(&mb, Bs, batch, g.N, g.K, BN)))
    return cudaErrorInvalidValue;
  const int64_t per_z = (int64_t)((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
  const int64_t zmax = std::max<int64_t>(1, (int64_t)1 << 30) / per_z;  // tile index fits an int
  for (int64_t z0 = 0; z0 < batch; z0 += zmax) {
    const int nz = (int)std::min<int64_t>(zmax, batch - z0);
    const int64_t tiles = per_z * nz;
    const int grid = (int)std::min<int64_t>(tiles, sms);
    gemm_kernel<BN, BMN><<<grid, NTH, smem, s>>>(ma, mb, g, (int)z0, nz);
  }
  return cudaGetLastError();
}

bool usable(int rows, int cols) {
  const int D = std::min(rows, cols);
  // K-major rows of the split arrays are TMA strides: a multiple of 16 bytes
  return D >= 128 && D % 8 == 0 && std::max(rows, cols) % 8 == 0 && encode_fn() != nullptr;
}

bool usable_packed(int rows, int cols) {
  const int D = std::min(rows, cols), E = std::max(rows, cols);
  return D == 64 && E % 8 == 0 && encode_fn() != nullptr;
}

cudaError_t gemm(const __half* As, const __half* Bs, const EpiArgs& g, int64_t batch, cudaStream_t s, bool b_mn) {
  if (g.pack && g.diag) return gemm_bn<128, false>(As, Bs, g, batch, s);
  if (b_mn) return g.N >= 256 ? gemm_bn<256, true>(As, Bs, g, batch, s) : gemm_bn<128, true>(As, Bs, g, batch, s);
  return g.N >= 256 ? gemm_bn<256, false>(As, Bs, g, batch, s) : gemm_bn<128, false>(As, Bs, g, batch, s);
}

}  // namespace pet2
}  // namespace atlas
