// Banded causal attention with RoPE (include/atlas_swa.h) on the tcgen05 tensor
// cores: the attention core of atlas_jax/model.py:77-135 for the MAG hybrid.
//
// Tiles are 128 queries x 128 keys x D = 64, bf16 operands in shared memory in the
// core-matrix layout of tc_ops.cuh, float32 accumulators in TMEM.  One CTA of four
// warps owns one 128-row block; thread i owns TMEM lane i, i.e. one query row (the
// forward and dQ kernels) or one key row (the dK/dV kernel), so every row
// statistic of the softmax stays in that thread's registers: no shuffles, no
// shared-memory reductions.  Only the band's key blocks are visited:
// ceil((window + 128) / 128) + 1 of them per row block instead of T / 128.
//
//   forward  per key block: S = Q K^T (TMEM), online softmax in registers,
//            P (bf16) -> smem, O_blk = P V (TMEM), O = O * corr + O_blk.
//   backward delta = rowsum(dO * O); dK/dV kernel per key block over its query
//            blocks: S^T = K Q^T and dP^T = V dO^T, P^T = exp(S^T - lse),
//            dS^T = P^T (dP^T - delta), dV += P^T dO, dK += dS^T Q (TMEM);
//            dQ kernel per query block over its key blocks: dQ += dS K.
//   RoPE (model.py:49-75) is applied to q and k as the tiles are loaded, and its
//   transpose to dq and dk as they are stored.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "atlas_swa.h"
#include "common.cuh"
#include "scan_internal.h"
#include "tc_ops.cuh"

namespace atlas {
namespace swa {

using namespace tcx;
constexpr int HD = 64;   // head dim
constexpr int BR = 128;  // rows per block (queries or keys)
constexpr int TILE = BR * HD * 2;       // one 128 x 64 bf16 tile
constexpr int PTILE = BR * BR * 2;      // one 128 x 128 bf16 tile
constexpr float LOG2E = 1.4426950408889634f;

struct Args {
  AtlasSwaParams p;
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  __nv_bfloat16 *out, *dq, *dk, *dv;
  float* lse;
  float* delta;
  int* status;
};

__device__ __forceinline__ uint8_t* align128(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 127) & ~(uintptr_t)127);
}

__device__ __forceinline__ void tmem_ld32x(uint32_t taddr, float* v) {
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + 16, v + 16);
}

// RoPE inverse frequencies, model.py:54-55: 1 / 10000^(2i / D)
__device__ __forceinline__ void init_invf(float* invf) {
  if (threadIdx.x < HD / 2) invf[threadIdx.x] = 1.0f / powf(10000.0f, (float)(2 * threadIdx.x) / (float)HD);
}

// Loads rows [r0, r0 + 128) of head (b, h) of a (B, T, H, 64) bf16 tensor into a
// 128 x 64 core-matrix tile (K-major for rows-as-M/N operands, MN-major when the rows
// are the K index), zero rows outside [0, T).  With rope, rows are rotated by their
// position (model.py:66-75: halves x1 = x[:32], x2 = x[32:]).  Each thread moves
// 16-byte groups c8 and c8 + 4 of a row, the two halves a rotation pairs.
__device__ void load_tile(uint8_t* tile, const __nv_bfloat16* x, int b, int h, int r0, int T, int H, bool rope,
                          const float* invf) {
  for (int u = threadIdx.x; u < BR * 4; u += blockDim.x) {
    const int r = u >> 2, c8 = u & 3, t = r0 + r;
    uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
    if (t >= 0 && t < T) {
      const __nv_bfloat16* row = x + (((size_t)b * T + t) * H + h) * HD;
      lo = *(const uint4*)(row + 8 * c8);
      hi = *(const uint4*)(row + 32 + 8 * c8);
      if (rope) {
        __nv_bfloat16* x1 = (__nv_bfloat16*)&lo;
        __nv_bfloat16* x2 = (__nv_bfloat16*)&hi;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float sn, cs;
          sincosf((float)t * invf[8 * c8 + j], &sn, &cs);
          const float a = __bfloat162float(x1[j]), bb = __bfloat162float(x2[j]);
          x1[j] = __float2bfloat16_rn(a * cs - bb * sn);
          x2[j] = __float2bfloat16_rn(bb * cs + a * sn);
        }
      }
    }
    *(uint4*)(tile + cm_off(r, 8 * c8, HD)) = lo;
    *(uint4*)(tile + cm_off(r, 32 + 8 * c8, HD)) = hi;
  }
}

// Writes one float row (64 values, this thread's) to (B, T, H, 64) bf16 at position
// t, optionally through the transpose of RoPE (the cotangent of a rotated input).
__device__ void store_row(__nv_bfloat16* x, int b, int h, int t, int T, int H, float* v, bool rope_t,
                          const float* invf) {
  if (t >= T) return;
  if (rope_t) {
#pragma unroll
    for (int i = 0; i < HD / 2; ++i) {  // [x1; x2] -> [x1 c + x2 s; x2 c - x1 s]
      float sn, cs;
      sincosf((float)t * invf[i], &sn, &cs);
      const float a = v[i], bb = v[i + 32];
      v[i] = a * cs + bb * sn;
      v[i + 32] = bb * cs - a * sn;
    }
  }
  __nv_bfloat16* row = x + (((size_t)b * T + t) * H + h) * HD;
#pragma unroll
  for (int c = 0; c < HD; c += 8) {
    uint4 pk;
    __nv_bfloat162* p2 = (__nv_bfloat162*)&pk;
#pragma unroll
    for (int j = 0; j < 4; ++j) p2[j] = __floats2bfloat162_rn(v[c + 2 * j], v[c + 2 * j + 1]);
    *(uint4*)(row + c) = pk;
  }
}

// 16 bf16 values of row r, columns c0..c0+15, into a 128-column core-matrix tile
__device__ __forceinline__ void store16(uint8_t* tile, int r, int c0, const float* v) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint4 pk;
    __nv_bfloat162* p2 = (__nv_bfloat162*)&pk;
#pragma unroll
    for (int j = 0; j < 4; ++j) p2[j] = __floats2bfloat162_rn(v[8 * half + 2 * j], v[8 * half + 2 * j + 1]);
    *(uint4*)(tile + cm_off(r, c0 + 8 * half, BR)) = pk;
  }
}

// D (+)= A B^T-style products over K: A (128 x K) K-major tile with tileC = ka;
// B either K-major (rows = N, tileC = kb) or MN-major (rows = K, tileC = N).
__device__ __forceinline__ void mma_tiles(uint32_t tmd, const uint8_t* A, int a_cols, const uint8_t* Bt, int b_cols,
                                          bool b_mn, int N, int K, bool accumulate) {
  const uint32_t id = idesc_bf16(128, N, false, b_mn);
  for (int ks = 0; ks < K / 16; ++ks) {
    const uint64_t da = desc_kmajor(smem_u32(A) + (uint32_t)ks * 256, a_cols);
    const uint64_t db = b_mn ? desc_mnmajor(smem_u32(Bt) + (uint32_t)(ks * 2) * (uint32_t)(b_cols * 16), b_cols)
                             : desc_kmajor(smem_u32(Bt) + (uint32_t)ks * 256, b_cols);
    mma_kf16(tmd, da, db, id, (accumulate || ks) ? 1u : 0u);
  }
}

__device__ __forceinline__ void cta_sync() {
  fence_before();
  __syncthreads();
  fence_after();
}

// every thread waits on the MMA completion barrier (bounded; a timeout is recorded
// in the status word and in *bad).  The barrier after the wait makes the verdict
// uniform, so all threads leave the block loop together.
__device__ __forceinline__ bool wait_mma(uint64_t* bar, uint32_t& phase, volatile int* bad, int* status) {
  const bool ok = *bad || mbar_wait(bar, phase);
  phase ^= 1;
  if (!ok) {
    set_status(status, ATLAS_ERR_DEVICE_TIMEOUT);
    *bad = 1;
  }
  cta_sync();
  return !*bad;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
struct FwdSmem {
  uint8_t Q[TILE], K[TILE], V[TILE], P[PTILE];
  float invf[HD / 2];
  uint64_t bar;
  uint32_t tmem;
  volatile int bad;
};

__global__ void __launch_bounds__(128) fwd_kernel(Args a) {
  extern __shared__ uint8_t raw[];
  FwdSmem& s = *(FwdSmem*)align128(raw);
  const AtlasSwaParams& P = a.p;
  const int T = P.T, H = P.H, W = P.window, tid = threadIdx.x, w = tid >> 5;
  const int b = blockIdx.y / H, h = blockIdx.y % H, q0 = blockIdx.x * BR, row = q0 + tid;
  const bool rope = P.rope != 0;
  init_invf(s.invf);
  if (w == 0) {
    tmem_alloc(&s.tmem, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.bar, 1);
    fence_mbar_init();
    s.bad = 0;
  }
  cta_sync();
  const uint32_t tm = s.tmem, lane = (uint32_t)(32 * w) << 16;
  load_tile(s.Q, a.q, b, h, q0, T, H, rope, s.invf);
  const int kb0 = max(0, q0 - W) / BR, kb1 = min(T - 1, q0 + BR - 1) / BR;
  const float sl2 = rsqrtf((float)HD) * LOG2E;  // scores in log2 units
  float m = -INFINITY, lsum = 0.f, o[HD];
#pragma unroll
  for (int i = 0; i < HD; ++i) o[i] = 0.f;
  uint32_t phase = 0;
  for (int kb = kb0; kb <= kb1 && !s.bad; ++kb) {
    const int k0 = kb * BR;
    load_tile(s.K, a.k, b, h, k0, T, H, rope, s.invf);
    load_tile(s.V, a.v, b, h, k0, T, H, false, s.invf);
    fence_async_smem();
    cta_sync();
    if (w == 0) {
      mma_tiles(tm, s.Q, HD, s.K, HD, false, BR, HD, false);  // S = Q K^T
      mma_commit(&s.bar);
    }
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) break;
    // online softmax of this thread's row over the block's keys (model.py:126-131)
    float mx = -INFINITY;
    for (int c = 0; c < BR; c += 16) {
      float v[16];
      tmem_ld16(tm + lane + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int key = k0 + c + j;
        if (key <= row && row - key <= W && key < T) mx = fmaxf(mx, v[j] * sl2);
      }
    }
    const float mn = fmaxf(m, mx);
    const float corr = mn == -INFINITY ? 1.f : exp2f(m - mn);
    float psum = 0.f;
    for (int c = 0; c < BR; c += 16) {
      float v[16];
      tmem_ld16(tm + lane + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int key = k0 + c + j;
        const bool ok = key <= row && row - key <= W && key < T;
        v[j] = ok ? exp2f(v[j] * sl2 - mn) : 0.f;
        psum += v[j];
      }
      store16(s.P, tid, c, v);
    }
    lsum = lsum * corr + psum;
    m = mn;
    fence_async_smem();
    cta_sync();
    if (w == 0) {
      mma_tiles(tm + 128, s.P, BR, s.V, HD, true, HD, BR, false);  // O_blk = P V
      mma_commit(&s.bar);
    }
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) break;
    for (int c = 0; c < HD; c += 32) {
      float v[32];
      tmem_ld32x(tm + lane + 128 + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) o[c + j] = fmaf(o[c + j], corr, v[j]);
    }
    cta_sync();  // the next block's loads overwrite K, V and P
  }
  if (!s.bad && row < T) {
    const float inv = 1.f / lsum;
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] *= inv;
    store_row(a.out, b, h, row, T, H, o, false, s.invf);
    a.lse[((size_t)b * H + h) * T + row] = (m + log2f(lsum)) * (1.f / LOG2E);
  }
  cta_sync();
  if (w == 0) tmem_dealloc(tm, 256);
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
// delta[b][h][t] = sum_d dO * O  (one thread per (b, t, h) row)
__global__ void delta_kernel(Args a) {
  const AtlasSwaParams& P = a.p;
  const long rows = (long)P.B * P.T * P.H;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (long)gridDim.x * blockDim.x) {
    const __nv_bfloat16* o = a.o + (size_t)i * HD;
    const __nv_bfloat16* d = a.dout + (size_t)i * HD;
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < HD; c += 8) {
      const uint4 ov = *(const uint4*)(o + c), dv = *(const uint4*)(d + c);
      const __nv_bfloat162* o2 = (const __nv_bfloat162*)&ov;
      const __nv_bfloat162* d2 = (const __nv_bfloat162*)&dv;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = __bfloat1622float2(o2[j]), y = __bfloat1622float2(d2[j]);
        acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
      }
    }
    const int h = (int)(i % P.H), t = (int)((i / P.H) % P.T), b = (int)(i / ((long)P.H * P.T));
    a.delta[((size_t)b * P.H + h) * P.T + t] = acc;
  }
}

struct KVSmem {
  uint8_t K[TILE], V[TILE], Q[TILE], dO[TILE], Pt[PTILE], dSt[PTILE];
  float lse2[BR], delta[BR], invf[HD / 2];
  uint64_t bar;
  uint32_t tmem;
  volatile int bad;
};

// dK, dV for one block of 128 keys over the query blocks that see it
__global__ void __launch_bounds__(128) dkv_kernel(Args a) {
  extern __shared__ uint8_t raw[];
  KVSmem& s = *(KVSmem*)align128(raw);
  const AtlasSwaParams& P = a.p;
  const int T = P.T, H = P.H, W = P.window, tid = threadIdx.x, w = tid >> 5;
  const int b = blockIdx.y / H, h = blockIdx.y % H, k0 = blockIdx.x * BR, kr = k0 + tid;
  const bool rope = P.rope != 0;
  init_invf(s.invf);
  if (w == 0) {
    tmem_alloc(&s.tmem, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.bar, 1);
    fence_mbar_init();
    s.bad = 0;
  }
  cta_sync();
  const uint32_t tm = s.tmem, lane = (uint32_t)(32 * w) << 16;
  load_tile(s.K, a.k, b, h, k0, T, H, rope, s.invf);
  load_tile(s.V, a.v, b, h, k0, T, H, false, s.invf);
  const int qb0 = k0 / BR, qb1 = min(T - 1, k0 + BR - 1 + W) / BR;
  const float sl2 = rsqrtf((float)HD) * LOG2E;
  const size_t bh = (size_t)b * H + h;
  uint32_t phase = 0;
  for (int qb = qb0; qb <= qb1; ++qb) {
    const int q0 = qb * BR;
    load_tile(s.Q, a.q, b, h, q0, T, H, rope, s.invf);
    load_tile(s.dO, a.dout, b, h, q0, T, H, false, s.invf);
    {
      const int t = q0 + tid;
      s.lse2[tid] = t < T ? a.lse[bh * T + t] * LOG2E : 0.f;
      s.delta[tid] = t < T ? a.delta[bh * T + t] : 0.f;
    }
    fence_async_smem();
    cta_sync();
    if (w == 0) {
      mma_tiles(tm, s.K, HD, s.Q, HD, false, BR, HD, false);         // S^T = K Q^T
      mma_tiles(tm + 128, s.V, HD, s.dO, HD, false, BR, HD, false);  // dP^T = V dO^T
      mma_commit(&s.bar);
    }
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) break;
    for (int c = 0; c < BR; c += 16) {
      float sv[16], dp[16];
      tmem_ld16(tm + lane + c, sv);
      tmem_ld16(tm + lane + 128 + c, dp);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int qq = q0 + c + j;
        const bool ok = kr <= qq && qq - kr <= W && qq < T && kr < T;
        const float pr = ok ? exp2f(sv[j] * sl2 - s.lse2[c + j]) : 0.f;
        sv[j] = pr;
        dp[j] = pr * (dp[j] - s.delta[c + j]);
      }
      store16(s.Pt, tid, c, sv);
      store16(s.dSt, tid, c, dp);
    }
    fence_async_smem();
    cta_sync();
    if (w == 0) {
      mma_tiles(tm + 256, s.Pt, BR, s.dO, HD, true, HD, BR, qb > qb0);  // dV += P^T dO
      mma_tiles(tm + 320, s.dSt, BR, s.Q, HD, true, HD, BR, qb > qb0);  // dK += dS^T Q
      mma_commit(&s.bar);
    }
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) break;
  }
  if (!s.bad) {
    float v[HD];
    tmem_ld32x(tm + lane + 256, v);
    tmem_ld32x(tm + lane + 288, v + 32);
    tmem_wait_ld();
    store_row(a.dv, b, h, kr, T, H, v, false, s.invf);
    tmem_ld32x(tm + lane + 320, v);
    tmem_ld32x(tm + lane + 352, v + 32);
    tmem_wait_ld();
    const float sc = rsqrtf((float)HD);
#pragma unroll
    for (int i = 0; i < HD; ++i) v[i] *= sc;
    store_row(a.dk, b, h, kr, T, H, v, rope, s.invf);
  }
  cta_sync();
  if (w == 0) tmem_dealloc(tm, 512);
}

struct QSmem {
  uint8_t Q[TILE], dO[TILE], K[TILE], V[TILE], dS[PTILE];
  float invf[HD / 2];
  uint64_t bar;
  uint32_t tmem;
  volatile int bad;
};

// dQ for one block of 128 queries over its band of key blocks
__global__ void __launch_bounds__(128) dq_kernel(Args a) {
  extern __shared__ uint8_t raw[];
  QSmem& s = *(QSmem*)align128(raw);
  const AtlasSwaParams& P = a.p;
  const int T = P.T, H = P.H, W = P.window, tid = threadIdx.x, w = tid >> 5;
  const int b = blockIdx.y / H, h = blockIdx.y % H, q0 = blockIdx.x * BR, row = q0 + tid;
  const bool rope = P.rope != 0;
  init_invf(s.invf);
  if (w == 0) {
    tmem_alloc(&s.tmem, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.bar, 1);
    fence_mbar_init();
    s.bad = 0;
  }
  cta_sync();
  const uint32_t tm = s.tmem, lane = (uint32_t)(32 * w) << 16;
  load_tile(s.Q, a.q, b, h, q0, T, H, rope, s.invf);
  load_tile(s.dO, a.dout, b, h, q0, T, H, false, s.invf);
  const size_t bh = (size_t)b * H + h;
  const float lse2 = row < T ? a.lse[bh * T + row] * LOG2E : 0.f;
  const float dl = row < T ? a.delta[bh * T + row] : 0.f;
  const int kb0 = max(0, q0 - W) / BR, kb1 = min(T - 1, q0 + BR - 1) / BR;
  const float sl2 = rsqrtf((float)HD) * LOG2E;
  uint32_t phase = 0;
  for (int kb = kb0; kb <= kb1; ++kb) {
    const int k0 = kb * BR;
    load_tile(s.K, a.k, b, h, k0, T, H, rope, s.invf);
    load_tile(s.V, a.v, b, h, k0, T, H, false, s.invf);
    fence_async_smem();
    cta_sync();
    if (w == 0) {
      mma_tiles(tm, s.Q, HD, s.K, HD, false, BR, HD, false);         // S = Q K^T
      mma_tiles(tm + 128, s.dO, HD, s.V, HD, false, BR, HD, false);  // dP = dO V^T
      mma_commit(&s.bar);
    }
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) break;
    for (int c = 0; c < BR; c += 16) {
      float sv[16], dp[16];
      tmem_ld16(tm + lane + c, sv);
      tmem_ld16(tm + lane + 128 + c, dp);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int key = k0 + c + j;
        const bool ok = key <= row && row - key <= W && key < T && row < T;
        const float pr = ok ? exp2f(sv[j] * sl2 - lse2) : 0.f;
        dp[j] = pr * (dp[j] - dl);
      }
      store16(s.dS, tid, c, dp);
    }
    fence_async_smem();
    cta_sync();
    if (w == 0) {
      mma_tiles(tm + 256, s.dS, BR, s.K, HD, true, HD, BR, kb > kb0);  // dQ += dS K
      mma_commit(&s.bar);
    }
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) break;
  }
  if (!s.bad) {
    float v[HD];
    tmem_ld32x(tm + lane + 256, v);
    tmem_ld32x(tm + lane + 288, v + 32);
    tmem_wait_ld();
    const float sc = rsqrtf((float)HD);
#pragma unroll
    for (int i = 0; i < HD; ++i) v[i] *= sc;
    store_row(a.dq, b, h, row, T, H, v, rope, s.invf);
  }
  cta_sync();
  if (w == 0) tmem_dealloc(tm, 512);
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
static int check(const AtlasSwaParams* p) {
  if (!p) return report_error(ATLAS_ERR_INVALID_ARGUMENT, "params is NULL");
  if (p->abi_version != ATLAS_ABI_VERSION) return report_error(ATLAS_ERR_INVALID_ARGUMENT, "abi_version mismatch");
  if (p->B <= 0 || p->T <= 0 || p->H <= 0 || p->window < 0)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "B, T, H must be positive and window >= 0");
  if (p->D != HD) return report_error(ATLAS_ERR_UNSUPPORTED, "head_dim must be 64");
  clear_error();
  return ATLAS_OK;
}

template <class S>
static size_t smem_of() {
  return sizeof(S) + 128;
}

static int launch_status(cudaError_t e) {
  return e == cudaSuccess ? ATLAS_OK : report_error(ATLAS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace swa
}  // namespace atlas

using namespace atlas;
using namespace atlas::swa;

extern "C" int atlas_swa_fwd(const AtlasSwaParams* p, const void* q, const void* k, const void* v, void* o,
                             float* lse, void* stream) {
  int rc = check(p);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse) return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  Args a{};
  a.p = *p;
  a.q = (const __nv_bfloat16*)q;
  a.k = (const __nv_bfloat16*)k;
  a.v = (const __nv_bfloat16*)v;
  a.out = (__nv_bfloat16*)o;
  a.lse = lse;
  a.status = device_status_ptr();
  const size_t sm = smem_of<FwdSmem>();
  cudaError_t e = cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return launch_status(e);
  fwd_kernel<<<dim3((p->T + BR - 1) / BR, p->B * p->H), 128, sm, (cudaStream_t)stream>>>(a);
  return launch_status(cudaGetLastError());
}

extern "C" size_t atlas_swa_workspace_bytes(const AtlasSwaParams* p) {
  if (check(p) != ATLAS_OK) return 0;
  return (size_t)p->B * p->H * p->T * sizeof(float);
}

extern "C" int atlas_swa_bwd(const AtlasSwaParams* p, const void* q, const void* k, const void* v, const void* o,
                             const float* lse, const void* dout, void* dq, void* dk, void* dv, void* workspace,
                             size_t workspace_bytes, void* stream) {
  int rc = check(p);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (!workspace || workspace_bytes < (size_t)p->B * p->H * p->T * sizeof(float))
    return report_error(ATLAS_ERR_WORKSPACE, "workspace smaller than atlas_swa_workspace_bytes()");
  Args a{};
  a.p = *p;
  a.q = (const __nv_bfloat16*)q;
  a.k = (const __nv_bfloat16*)k;
  a.v = (const __nv_bfloat16*)v;
  a.o = (const __nv_bfloat16*)o;
  a.dout = (const __nv_bfloat16*)dout;
  a.dq = (__nv_bfloat16*)dq;
  a.dk = (__nv_bfloat16*)dk;
  a.dv = (__nv_bfloat16*)dv;
  a.lse = const_cast<float*>(lse);
  a.delta = (float*)workspace;
  a.status = device_status_ptr();
  cudaStream_t s = (cudaStream_t)stream;
  const long rows = (long)p->B * p->T * p->H;
  delta_kernel<<<(int)std::min<long>((rows + 255) / 256, 148L * 16), 256, 0, s>>>(a);
  const dim3 grid((p->T + BR - 1) / BR, p->B * p->H);
  size_t sm = smem_of<KVSmem>();
  cudaError_t e = cudaFuncSetAttribute(dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return launch_status(e);
  dkv_kernel<<<grid, 128, sm, s>>>(a);
  // one CTA per SM (as for dkv_kernel): each allocates 512 TMEM columns, all of the SM's
  sm = std::max(smem_of<QSmem>(), (size_t)120 * 1024);
  e = cudaFuncSetAttribute(dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return launch_status(e);
  dq_kernel<<<grid, 128, sm, s>>>(a);
  return launch_status(cudaGetLastError());
}
