// Banded causal attention with RoPE (include/atlas_swa.h) on the tcgen05 tensor
// cores: the attention core of atlas_jax/model.py:77-135 for the MAG hybrid.
//
// Tiles are 128 queries x 128 keys x D = 64, bf16 operands in shared memory in the
// core-matrix layout of tc_ops.cuh, float32 accumulators in TMEM.  One CTA owns one
// 128-row block.  Warp w reads TMEM lane quadrant w % 4 (rows 32 (w % 4) ..): in the
// forward eight warps split a row's columns in halves (w / 4), so the softmax
// statistics of a row need one exchange through shared memory per key block; the
// backward kernels run sixteen warps, a column quarter (w / 4) each.
// Only the band's key blocks are visited: ceil((window + 128) / 128) + 1 of them per
// row block instead of T / 128.
//
//   rope     a pre-pass rotates q and k once (model.py:49-75, 117-121) into the
//            workspace; the tiles are then plain 16-byte copies (cp.async), the next
//            block's tiles in flight while the current block computes.
//   forward  per key block: S = Q K^T (TMEM), online softmax in registers,
//            P (bf16) -> smem, O_blk = P V (TMEM), O = O * corr + O_blk.
//   backward delta = rowsum(dO * O); dK/dV kernel per key block over its query
//            blocks: S^T = K Q^T and dP^T = V dO^T, P^T = exp(S^T - lse),
//            dS^T = P^T (dP^T - delta), dV += P^T dO, dK += dS^T Q (TMEM);
//            dQ kernel per query block over its key blocks: dQ += dS K.  dq and dk
//            leave through the transpose of the rotation.
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
constexpr int NTH = 256;
constexpr int NTB = 512;  // backward kernels: four warps per TMEM lane quadrant, a column quarter each
constexpr int TILE = BR * HD * 2;   // one 128 x 64 bf16 tile
constexpr int PTILE = BR * BR * 2;  // one 128 x 128 bf16 tile
constexpr float LOG2E = 1.4426950408889634f;

struct Args {
  AtlasSwaParams p;
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  __nv_bfloat16 *out, *dq, *dk, *dv;
  __nv_bfloat16 *qr, *kr;  // rotated q, k (workspace)
  float* lse;
  float* delta;
  int* status;
};

__device__ __forceinline__ uint8_t* align128(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 127) & ~(uintptr_t)127);
}

// RoPE inverse frequency i, model.py:54-55: 1 / 10000^(2i / D)
__device__ __forceinline__ float inv_freq(int i) { return 1.0f / powf(10000.0f, (float)(2 * i) / (float)HD); }

// q, k -> rotated qr, kr (model.py:66-75: x1 = x[:32], x2 = x[32:]; out = [x1 c - x2 s,
// x2 c + x1 s]); without rope a plain copy.  One thread per (row, group of 8 pairs, q|k).
__global__ void rope_kernel(Args a) {
  const AtlasSwaParams& P = a.p;
  const long units = (long)P.B * P.T * P.H * 4 * 2;
  for (long u = (long)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (long)gridDim.x * blockDim.x) {
    const int which = (int)(u & 1), c8 = (int)((u >> 1) & 3);
    const long rowi = u >> 3;
    const int t = (int)((rowi / P.H) % P.T);
    const __nv_bfloat16* src = (which ? a.k : a.q) + (size_t)rowi * HD;
    __nv_bfloat16* dst = (which ? a.kr : a.qr) + (size_t)rowi * HD;
    uint4 lo = *(const uint4*)(src + 8 * c8), hi = *(const uint4*)(src + 32 + 8 * c8);
    if (P.rope) {
      __nv_bfloat16* x1 = (__nv_bfloat16*)&lo;
      __nv_bfloat16* x2 = (__nv_bfloat16*)&hi;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float sn, cs;
        sincosf((float)t * inv_freq(8 * c8 + j), &sn, &cs);
        const float x = __bfloat162float(x1[j]), y = __bfloat162float(x2[j]);
        x1[j] = __float2bfloat16_rn(x * cs - y * sn);
        x2[j] = __float2bfloat16_rn(y * cs + x * sn);
      }
    }
    *(uint4*)(dst + 8 * c8) = lo;
    *(uint4*)(dst + 32 + 8 * c8) = hi;
  }
}

// 2^x on the SFU (ex2.approx: relative error ~2^-22; 2^-inf = 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Issues the copies of rows [r0, r0 + 128) of head (b, h) of a (B, T, H, 64) bf16
// tensor into a 128 x 64 core-matrix tile (K-major when the rows are the M/N index,
// MN-major when they are the K index); rows outside [0, T) are zero-filled.
__device__ void load_tile_async(uint8_t* tile, const __nv_bfloat16* x, int b, int h, int r0, int T, int H) {
  for (int u = threadIdx.x; u < BR * 8; u += blockDim.x) {
    const int r = u >> 3, c8 = u & 7, t = r0 + r;
    uint8_t* d = tile + cm_off(r, 8 * c8, HD);
    if (t >= 0 && t < T)
      cp_async16(d, x + (((size_t)b * T + t) * H + h) * HD + 8 * c8);
    else
      *(uint4*)d = make_uint4(0, 0, 0, 0);
  }
}

// Column split of a 64-wide row between the two warps of a lane quadrant: half ch
// owns columns [16 ch, 16 ch + 16) and [32 + 16 ch, 32 + 16 ch + 16), so both halves of
// every RoPE pair (i, i + 32) stay with one thread.
__device__ __forceinline__ int col_of(int ch, int j) { return (j < 16 ? 0 : 16) + 16 * ch + j; }

// Writes this thread's 32 values of row t (columns col_of(ch, 0..31)) of a
// (B, T, H, 64) bf16 tensor, optionally through the transpose of RoPE (the cotangent
// of a rotated input: [g1; g2] -> [g1 c + g2 s; g2 c - g1 s]).
__device__ void store_half_row(__nv_bfloat16* x, int b, int h, int t, int T, int H, int ch, float* v, bool rope_t) {
  if (t >= T) return;
  if (rope_t) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float sn, cs;
      sincosf((float)t * inv_freq(16 * ch + j), &sn, &cs);
      const float g1 = v[j], g2 = v[16 + j];
      v[j] = g1 * cs + g2 * sn;
      v[16 + j] = g2 * cs - g1 * sn;
    }
  }
  __nv_bfloat16* row = x + (((size_t)b * T + t) * H + h) * HD;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint4 pk;
    __nv_bfloat162* p2 = (__nv_bfloat162*)&pk;
#pragma unroll
    for (int j = 0; j < 4; ++j) p2[j] = __floats2bfloat162_rn(v[8 * g + 2 * j], v[8 * g + 2 * j + 1]);
    *(uint4*)(row + col_of(ch, 8 * g)) = pk;
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

// this thread's 32 columns col_of(ch, .) of a 64-column TMEM accumulator row
__device__ __forceinline__ void tmem_ld_half(uint32_t taddr, int ch, float* v) {
  tmem_ld16(taddr + 16 * ch, v);
  tmem_ld16(taddr + 32 + 16 * ch, v + 16);
}

// D (+)= A * B over K: A (128 x K) K-major tile with a_cols columns; B either K-major
// (rows = N, b_cols = K) or MN-major (rows = K, b_cols = N).
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

// cp.async copies of this thread landed -> visible to every thread and to the tensor core
__device__ __forceinline__ void tiles_ready() {
  cp_async_wait<0>();
  fence_async_smem();
  cta_sync();
}

struct Roles {
  uint32_t tm, lane;
  int w, qd, ch, rloc;
};

// TMEM allocation (warp 0), barrier init, and this thread's roles
template <class S>
__device__ __forceinline__ Roles setup(S& s, uint32_t cols) {
  const int tid = threadIdx.x, w = tid >> 5;
  if (w == 0) {
    tmem_alloc(&s.tmem, cols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.bar, 1);
    fence_mbar_init();
    s.bad = 0;
  }
  cta_sync();
  Roles u;
  u.w = w;
  u.qd = w & 3;
  u.ch = w >> 2;
  u.rloc = 32 * u.qd + (tid & 31);
  u.tm = s.tmem;
  u.lane = (uint32_t)(32 * u.qd) << 16;
  return u;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
struct FwdSmem {
  uint8_t Q[TILE], K[2][TILE], V[TILE], P[PTILE];
  float mx[2][BR], ls[2][BR];
  uint64_t bar;
  uint32_t tmem;
  volatile int bad;
};

__global__ void __launch_bounds__(NTH) fwd_kernel(Args a) {
  extern __shared__ uint8_t raw[];
  FwdSmem& s = *(FwdSmem*)align128(raw);
  const AtlasSwaParams& P = a.p;
  const int T = P.T, H = P.H, W = P.window;
  const int b = blockIdx.y / H, h = blockIdx.y % H, q0 = blockIdx.x * BR;
  const Roles u = setup(s, 256);
  const int row = q0 + u.rloc, ch = u.ch;
  const int kb0 = max(0, q0 - W) / BR, kb1 = min(T - 1, q0 + BR - 1) / BR;
  load_tile_async(s.Q, a.qr, b, h, q0, T, H);
  load_tile_async(s.K[0], a.kr, b, h, kb0 * BR, T, H);
  cp_async_commit();
  load_tile_async(s.V, a.v, b, h, kb0 * BR, T, H);
  cp_async_commit();
  const float sl2 = rsqrtf((float)HD) * LOG2E;  // scores in log2 units
  float m = -INFINITY, lsum = 0.f, o[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i] = 0.f;
  uint32_t phase = 0;
  bool done = true;
  for (int kb = kb0; kb <= kb1; ++kb) {
    const int k0 = kb * BR, cur = (kb - kb0) & 1;
    cp_async_wait<1>();  // Q and K[cur]; V may still be in flight
    fence_async_smem();
    cta_sync();
    if (u.w == 0) {
      mma_tiles(u.tm, s.Q, HD, s.K[cur], HD, false, BR, HD, false);  // S = Q K^T
      mma_commit(&s.bar);
    }
    if (kb < kb1) load_tile_async(s.K[cur ^ 1], a.kr, b, h, k0 + BR, T, H);
    cp_async_commit();  // (possibly empty group: keeps the group count uniform)
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) {
      done = false;
      break;
    }
    // online softmax over this block's keys (model.py:126-131); this thread holds
    // keys [64 ch, 64 ch + 64) of its row.  Blocks wholly inside the band skip the mask.
    float sv[64];
#pragma unroll
    for (int c = 0; c < 64; c += 16) tmem_ld16(u.tm + u.lane + 64 * ch + c, sv + c);
    tmem_wait_ld();
    const bool full = k0 + BR - 1 <= q0 && q0 + BR - 1 - k0 <= W && k0 + BR <= T;
    float mx = -INFINITY;
    if (full) {
#pragma unroll
      for (int j = 0; j < 64; ++j) mx = fmaxf(mx, sv[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const int key = k0 + 64 * ch + j;
        if (!(key <= row && row - key <= W && key < T)) sv[j] = -INFINITY;
        mx = fmaxf(mx, sv[j]);
      }
    }
    s.mx[ch][u.rloc] = mx * sl2;
    cta_sync();
    const float mn = fmaxf(m, fmaxf(s.mx[0][u.rloc], s.mx[1][u.rloc]));
    const float corr = mn == -INFINITY ? 1.f : ex2(m - mn);
    const float msub = mn == -INFINITY ? 0.f : mn;
    float psum = 0.f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      sv[j] = ex2(fmaf(sv[j], sl2, -msub));  // masked keys: ex2(-inf) = 0
      psum += sv[j];
    }
#pragma unroll
    for (int c = 0; c < 64; c += 16) store16(s.P, u.rloc, 64 * ch + c, sv + c);
    lsum = lsum * corr + psum;
    m = mn;
    cp_async_wait<1>();  // V of this block (the newest group is the next K)
    fence_async_smem();
    cta_sync();
    if (u.w == 0) {
      mma_tiles(u.tm + 128, s.P, BR, s.V, HD, true, HD, BR, false);  // O_blk = P V
      mma_commit(&s.bar);
    }
    __syncwarp();
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) {
      done = false;
      break;
    }
    if (kb < kb1) load_tile_async(s.V, a.v, b, h, k0 + BR, T, H);
    cp_async_commit();
    float v[32];
    tmem_ld_half(u.tm + u.lane + 128, ch, v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = fmaf(o[j], corr, v[j]);
  }
  cp_async_wait<0>();
  if (done) {
    s.ls[ch][u.rloc] = lsum;
    cta_sync();
    const float tot = s.ls[0][u.rloc] + s.ls[1][u.rloc];
    if (row < T) {
      const float inv = 1.f / tot;
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] *= inv;
      store_half_row(a.out, b, h, row, T, H, ch, o, false);
      if (ch == 0) a.lse[((size_t)b * H + h) * T + row] = (m + log2f(tot)) * (1.f / LOG2E);
    }
  }
  cta_sync();
  if (u.w == 0) tmem_dealloc(u.tm, 256);
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
  uint8_t K[TILE], V[TILE], Q[3][TILE], dO[3][TILE], Pt[PTILE], dSt[PTILE];
  float lse2[3][BR], delta[3][BR];
  uint64_t bar;   // S^T / dP^T group
  uint64_t barv;  // dV / dK group
  uint32_t tmem;
  volatile int bad;
};

// dK, dV of one block of 128 keys over the query blocks that see it.  Software
// pipelined over the query blocks (three Q / dO buffers): once the threads hold query
// block qb's S^T and dP^T in registers, the MMAs of block qb + 1's S^T and dP^T are
// issued into the same TMEM columns, so they run while the threads form P^T and dS^T
// of block qb; block qb's dV / dK MMAs follow them on the tensor pipe.
__global__ void __launch_bounds__(NTB, 1) dkv_kernel(Args a) {
  extern __shared__ uint8_t raw[];
  KVSmem& s = *(KVSmem*)align128(raw);
  const AtlasSwaParams& P = a.p;
  const int T = P.T, H = P.H, W = P.window, tid = threadIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y % H, k0 = blockIdx.x * BR;
  const Roles u = setup(s, 512);
  if (tid == 0) {
    mbar_init(&s.barv, 1);
    fence_mbar_init();
  }
  const int kr = k0 + u.rloc, ch = u.ch;
  const int qb0 = k0 / BR, qb1 = min(T - 1, k0 + BR - 1 + W) / BR;
  const size_t bh = (size_t)b * H + h;
  auto stage = [&](int qb, int buf) {  // Q, dO tiles and the queries' lse, delta
    load_tile_async(s.Q[buf], a.qr, b, h, qb * BR, T, H);
    load_tile_async(s.dO[buf], a.dout, b, h, qb * BR, T, H);
    if (tid < BR) {
      const int t = qb * BR + tid;
      s.lse2[buf][tid] = t < T ? a.lse[bh * T + t] * LOG2E : 0.f;
      s.delta[buf][tid] = t < T ? a.delta[bh * T + t] : 0.f;
    }
  };
  auto issue_sdp = [&](int buf) {
    if (u.w == 0) {
      mma_tiles(u.tm, s.K, HD, s.Q[buf], HD, false, BR, HD, false);         // S^T = K Q^T
      mma_tiles(u.tm + 128, s.V, HD, s.dO[buf], HD, false, BR, HD, false);  // dP^T = V dO^T
      mma_commit(&s.bar);
    }
    __syncwarp();
  };
  load_tile_async(s.K, a.kr, b, h, k0, T, H);
  load_tile_async(s.V, a.v, b, h, k0, T, H);
  stage(qb0, 0);
  cp_async_commit();
  if (qb0 + 1 <= qb1) stage(qb0 + 1, 1);
  cp_async_commit();
  cp_async_wait<1>();  // K, V and block qb0's tiles
  fence_async_smem();
  cta_sync();
  issue_sdp(0);
  const float sl2 = rsqrtf((float)HD) * LOG2E;
  uint32_t phase = 0, phase_v = 0;
  bool done = true;
  for (int qb = qb0; qb <= qb1; ++qb) {
    const int q0 = qb * BR, cur = (qb - qb0) % 3;
    const bool full = k0 + BR - 1 <= q0 && q0 + BR - 1 - k0 <= W && q0 + BR <= T;  // no mask needed
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) {  // S^T, dP^T of block qb
      done = false;
      break;
    }
    float sv[32], dp[32];  // this thread's column quarter [32 ch, 32 ch + 32) of the row
#pragma unroll
    for (int c = 0; c < 32; c += 16) {
      tmem_ld16(u.tm + u.lane + 32 * ch + c, sv + c);
      tmem_ld16(u.tm + u.lane + 128 + 32 * ch + c, dp + c);
    }
    tmem_wait_ld();
    // dV / dK of block qb - 1 read Q / dO buffer (qb + 2) % 3 and Pt / dSt
    if (qb > qb0 && !wait_mma(&s.barv, phase_v, &s.bad, a.status)) {
      done = false;
      break;
    }
    if (qb + 2 <= qb1) stage(qb + 2, (qb + 2 - qb0) % 3);
    cp_async_commit();
    if (qb < qb1) {
      cp_async_wait<1>();  // block qb + 1's tiles (the newest group is block qb + 2)
      fence_async_smem();
      cta_sync();          // also: every thread's S^T / dP^T loads of block qb are done
      issue_sdp((qb + 1 - qb0) % 3);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int cc = 32 * ch + j;
      const int qq = q0 + cc;
      const bool ok = full || (kr <= qq && qq - kr <= W && qq < T && kr < T);
      const float pr = ok ? ex2(fmaf(sv[j], sl2, -s.lse2[cur][cc])) : 0.f;
      sv[j] = pr;
      dp[j] = pr * (dp[j] - s.delta[cur][cc]);
    }
#pragma unroll
    for (int c = 0; c < 32; c += 16) {
      store16(s.Pt, u.rloc, 32 * ch + c, sv + c);
      store16(s.dSt, u.rloc, 32 * ch + c, dp + c);
    }
    fence_async_smem();
    cta_sync();
    if (u.w == 0) {
      mma_tiles(u.tm + 256, s.Pt, BR, s.dO[cur], HD, true, HD, BR, qb > qb0);  // dV += P^T dO
      mma_tiles(u.tm + 320, s.dSt, BR, s.Q[cur], HD, true, HD, BR, qb > qb0);  // dK += dS^T Q
      mma_commit(&s.barv);
    }
    __syncwarp();
  }
  if (done && !wait_mma(&s.barv, phase_v, &s.bad, a.status)) done = false;
  cp_async_wait<0>();
  if (done && ch < 2) {  // two warps per lane quadrant write dV / dK (column halves)
    float v[32];
    tmem_ld_half(u.tm + u.lane + 256, ch, v);
    tmem_wait_ld();
    store_half_row(a.dv, b, h, kr, T, H, ch, v, false);
    tmem_ld_half(u.tm + u.lane + 320, ch, v);
    tmem_wait_ld();
    const float sc = rsqrtf((float)HD);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= sc;
    store_half_row(a.dk, b, h, kr, T, H, ch, v, P.rope != 0);
  }
  cta_sync();
  if (u.w == 0) tmem_dealloc(u.tm, 512);
}

struct QSmem {
  uint8_t Q[TILE], dO[TILE], K[3][TILE], V[3][TILE], dS[PTILE];
  uint64_t bar;   // S / dP group
  uint64_t barq;  // dQ group
  uint32_t tmem;
  volatile int bad;
};

// dQ of one block of 128 queries over its band of key blocks, software pipelined
// like dkv_kernel (three K / V buffers; key block kb + 1's S and dP MMAs run while the
// threads form dS of block kb).
__global__ void __launch_bounds__(NTB, 1) dq_kernel(Args a) {
  extern __shared__ uint8_t raw[];
  QSmem& s = *(QSmem*)align128(raw);
  const AtlasSwaParams& P = a.p;
  const int T = P.T, H = P.H, W = P.window, tid = threadIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y % H, q0 = blockIdx.x * BR;
  const Roles u = setup(s, 512);
  if (tid == 0) {
    mbar_init(&s.barq, 1);
    fence_mbar_init();
  }
  const int row = q0 + u.rloc, ch = u.ch;
  const size_t bh = (size_t)b * H + h;
  const float lse2 = row < T ? a.lse[bh * T + row] * LOG2E : 0.f;
  const float dl = row < T ? a.delta[bh * T + row] : 0.f;
  const int kb0 = max(0, q0 - W) / BR, kb1 = min(T - 1, q0 + BR - 1) / BR;
  auto stage = [&](int kb, int buf) {
    load_tile_async(s.K[buf], a.kr, b, h, kb * BR, T, H);
    load_tile_async(s.V[buf], a.v, b, h, kb * BR, T, H);
  };
  auto issue_sdp = [&](int buf) {
    if (u.w == 0) {
      mma_tiles(u.tm, s.Q, HD, s.K[buf], HD, false, BR, HD, false);         // S = Q K^T
      mma_tiles(u.tm + 128, s.dO, HD, s.V[buf], HD, false, BR, HD, false);  // dP = dO V^T
      mma_commit(&s.bar);
    }
    __syncwarp();
  };
  load_tile_async(s.Q, a.qr, b, h, q0, T, H);
  load_tile_async(s.dO, a.dout, b, h, q0, T, H);
  stage(kb0, 0);
  cp_async_commit();
  if (kb0 + 1 <= kb1) stage(kb0 + 1, 1);
  cp_async_commit();
  cp_async_wait<1>();
  fence_async_smem();
  cta_sync();
  issue_sdp(0);
  const float sl2 = rsqrtf((float)HD) * LOG2E;
  uint32_t phase = 0, phase_q = 0;
  bool done = true;
  for (int kb = kb0; kb <= kb1; ++kb) {
    const int k0 = kb * BR, cur = (kb - kb0) % 3;
    const bool full = k0 + BR - 1 <= q0 && q0 + BR - 1 - k0 <= W && q0 + BR <= T;  // no mask needed
    if (!wait_mma(&s.bar, phase, &s.bad, a.status)) {  // S, dP of block kb
      done = false;
      break;
    }
    float sv[32], dp[32];  // this thread's column quarter [32 ch, 32 ch + 32) of the row
#pragma unroll
    for (int c = 0; c < 32; c += 16) {
      tmem_ld16(u.tm + u.lane + 32 * ch + c, sv + c);
      tmem_ld16(u.tm + u.lane + 128 + 32 * ch + c, dp + c);
    }
    tmem_wait_ld();
    // dQ of block kb - 1 read K buffer (kb + 2) % 3 and dS
    if (kb > kb0 && !wait_mma(&s.barq, phase_q, &s.bad, a.status)) {
      done = false;
      break;
    }
    if (kb + 2 <= kb1) stage(kb + 2, (kb + 2 - kb0) % 3);
    cp_async_commit();
    if (kb < kb1) {
      cp_async_wait<1>();
      fence_async_smem();
      cta_sync();  // also: every thread's S / dP loads of block kb are done
      issue_sdp((kb + 1 - kb0) % 3);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int key = k0 + 32 * ch + j;
      const bool ok = full || (key <= row && row - key <= W && key < T && row < T);
      const float pr = ok ? ex2(fmaf(sv[j], sl2, -lse2)) : 0.f;
      dp[j] = pr * (dp[j] - dl);
    }
#pragma unroll
    for (int c = 0; c < 32; c += 16) store16(s.dS, u.rloc, 32 * ch + c, dp + c);
    fence_async_smem();
    cta_sync();
    if (u.w == 0) {
      mma_tiles(u.tm + 256, s.dS, BR, s.K[cur], HD, true, HD, BR, kb > kb0);  // dQ += dS K
      mma_commit(&s.barq);
    }
    __syncwarp();
  }
  if (done && !wait_mma(&s.barq, phase_q, &s.bad, a.status)) done = false;
  cp_async_wait<0>();
  if (done && ch < 2) {  // two warps per lane quadrant write dQ (column halves)
    float v[32];
    tmem_ld_half(u.tm + u.lane + 256, ch, v);
    tmem_wait_ld();
    const float sc = rsqrtf((float)HD);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= sc;
    store_half_row(a.dq, b, h, row, T, H, ch, v, P.rope != 0);
  }
  cta_sync();
  if (u.w == 0) tmem_dealloc(u.tm, 512);
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

static size_t act_bytes(const AtlasSwaParams& p) {
  return ((size_t)p.B * p.T * p.H * HD * 2 + 255) & ~(size_t)255;
}
static size_t ws_bytes(const AtlasSwaParams& p) { return 2 * act_bytes(p) + (size_t)p.B * p.H * p.T * sizeof(float); }

static int launch_status(cudaError_t e) {
  return e == cudaSuccess ? ATLAS_OK : report_error(ATLAS_ERR_CUDA, cudaGetErrorString(e));
}

static int elem_grid(long n) { return (int)std::max(1L, std::min((n + 255) / 256, 148L * 16)); }

// rotated q, k into the workspace
static void carve(Args& a, void* ws) {
  uint8_t* w = (uint8_t*)ws;
  a.qr = (__nv_bfloat16*)w;
  a.kr = (__nv_bfloat16*)(w + act_bytes(a.p));
  a.delta = (float*)(w + 2 * act_bytes(a.p));
}

template <class S>
static cudaError_t set_smem(const void* fn, size_t bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace swa
}  // namespace atlas

using namespace atlas;
using namespace atlas::swa;

extern "C" size_t atlas_swa_workspace_bytes(const AtlasSwaParams* p) {
  if (check(p) != ATLAS_OK) return 0;
  return ws_bytes(*p);
}

extern "C" int atlas_swa_fwd(const AtlasSwaParams* p, const void* q, const void* k, const void* v, void* o,
                             float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check(p);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse) return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (!workspace || workspace_bytes < ws_bytes(*p))
    return report_error(ATLAS_ERR_WORKSPACE, "workspace smaller than atlas_swa_workspace_bytes()");
  Args a{};
  a.p = *p;
  a.q = (const __nv_bfloat16*)q;
  a.k = (const __nv_bfloat16*)k;
  a.v = (const __nv_bfloat16*)v;
  a.out = (__nv_bfloat16*)o;
  a.lse = lse;
  a.status = device_status_ptr();
  carve(a, workspace);
  cudaStream_t s = (cudaStream_t)stream;
  rope_kernel<<<elem_grid((long)p->B * p->T * p->H * 8), 256, 0, s>>>(a);
  const size_t sm = sizeof(FwdSmem) + 128;
  cudaError_t e = set_smem<FwdSmem>((const void*)fwd_kernel, sm);
  if (e != cudaSuccess) return launch_status(e);
  fwd_kernel<<<dim3((p->T + BR - 1) / BR, p->B * p->H), NTH, sm, s>>>(a);
  return launch_status(cudaGetLastError());
}

extern "C" int atlas_swa_bwd(const AtlasSwaParams* p, const void* q, const void* k, const void* v, const void* o,
                             const float* lse, const void* dout, void* dq, void* dk, void* dv, void* workspace,
                             size_t workspace_bytes, void* stream) {
  int rc = check(p);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (!workspace || workspace_bytes < ws_bytes(*p))
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
  a.status = device_status_ptr();
  carve(a, workspace);
  cudaStream_t s = (cudaStream_t)stream;
  rope_kernel<<<elem_grid((long)p->B * p->T * p->H * 8), 256, 0, s>>>(a);
  delta_kernel<<<elem_grid((long)p->B * p->T * p->H), 256, 0, s>>>(a);
  const dim3 grid((p->T + BR - 1) / BR, p->B * p->H);
  // each CTA of these two kernels allocates all 512 TMEM columns of its SM; their
  // shared-memory requests (>= 114 KB) keep them at one CTA per SM
  size_t sm = std::max(sizeof(KVSmem) + 128, (size_t)120 * 1024);
  cudaError_t e = set_smem<KVSmem>((const void*)dkv_kernel, sm);
  if (e != cudaSuccess) return launch_status(e);
  dkv_kernel<<<grid, NTB, sm, s>>>(a);
  sm = std::max(sizeof(QSmem) + 128, (size_t)120 * 1024);
  e = set_smem<QSmem>((const void*)dq_kernel, sm);
  if (e != cudaSuccess) return launch_status(e);
  dq_kernel<<<grid, NTB, sm, s>>>(a);
  return launch_status(cudaGetLastError());
}
