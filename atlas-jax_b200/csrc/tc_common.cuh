// Shared pieces of the tcgen05 scan kernels (forward and backward).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

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
constexpr int XT_BYTES = E * D * 2;  // 16-bit E x D tile
constexpr int AT_BYTES = D * D * 2;  // 16-bit D x D tile
// X~, A, G~ and Ps live in "stacked" tiles of 128 columns: logical column d is
// stored as its fp16 hi part at stacked column stk(d) = 32 * (d / 16) + d % 16 and
// its lo part 16 columns later (XLO bytes on), i.e. blocks of 16 hi columns
// alternate with blocks of 16 lo columns.  One M=128 x N=128 MMA over two stacked
// tiles (both MN-major) then yields every hi/lo product pair Zx^T Yy, with the hi
// row and the lo row of logical row i in lanes 32 * (i / 16) + i % 16 and that + 16.
constexpr int XC = 128;
constexpr uint32_t XLO = 256;
__host__ __device__ constexpr int stk(int d) { return ((d >> 4) << 5) | (d & 15); }
constexpr int TMEM_COLS = 512;  // two in-flight problems of 256 columns each
// TMEM column map of one in-flight Polar Express problem (256 columns):
constexpr uint32_t TM_GRAM = 0;   // Gram stack (128 cols); then A (16 cols per lane) for the A*A epilogue
constexpr uint32_t TM_X = 0;      // X~ B'^T: rows 0-127 in cols [0,64), rows 128-255 in [64,128) (after the Gram is read)
constexpr uint32_t TM_A2 = 128;   // A*A stack (128 cols)

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
// Dynamic work distribution of the persistent scan kernels: thread 0 of cluster rank 0
// takes the next item ticket and publishes it to both CTAs' `slot`; every thread of the
// cluster reads it after the cluster barrier.  Items are numbered so that an item's
// predecessor (the same chain's neighbouring chunk) has a smaller ticket, so it was taken
// by a cluster that is already running: a cluster that starts late, or never, cannot
// hold up the others.  The slot is rewritten only at the next call, after the item's
// own cluster barriers.
__device__ __forceinline__ long next_item(int* ticket, int* slot) {
  if (threadIdx.x == 0 && cluster_rank() == 0) {
    const int t = atomicAdd(ticket, 1);
    *slot = t;
    uint32_t la = smem_u32(slot), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(1));
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(ra), "r"(t) : "memory");
  }
  cluster_sync();
  return *(volatile int*)slot;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Operand split of every Polar Express product: a float32 value x is stored as two
// fp16 parts of y = KSPLIT * x, hi = fp16(y) and lo = fp16(y - hi), so hi + lo holds
// about 22 significant bits (fp16 has 11; the lo part's exponent keeps the residual
// exact down to the fp16 subnormal floor).  The power-of-two pre-scale keeps the
// small entries of the normalised iterates out of that floor.  Forward iterates are
// bounded by the Frobenius normalisation: |X| <= 1.2, |A| <= 1.5, |B'| < 64, so
// KSPLIT * |x| stays far below the fp16 maximum (65504).  A product of two split
// operands accumulates KSPLIT^2 times the true value; KUNSC2 undoes that.
// Compared with a bf16 split (8 + 8 bits) this is what lets B' = a I + b A + c A A
// carry the a X term: the split's representation error of X, amplified by a <= 8.2
// and by the five steps, was the tensor path's dominant error term.
constexpr float KSPLIT = 256.f;
constexpr float KUNSC2 = 1.f / 65536.f;

__device__ __forceinline__ uint64_t f32x2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f32x2_unpack(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
// Same arithmetic as scalar fmul / fsub (round to nearest), two lanes per instruction.
__device__ __forceinline__ uint64_t f32x2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// acc[0..3] += f * g (four lanes as two f32x2 FMAs; same rounding as fmaf)
__device__ __forceinline__ void fma4(float* acc, float f, float4 g) {
  const uint64_t ff = f32x2_pack(f, f);
  const float2 lo = f32x2_unpack(f32x2_fma(ff, f32x2_pack(g.x, g.y), f32x2_pack(acc[0], acc[1])));
  const float2 hi = f32x2_unpack(f32x2_fma(ff, f32x2_pack(g.z, g.w), f32x2_pack(acc[2], acc[3])));
  acc[0] = lo.x;
  acc[1] = lo.y;
  acc[2] = hi.x;
  acc[3] = hi.y;
}
// v[j] = a * v[j] + b * u[j] for n lanes (n even), as fmaf(a, v[j], b * u[j]) rounds
template <int n>
__device__ __forceinline__ void axpby(float* v, float a, const float* u, float b) {
  const uint64_t a2 = f32x2_pack(a, a), b2 = f32x2_pack(b, b);
#pragma unroll
  for (int j = 0; j < n; j += 2) {
    const uint64_t t = f32x2_mul(b2, f32x2_pack(u[j], u[j + 1]));
    const float2 r = f32x2_unpack(f32x2_fma(a2, f32x2_pack(v[j], v[j + 1]), t));
    v[j] = r.x;
    v[j + 1] = r.y;
  }
}
__device__ __forceinline__ uint64_t f32x2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Split 8 consecutive float32 values (times scale) into fp16 hi and lo parts and
// store them as one 16-byte core-matrix row segment in each tile.
__device__ __forceinline__ void store_split8(uint8_t* th, uint8_t* tl, uint32_t off, const float* v,
                                             float scale = KSPLIT) {
  uint32_t h[4], l[4];
  const uint64_t sc2 = f32x2_pack(scale, scale);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint64_t y = f32x2_mul(f32x2_pack(v[2 * k], v[2 * k + 1]), sc2);
    const float2 yf = f32x2_unpack(y);
    const __half2 hv = __floats2half2_rn(yf.x, yf.y);  // .x (low half) = y0
    const float2 hf = __half22float2(hv);
    const float2 lf = f32x2_unpack(f32x2_sub(y, f32x2_pack(hf.x, hf.y)));
    const __half2 lv = __floats2half2_rn(lf.x, lf.y);
    h[k] = *reinterpret_cast<const uint32_t*>(&hv);
    l[k] = *reinterpret_cast<const uint32_t*>(&lv);
  }
  *(uint4*)(th + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *(uint4*)(tl + off) = make_uint4(l[0], l[1], l[2], l[3]);
}
// 32 consecutive columns [c0, c0+32) of row r of a tile with C columns.
__device__ __forceinline__ void store_split32(uint8_t* th, uint8_t* tl, int r, int c0, int C, const float* v,
                                              float scale = KSPLIT) {
#pragma unroll
  for (int k = 0; k < 4; ++k) store_split8(th, tl, cm_off(r, c0 + 8 * k, C), v + 8 * k, scale);
}
// Logical columns [c0, c0+n) (c0 a multiple of 8) of row r of a stacked tile.
template <int n>
__device__ __forceinline__ void store_stk(uint8_t* t, int r, int c0, const float* v, float scale = KSPLIT) {
#pragma unroll
  for (int k = 0; k < n / 8; ++k) store_split8(t, t + XLO, cm_off(r, stk(c0 + 8 * k), XC), v + 8 * k, scale);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + 16, v + 16);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  tmem_st16(taddr, v);
  tmem_st16(taddr + 16, v + 16);
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Finishes one row of a stacked product whose 128 TMEM columns [64 ch, 64 ch + 64)
// the lane loaded into v (hi parts of logical columns 32ch..+15, their lo parts,
// then the same for 32ch+16..+31).  Lanes l < 16 hold the hi row i (Zh^T Yh | Zh^T Yl),
// lanes l >= 16 the lo row i (Zl^T Yh | Zl^T Yl).  Afterwards lane l < 16 holds
// columns 32ch..32ch+15 of  unscale * (Zh^T Yh + Zh^T Yl + Zl^T Yh + Zl^T Yl)  in
// r[0..15], lane l + 16 columns 32ch+16..32ch+31.
__device__ __forceinline__ void stack_finish(const float* v, float* r, float unscale = KUNSC2) {
  const bool hi = (threadIdx.x & 16) == 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float keep = hi ? v[j] + v[16 + j] : v[32 + j] + v[48 + j];
    const float send = hi ? v[32 + j] + v[48 + j] : v[j] + v[16 + j];
    r[j] = unscale * (keep + __shfl_xor_sync(0xffffffffu, send, 16));
  }
}
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + 16, v + 16);
  tmem_ld16(taddr + 32, v + 32);
  tmem_ld16(taddr + 48, v + 48);
}

// Momentum window term of one token (memory_layer.py:233-253, 543-560):
//   S[e][d] += wgt * sum_{i = i0..r} gamma_i F[i][e] G[i][d]
// for this thread's rows e0, e1 and columns dc..dc+31.  F (global; each row is
// re-read by the next Omega tokens, mostly from L1) is read eight window entries at
// a time so their loads overlap.
__device__ __forceinline__ void momentum_window(float (*Sv)[32], const float* F, const float* G, const float* gam,
                                                int i0, int r, float wgt, bool win, int e0, int e1, int dc) {
  for (int ib = i0; ib <= r; ib += 8) {
    float fa[8], fb[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = min(ib + k, r);
      const float c = ib + k <= r ? wgt * (win ? gam[i] : 1.f) : 0.f;
      fa[k] = c * F[i * E + e0];
      fb[k] = c * F[i * E + e1];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (ib + k > r) break;
      const float4* g4 = (const float4*)&G[(ib + k) * D + dc];
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 g = g4[j4];
        fma4(&Sv[0][4 * j4], fa[k], g);
        fma4(&Sv[1][4 * j4], fb[k], g);
      }
    }
  }
}

// Per-token E-vectors of a chunk that feed (token x d) products on CUDA cores (the
// frozen pass's act, the backward's d(W1^T err) and dh) are kept transposed, [e][i]
// with i the token of the chunk, so four consecutive tokens of one e are one 16-byte load.  The
// 16-byte groups of a row are XOR-swizzled by e so the row-per-thread writes spread
// over the banks.
__device__ __forceinline__ int tsw(int e, int i) { return e * MAXCS + ((((i >> 2) ^ (e & 15))) << 2) + (i & 3); }

// acc[u][v] = sum_e Wt[e][4dq + v] * V[e][4iq + u]  (Wt: E x D row-major in shared
// memory, V: tsw layout), the 4 x 4 (token x d) tile of one thread: thread (dq, iq) owns
// d = 4dq..4dq+3 and tokens i = 4iq..4iq+3.
__device__ __forceinline__ void tile_tok_d(const float* Wt, const float* V, int dq, int iq, float (*acc)[4]) {
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) acc[u][v] = 0.f;
#pragma unroll 4
  for (int e = 0; e < E; ++e) {
    const float4 wv = *(const float4*)&Wt[e * D + 4 * dq];
    const float4 av = *(const float4*)&V[tsw(e, 4 * iq)];
    const float wa[4] = {wv.x, wv.y, wv.z, wv.w}, aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(aa[u], wa[v], acc[u][v]);
  }
}

// Gv += c f_i g_i^T for this thread's rows e0, e1 and columns dc..dc+31.
__device__ __forceinline__ void rank1_add(float (*Gv)[32], const float* F, const float* G, int i, float c, int e0,
                                          int e1, int dc) {
  const float fa = c * F[i * E + e0], fb = c * F[i * E + e1];
  const float4* g4 = (const float4*)&G[i * D + dc];
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    const float4 g = g4[j4];
    fma4(&Gv[0][4 * j4], fa, g);
    fma4(&Gv[1][4 * j4], fb, g);
  }
}

// Omega-window sum of token r's per-token gradients, G_r = sum_{i in win(r)} c_i f_i g_i^T
// (c_i = gamma_i; window [max(0, r - omega + 1), r] of the chunk, or just r when the
// window is off; memory_layer.py:233-253).  The first token of a Polar Express pair
// builds it from the window; the second (slide) moves the previous token's sum on by
// one token: add token r, drop token r - omega if it was in the previous window.
__device__ __forceinline__ void window_sum(float (*Gv)[32], const float* F, const float* G, const float* gam, int r,
                                           int omega, bool win, bool slide, int e0, int e1, int dc) {
  if (!slide) {
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) Gv[0][jj] = Gv[1][jj] = 0.f;
    momentum_window(Gv, F, G, gam, win ? max(0, r - omega + 1) : r, r, 1.f, win, e0, e1, dc);
  } else {
    rank1_add(Gv, F, G, r, win ? gam[r] : 1.f, e0, e1, dc);
    const int io = r - (win ? omega : 1);
    if (io >= 0) rank1_add(Gv, F, G, io, -(win ? gam[io] : 1.f), e0, e1, dc);
  }
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

// Same, over the 8 epilogue warps only (kernels with a dedicated MMA warp).
__device__ __forceinline__ float block_sum_epi(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  asm volatile("bar.sync 1, 256;" ::: "memory");
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  asm volatile("bar.sync 1, 256;" ::: "memory");
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

// Three-term split product (fp16 parts) into TMEM column `tmd`:
//   D (+)= Ah*Bh + Ah*Bl + Al*Bh   (M x 64, contraction length K)
// ca / cb are the column counts of the A / B core-matrix tiles: 64 for plain
// tiles, XC for a stacked A tile (K-major only; al = ah + XLO).  amn / bmn pick the MN-major view (rows = K index)
// instead of the K-major view (rows = M/N).  a_off is a byte offset into the A
// tiles (selects the 128-row half for M = 128).  Descriptors are built once per
// term; stepping K by 16 adds to the 14-bit start-address field (shared-memory
// addresses < 256 KB never carry out of it).
template <int K, int NTERM = 3>
__device__ __forceinline__ void mma3(uint32_t tmd, const uint8_t* ah, const uint8_t* al, bool amn, int ca,
                                     const uint8_t* bh, const uint8_t* bl, bool bmn, int cb, int M, uint32_t a_off,
                                     bool accumulate) {
  const uint32_t id = idesc_f16(M, 64, amn, bmn);
  // K-major stacked tiles hold 16 hi columns per 32 stacked columns: 512 bytes per 16 of K
  const uint64_t sa = amn ? (uint64_t)(2 * 16 * ca) >> 4 : (ca == XC ? (512 >> 4) : (256 >> 4));
  const uint64_t sb = bmn ? (uint64_t)(2 * 16 * cb) >> 4 : (256 >> 4);
  const uint8_t* ta[4] = {ah, ah, al, al};
  const uint8_t* tb[4] = {bh, bl, bh, bl};
#pragma unroll
  for (int t = 0; t < NTERM; ++t) {
    const uint32_t aa = smem_u32(ta[t]) + a_off, bb = smem_u32(tb[t]);
    const uint64_t da = amn ? desc_mnmajor(aa, ca) : desc_kmajor(aa, ca);
    const uint64_t db = bmn ? desc_mnmajor(bb, cb) : desc_kmajor(bb, cb);
#pragma unroll
    for (int ks = 0; ks < K / 16; ++ks)
      mma_kf16(tmd, da + ks * sa, db + ks * sb, id, (accumulate || t || ks) ? 1u : 0u);
  }
}

// D (+)= Z^T Y over two stacked tiles (K x 64 logical, MN-major): one
// M=128 x N=128 MMA per 16 of K; see stack_finish for the result layout.
template <int K>
__device__ __forceinline__ void mma_stack(uint32_t tmd, const uint8_t* z, const uint8_t* y, bool accumulate) {
  const uint32_t id = idesc_f16(128, 128, true, true);
  const uint64_t dz = desc_mnmajor(smem_u32(z), XC), dy = desc_mnmajor(smem_u32(y), XC);
  constexpr uint64_t step = (uint64_t)(2 * 16 * XC) >> 4;
#pragma unroll
  for (int ks = 0; ks < K / 16; ++ks)
    mma_kf16(tmd, dz + ks * step, dy + ks * step, id, (accumulate || ks) ? 1u : 0u);
}

// Optional phase timers (build with -DATLAS_PHASE_PROF; thread 0 accumulates
// clock64() deltas into a shared array; off in the product build).
#ifdef ATLAS_PHASE_PROF
#define PROF_DECL __shared__ unsigned long long s_prof[32];
#define PROF_INIT if (threadIdx.x < 32) s_prof[threadIdx.x] = 0;
#define PROF_T(v) long long v = clock64();
#define PROF_ADD(slot, v) if (threadIdx.x == 0) s_prof[slot] += clock64() - v;
#define PROF_PTR s_prof
#define PROF_FLUSH(g) if (threadIdx.x < 32) atomicAdd(&g[threadIdx.x], s_prof[threadIdx.x]);
#else
#define PROF_DECL
#define PROF_INIT
#define PROF_T(v)
#define PROF_ADD(slot, v)
#define PROF_PTR nullptr
#define PROF_FLUSH(g)
#endif


}  // namespace tc
}  // namespace atlas

namespace atlas {
namespace tc {

// Host: upper bound on resident 2-CTA clusters (one CTA per SM).
inline int max_clusters_bound() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms / 2;
}

// One Polar Express problem in flight: its operand tiles, TMEM base column,
// completion barrier, and (optionally) where to save each step's operand tiles.
// X~ (E x 64) and A (64 x 64) are stacked tiles (Xl = Xh + XLO, Al = Ah + XLO);
// B' is two plain 64-column tiles (Bl = Bh + AT_BYTES).
struct PESlot {
  uint8_t *Xh, *Xl, *Ah, *Al, *Bh, *Bl;
  uint64_t* bar;
  uint32_t tm;       // TMEM base of this slot: X~ at +TM_X (+64), Gram at +TM_GRAM, A*A at +TM_A2
  uint32_t phase;
  uint8_t* ns;       // global destination of step k's tiles at ns + k * NS_TILE_BYTES, or null
  int save_last;     // unused (every step is saved when ns is set)
};
// Saved per step: stacked X~ (2 * XT_BYTES), stacked A (2 * AT_BYTES), B' hi, B' lo.
constexpr size_t NS_TILE_BYTES = 2 * XT_BYTES + 4 * AT_BYTES;

__device__ __forceinline__ void pe_issue(const PESlot& p, int type) {
  if (type == 0) {         // Gram stack: X~^T X~ over the hi/lo pairs
    mma_stack<E>(p.tm + TM_GRAM, p.Xh, p.Xh, false);
  } else if (type == 1) {  // A A = A^T A (A symmetric)
    mma_stack<D>(p.tm + TM_A2, p.Ah, p.Ah, false);
  } else {                 // X~ B'^T, two 128-row halves
    mma3<D>(p.tm + TM_X, p.Xh, p.Xl, false, XC, p.Bh, p.Bl, false, 64, 128, 0, false);
    mma3<D>(p.tm + TM_X + 64, p.Xh, p.Xl, false, XC, p.Bh, p.Bl, false, 64, 128, 16 * 16 * XC, false);
  }
}

}  // namespace tc
}  // namespace atlas

namespace atlas {
namespace tc {

// ---------------------------------------------------------------------------
// Producer / consumer form of the interleaved Polar Express (dedicated MMA warp).
// The 8 epilogue warps (consumers) and one MMA warp (producer) hand off through
// per-slot mbarriers: ready[s] (8 arrivals: one per epilogue warp after its tile
// stores) and done[s] (tcgen05.commit).  No CTA-wide barrier inside the loop.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// named barrier over the 8 epilogue warps only
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

struct PEBars {
  uint64_t* ready[2];
  uint64_t* done[2];
  uint32_t ready_phase[2];  // used by the producer
  uint32_t done_phase[2];   // used by the consumers
};

// Epilogue warp: publish this warp's tile stores of slot s to the producer.
__device__ __forceinline__ void pe_publish(PEBars& B, int s) {
  fence_async_smem();
  fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(B.ready[s]);
}

// Consumers (threads 0..255).  X0 of every slot is already stored by these threads.
// On return each slot's final X~ is in TMEM (tm + TM_X, + 64), KSPLIT^2 times its value.
//
// Gram and A*A come back as hi/lo stacks (see stack_finish): warp w reads the
// 64 columns of column half w / 4 of its lane quadrant, and each lane finishes 16
// entries (row rr, columns d0..d0+15) of the symmetric product with one shuffle
// per entry.  The lane writes its 16 entries of A back over its own TMEM lane for
// the A*A epilogue (B' = a I + b A + c A A), which uses the same lane/column map.
static __device__ __forceinline__ bool pe_consume(PESlot* sl, PEBars& B, int nslots, int steps, volatile int* bad,
                                                  unsigned long long* prof = nullptr) {
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, qd = w & 3, ch = w >> 2;
  const int dc = 32 * ch, e0 = 32 * qd + l, e1 = e0 + 128;
  const int rr = 16 * qd + (l & 15), d0 = dc + (l & 16);
  const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
  const int P = 3 * steps;
  bool ok = true;
#pragma unroll
  for (int s = 0; s < 2; ++s)
    if (s < nslots) pe_publish(B, s);
  for (int p = 0; p < P; ++p) {
    const int type = p % 3, st = p / 3;
#pragma unroll
    for (int s = 0; s < 2; ++s) {  // static slot index: sl[] and B stay in registers
      if (s >= nslots) break;
      PESlot& q = sl[s];
      long long tw = prof ? clock64() : 0;
      if (!*bad && !mbar_wait(B.done[s], B.done_phase[s])) ok = false;
      B.done_phase[s] ^= 1;
      fence_after();
      long long te = prof ? clock64() : 0;
      if (prof && threadIdx.x == 0) prof[11] += te - tw;
      if (type == 0) {
        float v[64], a[16];
        tmem_ld64(q.tm + lane_off + TM_GRAM + 2 * dc, v);
        tmem_wait_ld();
        stack_finish(v, a);  // A[rr][d0 + j]
        store_stk<16>(q.Ah, rr, d0, a);
        tmem_st16(q.tm + lane_off + TM_GRAM + 2 * dc, a);
        tmem_wait_st();
      } else if (type == 1) {
        const float ca = (float)kPE[st][0], cb = (float)kPE[st][1], cc = (float)kPE[st][2];
        float v[64], av[16], b2[16];
        tmem_ld64(q.tm + lane_off + TM_A2 + 2 * dc, v);
        tmem_ld16(q.tm + lane_off + TM_GRAM + 2 * dc, av);
        tmem_wait_ld();
        stack_finish(v, b2);  // (A A)[rr][d0 + j]
#pragma unroll
        for (int j = 0; j < 16; ++j) b2[j] = fmaf(cc, b2[j], cb * av[j]) + (rr == d0 + j ? ca : 0.f);
        store_split8(q.Bh, q.Bl, cm_off(rr, d0, D), b2);  // B'[rr][d0..d0+15]
        store_split8(q.Bh, q.Bl, cm_off(rr, d0 + 8, D), b2 + 8);
      } else if (st + 1 < steps) {
        float x0[32], x1[32];
        tmem_ld32(q.tm + lane_off + TM_X + dc, x0);
        tmem_ld32(q.tm + lane_off + TM_X + 64 + dc, x1);
        tmem_wait_ld();
        store_stk<32>(q.Xh, e0, dc, x0, KSPLIT * KUNSC2);
        store_stk<32>(q.Xh, e1, dc, x1, KSPLIT * KUNSC2);
      }
      if (p + 1 < P) pe_publish(B, s);
      if (prof && threadIdx.x == 0) prof[12] += clock64() - te;
#ifdef ATLAS_PHASE_PROF_EPI
      if (prof && threadIdx.x == 0) prof[7 + type] += clock64() - te;
#endif
    }
  }
  return ok;
}

// Producer (one whole warp).  Mirrors pe_consume's schedule; when q.ns is set it
// saves the tile just published (X_st before the Gram, A_st before A*A, B'_st
// before X~ B'^T) with one bulk copy (one bulk group) per slot and phase.  A saved
// tile is next rewritten by the epilogue that follows the commit two phases
// later (X_st by the X~ B'^T epilogue, A_st by the next Gram epilogue, B'_st by
// the next A*A epilogue).  By that commit the lead lane has issued exactly
// 2 * nslots newer groups, so waiting until at most 2 * nslots groups are still
// reading shared memory before every commit keeps each copy ahead of its
// overwrite with the most slack.
static __device__ __forceinline__ bool pe_produce(PESlot* sl, PEBars& B, int nslots, int steps, volatile int* bad) {
  const int P = 3 * steps;
  const bool lead = (threadIdx.x & 31) == 0;
  const uint64_t pol = l2_evict_first_policy();  // saved tiles are read once, much later
  bool ok = true;
  for (int p = 0; p < P; ++p) {
    const int type = p % 3, st = p / 3;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (s >= nslots) break;
      PESlot& q = sl[s];
      if (!*bad && !mbar_wait(B.ready[s], B.ready_phase[s])) ok = false;
      B.ready_phase[s] ^= 1;
      fence_after();
      if (q.ns && lead) {
        uint8_t* o = q.ns + (size_t)st * NS_TILE_BYTES;
        if (type == 0)
          bulk_s2g_hint(o, q.Xh, 2 * XT_BYTES, pol);
        else if (type == 1)
          bulk_s2g_hint(o + 2 * XT_BYTES, q.Ah, 2 * AT_BYTES, pol);
        else
          bulk_s2g_hint(o + 2 * XT_BYTES + 2 * AT_BYTES, q.Bh, 2 * AT_BYTES, pol);
        bulk_commit();
      }
      __syncwarp();
      if (!*bad) {
        pe_issue(q, type);
        if (q.ns && lead) {
          if (nslots == 2)
            asm volatile("cp.async.bulk.wait_group.read 4;" ::: "memory");
          else
            asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory");
        }
        __syncwarp();
        mma_commit(B.done[s]);
      }
    }
  }
  if (lead) bulk_wait0();
  __syncwarp();
  return ok;
}

}  // namespace tc
}  // namespace atlas
