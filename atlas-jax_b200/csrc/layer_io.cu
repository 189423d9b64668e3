// Fused prologue / epilogue of the Atlas memory layer around the scan
// (include/atlas_layer.h): ShortConv + rms_norm + polynomial features of q/k/v and
// the sigmoid gates (atlas_jax/memory_layer.py:606-633, 303-329, 211-216, 455-462),
// and the retrieve gate (720-722), forward and VJP.
//
// These are HBM-bound elementwise passes over the one concatenated projection
// (B*T, NP).  Mapping:
//   qkv   one warp per (token, which in {q,k,v}, head): the head's D channels sit
//         D/32 per lane, so the causal conv reads K coalesced rows and rms_norm is a
//         warp reduction, with no shared memory and no block barrier;
//   gates one thread per (token, gate column);
//   conv parameter gradients: one thread per channel over a tile of tokens (the
//         reduction over B*T stays in registers; one atomic per thread and tile).
// Grids are grid-stride loops sized to the SM count.
#include <algorithm>
#include <cstdio>

#include "atlas_layer.h"
#include "common.cuh"
#include "scan_internal.h"

namespace atlas {
namespace lio {

constexpr int MAXL = 8;  // ceil(D / 32) <= 8
constexpr int MAXK = 8;  // conv kernel size
constexpr int MAXP = 4;  // polynomial degree

struct Geo {
  int B, T, H, D, K, P, G, di, NP, has_gamma, has_ret;
  int ld;  // row stride of proj / dproj (elements)
  float max_lr;
};

inline Geo geo(const AtlasLayerParams& p) {
  Geo g;
  g.B = p.B, g.T = p.T, g.H = p.H, g.D = p.D, g.K = p.conv_kernel, g.P = p.poly_degree;
  g.has_gamma = p.has_gamma ? 1 : 0;
  g.has_ret = p.has_retrieve ? 1 : 0;
  g.G = 3 + g.has_gamma + g.has_ret;
  g.di = p.H * p.D;
  g.NP = 3 * g.di + g.G * p.H;
  g.ld = p.proj_stride > 0 ? p.proj_stride : g.NP;
  g.max_lr = p.max_lr;
  return g;
}

struct GatePtrs {
  float* p[5];  // alpha, eta, theta, gamma, retrieve (by column-group order below)
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

// phi(x) = sum_i a_i x^(i+1)  (memory_layer.py:455-462) and phi'(x)
__device__ __forceinline__ float poly_f(const float* a, int P, float x) {
  float r = 0.f, xp = x;
  for (int i = 0; i < P; ++i) {
    r = fmaf(a[i], xp, r);
    xp *= x;
  }
  return r;
}
__device__ __forceinline__ float poly_d(const float* a, int P, float x) {
  float r = 0.f, xp = 1.f;
  for (int i = 0; i < P; ++i) {
    r = fmaf(a[i] * (float)(i + 1), xp, r);
    xp *= x;
  }
  return r;
}

// Causal depthwise conv of channel c at token t of batch b (memory_layer.py:318-329):
//   out = bias[c] + sum_j w[j][c] * P[t - (K-1) + j][c]   (weights tap-major)
template <typename TA>
__device__ __forceinline__ float conv_at(const TA* proj, const float* w, const float* bias, const Geo& g, int b,
                                         int t, int col, int c) {
  float acc = bias[c];
  for (int j = 0; j < g.K; ++j) {
    const int ts = t - (g.K - 1) + j;
    if (ts >= 0) acc = fmaf(w[(size_t)j * g.di + c], ld_act(proj, ((size_t)b * g.T + ts) * g.ld + col), acc);
  }
  return acc;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <typename TA>
__global__ void __launch_bounds__(256) qkv_fwd_kernel(Geo g, const TA* proj, const float* conv_w,
                                                      const float* conv_b, const float* poly, TA* q, TA* k, TA* v) {
  __shared__ float pa[MAXP];
  if (threadIdx.x < g.P) pa[threadIdx.x] = poly[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31, L = (g.D + 31) / 32;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  const long items = (long)g.B * g.T * 3 * g.H;
  for (long it = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += nwarps) {
    const int h = (int)(it % g.H), wsel = (int)((it / g.H) % 3);
    const long n = it / (3 * g.H);
    const int b = (int)(n / g.T), t = (int)(n % g.T);
    const float* w = conv_w + (size_t)wsel * g.di * g.K;
    const float* bb = conv_b + (size_t)wsel * g.di;
    float x[MAXL];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L && lane + 32 * i < g.D) {
        const int c = h * g.D + lane + 32 * i;
        x[i] = conv_at(proj, w, bb, g, b, t, wsel * g.di + c, c);
      }
    TA* out = wsel == 0 ? q : (wsel == 1 ? k : v);
    if (wsel == 1 && g.P > 0) {  // k = rms_norm(phi(conv))
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) x[i] = poly_f(pa, g.P, x[i]);
    }
    if (wsel < 2) {  // rms_norm over the head (memory_layer.py:211-216)
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) ss = fmaf(x[i], x[i], ss);
      const float r = rsqrtf(warp_sum(ss) / g.D + 1e-6f);
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) x[i] *= r;
    }
    if (wsel == 0 && g.P > 0) {  // q = phi(rms_norm(conv))
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) x[i] = poly_f(pa, g.P, x[i]);
    }
    const size_t o = (((size_t)b * g.T + t) * g.H + h) * g.D;
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L && lane + 32 * i < g.D) st_act(out, o + lane + 32 * i, x[i]);
  }
}

// sigmoid gates (memory_layer.py:620-633, 720-722): one thread per (token, gate column)
template <typename TA>
__global__ void gates_fwd_kernel(Geo g, const TA* proj, const float* gate_bias, GatePtrs out) {
  const long items = (long)g.B * g.T * g.G * g.H;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (long)gridDim.x * blockDim.x) {
    const int col = (int)(i % (g.G * g.H)), gi = col / g.H, h = col % g.H;
    const long n = i / (g.G * g.H);
    const bool ret = g.has_ret && gi == g.G - 1;
    float z = ld_act(proj, (size_t)n * g.ld + 3 * g.di + col);
    if (!ret) z += gate_bias[col];
    float s = sigmoidf_(z);
    if (gi == 1) s *= g.max_lr;
    out.p[gi][(size_t)n * g.H + h] = s;
  }
}

template <typename TA>
__global__ void retrieve_fwd_kernel(Geo g, const TA* y, const float* r, TA* yg) {
  const long items = (long)g.B * g.T * g.H * g.D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (long)gridDim.x * blockDim.x)
    st_act(yg, i, ld_act(y, i) * r[i / g.D]);
}

// one warp per (token, head): dy = dyg * r, dr = sum_d dyg * y
template <typename TA>
__global__ void retrieve_bwd_kernel(Geo g, const TA* y, const float* r, const TA* dyg, TA* dy, float* dr) {
  const int lane = threadIdx.x & 31;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5), items = (long)g.B * g.T * g.H;
  for (long it = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += nwarps) {
    const float rv = r[it];
    float acc = 0.f;
    for (int d = lane; d < g.D; d += 32) {
      const size_t o = (size_t)it * g.D + d;
      const float gv = ld_act(dyg, o);
      acc = fmaf(gv, ld_act(y, o), acc);
      st_act(dy, o, gv * rv);
    }
    acc = warp_sum(acc);
    if (lane == 0) dr[it] = acc;
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
// Pass 1, one warp per (token, which, head): the cotangent dc of the conv output
// (float32, into the workspace) through rms_norm and the polynomial, and the
// polynomial coefficients' gradient (block partials in shared memory, one atomic
// per coefficient and block).
template <typename TA>
__global__ void __launch_bounds__(256) qkv_bwd1_kernel(Geo g, const TA* proj, const float* conv_w,
                                                       const float* conv_b, const float* poly, const TA* dq,
                                                       const TA* dk, const TA* dv, float* dc, float* dpoly) {
  __shared__ float pa[MAXP], pacc[MAXP];
  if (threadIdx.x < MAXP) {
    pa[threadIdx.x] = threadIdx.x < g.P ? poly[threadIdx.x] : 0.f;
    pacc[threadIdx.x] = 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, L = (g.D + 31) / 32;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  const long items = (long)g.B * g.T * 3 * g.H;
  float mypoly[MAXP] = {0.f, 0.f, 0.f, 0.f};
  for (long it = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += nwarps) {
    const int h = (int)(it % g.H), wsel = (int)((it / g.H) % 3);
    const long n = it / (3 * g.H);
    const int b = (int)(n / g.T), t = (int)(n % g.T);
    const float* w = conv_w + (size_t)wsel * g.di * g.K;
    const float* bb = conv_b + (size_t)wsel * g.di;
    const TA* dout = wsel == 0 ? dq : (wsel == 1 ? dk : dv);
    const size_t o = (((size_t)b * g.T + t) * g.H + h) * g.D;
    float c[MAXL], go[MAXL];
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L && lane + 32 * i < g.D) {
        const int ch = h * g.D + lane + 32 * i;
        c[i] = wsel < 2 ? conv_at(proj, w, bb, g, b, t, wsel * g.di + ch, ch) : 0.f;
        go[i] = dout ? ld_act(dout, o + lane + 32 * i) : 0.f;
      }
    if (wsel == 0) {  // out = phi(u), u = c r
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) ss = fmaf(c[i], c[i], ss);
      const float r = rsqrtf(warp_sum(ss) / g.D + 1e-6f);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) {
          if (g.P > 0) {
            const float u = c[i] * r;
            float xp = u;
            for (int j = 0; j < g.P; ++j) {
              mypoly[j] = fmaf(go[i], xp, mypoly[j]);
              xp *= u;
            }
            go[i] *= poly_d(pa, g.P, u);  // du
          }
          dot = fmaf(go[i], c[i], dot);
        }
      dot = warp_sum(dot);
      const float r3 = r * r * r / g.D;
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) go[i] = r * go[i] - r3 * c[i] * dot;
    } else if (wsel == 1) {  // out = rms(p), p = phi(c) (or p = c)
      float p[MAXL], ss = 0.f;
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) {
          p[i] = g.P > 0 ? poly_f(pa, g.P, c[i]) : c[i];
          ss = fmaf(p[i], p[i], ss);
        }
      const float r = rsqrtf(warp_sum(ss) / g.D + 1e-6f);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) dot = fmaf(go[i], p[i], dot);
      dot = warp_sum(dot);
      const float r3 = r * r * r / g.D;
#pragma unroll
      for (int i = 0; i < MAXL; ++i)
        if (i < L && lane + 32 * i < g.D) {
          float dp = r * go[i] - r3 * p[i] * dot;
          if (g.P > 0) {
            float xp = c[i];
            for (int j = 0; j < g.P; ++j) {
              mypoly[j] = fmaf(dp, xp, mypoly[j]);
              xp *= c[i];
            }
            dp *= poly_d(pa, g.P, c[i]);
          }
          go[i] = dp;
        }
    }
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L && lane + 32 * i < g.D) dc[(size_t)n * 3 * g.di + wsel * g.di + h * g.D + lane + 32 * i] = go[i];
  }
  if (g.P > 0) {
    for (int j = 0; j < g.P; ++j) {
      const float s = warp_sum(mypoly[j]);
      if (lane == 0) atomicAdd(&pacc[j], s);
    }
    __syncthreads();
    if (threadIdx.x < g.P) atomicAdd(&dpoly[threadIdx.x], pacc[threadIdx.x]);
  }
}

// Pass 2, one thread per channel column and a tile of TT tokens of one batch row:
//   dproj[t][c] = sum_j w[c][j] dc[t + K-1-j][c]   (the conv's transpose)
//   dw[c][j]   += sum_t dc[t][c] proj[t - (K-1) + j][c],  db[c] += sum_t dc[t][c]
constexpr int TT = 128;
template <typename TA>
__global__ void __launch_bounds__(256) qkv_bwd2_kernel(Geo g, const TA* proj, const float* conv_w, const float* dc,
                                                       TA* dproj, float* dconv_w, float* dconv_b) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;  // 0 .. 3 di
  if (col >= 3 * g.di) return;
  const int wsel = col / g.di, c = col % g.di;
  const int tiles = (g.T + TT - 1) / TT;
  const int b = blockIdx.y / tiles, t0 = (blockIdx.y % tiles) * TT, t1 = min(g.T, t0 + TT);
  float wv[MAXK], dw[MAXK];
#pragma unroll
  for (int j = 0; j < MAXK; ++j) {
    wv[j] = j < g.K ? conv_w[((size_t)wsel * g.K + j) * g.di + c] : 0.f;
    dw[j] = 0.f;
  }
  float db = 0.f;
  const size_t rowdc = (size_t)3 * g.di;
  for (int t = t0; t < t1; ++t) {
    const size_t n = (size_t)b * g.T + t;
    const float d = dc[n * rowdc + col];
    db += d;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < MAXK; ++j)
      if (j < g.K) {
        const int ts = t - (g.K - 1) + j;  // input token feeding output t through tap j
        if (ts >= 0) dw[j] = fmaf(d, ld_act(proj, ((size_t)b * g.T + ts) * g.ld + col), dw[j]);
        const int to = t + (g.K - 1) - j;  // output token that reads input t through tap j
        if (to < g.T) acc = fmaf(wv[j], dc[((size_t)b * g.T + to) * rowdc + col], acc);
      }
    st_act(dproj, n * g.ld + col, acc);
  }
#pragma unroll
  for (int j = 0; j < MAXK; ++j)
    if (j < g.K) atomicAdd(&dconv_w[((size_t)wsel * g.K + j) * g.di + c], dw[j]);
  atomicAdd(&dconv_b[col], db);
}

// gate VJP: dz = dgate * s (1 - s) (x max_lr for eta), into dproj; bias gradients
// reduced per block in shared memory (dynamic, G*H floats)
struct GateGrads {
  const float* p[5];
};
template <typename TA>
__global__ void gates_bwd_kernel(Geo g, const TA* proj, const float* gate_bias, GateGrads dg, TA* dproj,
                                 float* dbias) {
  extern __shared__ float sb[];
  const int GH = g.G * g.H;
  for (int i = threadIdx.x; i < GH; i += blockDim.x) sb[i] = 0.f;
  __syncthreads();
  const int ncol = g.ld - 3 * g.di;  // gate columns, then the row padding (written 0)
  const long items = (long)g.B * g.T * ncol;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (long)gridDim.x * blockDim.x) {
    const int col = (int)(i % ncol), gi = col / g.H, h = col % g.H;
    const long n = i / ncol;
    if (col >= GH) {
      st_act(dproj, (size_t)n * g.ld + 3 * g.di + col, 0.f);
      continue;
    }
    const bool ret = g.has_ret && gi == g.G - 1;
    float z = ld_act(proj, (size_t)n * g.ld + 3 * g.di + col);
    if (!ret) z += gate_bias[col];
    const float s = sigmoidf_(z);
    float d = dg.p[gi] ? dg.p[gi][(size_t)n * g.H + h] : 0.f;
    if (gi == 1) d *= g.max_lr;
    const float dz = d * s * (1.f - s);
    st_act(dproj, (size_t)n * g.ld + 3 * g.di + col, dz);
    if (!ret) atomicAdd(&sb[col], dz);
  }
  __syncthreads();
  const int nb = (g.G - g.has_ret) * g.H;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) atomicAdd(&dbias[i], sb[i]);
}


// ---------------------------------------------------------------------------
// 16-byte variants: one lane moves 8 consecutive channels, D / 8 lanes per head,
// 32 / (D / 8) heads per warp (used when D / 8 divides 32 and the rows of proj are
// 16-byte aligned)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ld8(const float* p, float* v) {
  const float4 a = *(const float4*)p, b = *(const float4*)(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *(const uint4*)p;
  const __nv_bfloat162* h = (const __nv_bfloat162*)&u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x, v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void st8(float* p, const float* v) {
  *(float4*)p = make_float4(v[0], v[1], v[2], v[3]);
  *(float4*)(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = (__nv_bfloat162*)&u;
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  *(uint4*)p = u;
}
// sum over the Lh lanes of one head (an aligned group of the warp)
__device__ __forceinline__ float group_sum(float v, int Lh) {
  for (int o = Lh >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct VecMap {
  int Lh, hpw, ngroups;
};
inline VecMap vec_map(const Geo& g) {
  VecMap m;
  m.Lh = g.D / 8;
  m.hpw = 32 / m.Lh;
  m.ngroups = (g.H + m.hpw - 1) / m.hpw;
  return m;
}
inline bool vec_ok(const Geo& g, int esize) {
  return g.D % 8 == 0 && g.D >= 8 && 32 % (g.D / 8) == 0 && ((size_t)g.ld * esize) % 16 == 0 &&
         ((size_t)g.di * esize) % 16 == 0;
}

// conv of channels c0..c0+7 (column col0 of proj) at token t of batch b
template <typename TA>
__device__ __forceinline__ void conv8(const TA* proj, const float* w, const float* bias, const Geo& g, int b, int t,
                                      int col0, int c0, float* x) {
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = bias[c0 + i];
  for (int j = 0; j < g.K; ++j) {
    const int ts = t - (g.K - 1) + j;
    if (ts < 0) continue;
    float pv[8];
    ld8(proj + ((size_t)b * g.T + ts) * g.ld + col0, pv);
    const float4 w0 = *(const float4*)(w + (size_t)j * g.di + c0), w1 = *(const float4*)(w + (size_t)j * g.di + c0 + 4);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = fmaf(wv[i], pv[i], x[i]);
  }
}

template <typename TA>
__global__ void __launch_bounds__(256) qkv_fwd_vec_kernel(Geo g, VecMap m, const TA* proj, const float* conv_w,
                                                          const float* conv_b, const float* poly, TA* q, TA* k,
                                                          TA* v) {
  __shared__ float pa[MAXP];
  if (threadIdx.x < MAXP) pa[threadIdx.x] = threadIdx.x < g.P ? poly[threadIdx.x] : 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31, hl = lane / m.Lh, part = lane % m.Lh;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  const long items = (long)g.B * g.T * 3 * m.ngroups;
  for (long it = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += nwarps) {
    const int hg = (int)(it % m.ngroups), wsel = (int)((it / m.ngroups) % 3);
    const long n = it / (3 * m.ngroups);
    const int b = (int)(n / g.T), t = (int)(n % g.T), h = hg * m.hpw + hl;
    const bool valid = h < g.H;
    const int c0 = h * g.D + 8 * part;
    float x[8];
    if (valid)
      conv8(proj, conv_w + (size_t)wsel * g.di * g.K, conv_b + (size_t)wsel * g.di, g, b, t, wsel * g.di + c0, c0, x);
    else
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = 0.f;
    if (wsel == 1 && g.P > 0)
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = poly_f(pa, g.P, x[i]);
    if (wsel < 2) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
      const float r = rsqrtf(group_sum(ss, m.Lh) / g.D + 1e-6f);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] *= r;
    }
    if (wsel == 0 && g.P > 0)
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = poly_f(pa, g.P, x[i]);
    if (valid) {
      TA* out = wsel == 0 ? q : (wsel == 1 ? k : v);
      st8(out + (((size_t)b * g.T + t) * g.H + h) * g.D + 8 * part, x);
    }
  }
}

template <typename TA>
__global__ void __launch_bounds__(256) qkv_bwd1_vec_kernel(Geo g, VecMap m, const TA* proj, const float* conv_w,
                                                           const float* conv_b, const float* poly, const TA* dq,
                                                           const TA* dk, const TA* dv, float* dc, float* dpoly) {
  __shared__ float pa[MAXP], pacc[MAXP];
  if (threadIdx.x < MAXP) {
    pa[threadIdx.x] = threadIdx.x < g.P ? poly[threadIdx.x] : 0.f;
    pacc[threadIdx.x] = 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, hl = lane / m.Lh, part = lane % m.Lh;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  const long items = (long)g.B * g.T * 3 * m.ngroups;
  float mypoly[MAXP] = {0.f, 0.f, 0.f, 0.f};
  for (long it = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += nwarps) {
    const int hg = (int)(it % m.ngroups), wsel = (int)((it / m.ngroups) % 3);
    const long n = it / (3 * m.ngroups);
    const int b = (int)(n / g.T), t = (int)(n % g.T), h = hg * m.hpw + hl;
    const bool valid = h < g.H;
    const int c0 = h * g.D + 8 * part;
    const TA* dout = wsel == 0 ? dq : (wsel == 1 ? dk : dv);
    float c[8], go[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = go[i] = 0.f;
    if (valid) {
      if (wsel < 2)
        conv8(proj, conv_w + (size_t)wsel * g.di * g.K, conv_b + (size_t)wsel * g.di, g, b, t, wsel * g.di + c0, c0,
              c);
      if (dout) ld8(dout + (((size_t)b * g.T + t) * g.H + h) * g.D + 8 * part, go);
    }
    if (wsel == 0) {  // out = phi(u), u = c r
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(c[i], c[i], ss);
      const float r = rsqrtf(group_sum(ss, m.Lh) / g.D + 1e-6f);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (g.P > 0) {
          const float u = c[i] * r;
          float xp = u;
          for (int j = 0; j < g.P; ++j) {
            mypoly[j] = fmaf(go[i], xp, mypoly[j]);
            xp *= u;
          }
          go[i] *= poly_d(pa, g.P, u);
        }
        dot = fmaf(go[i], c[i], dot);
      }
      dot = group_sum(dot, m.Lh);
      const float r3 = r * r * r / g.D;
#pragma unroll
      for (int i = 0; i < 8; ++i) go[i] = r * go[i] - r3 * c[i] * dot;
    } else if (wsel == 1) {  // out = rms(p), p = phi(c)
      float p[8], ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        p[i] = g.P > 0 ? poly_f(pa, g.P, c[i]) : c[i];
        ss = fmaf(p[i], p[i], ss);
      }
      const float r = rsqrtf(group_sum(ss, m.Lh) / g.D + 1e-6f);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) dot = fmaf(go[i], p[i], dot);
      dot = group_sum(dot, m.Lh);
      const float r3 = r * r * r / g.D;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float dp = r * go[i] - r3 * p[i] * dot;
        if (g.P > 0) {
          float xp = c[i];
          for (int j = 0; j < g.P; ++j) {
            mypoly[j] = fmaf(dp, xp, mypoly[j]);
            xp *= c[i];
          }
          dp *= poly_d(pa, g.P, c[i]);
        }
        go[i] = dp;
      }
    }
    if (valid) {
      float* o = dc + (size_t)n * 3 * g.di + wsel * g.di + c0;
      *(float4*)o = make_float4(go[0], go[1], go[2], go[3]);
      *(float4*)(o + 4) = make_float4(go[4], go[5], go[6], go[7]);
    }
  }
  if (g.P > 0) {
    for (int j = 0; j < g.P; ++j) {
      const float sm = warp_sum(mypoly[j]);
      if (lane == 0) atomicAdd(&pacc[j], sm);
    }
    __syncthreads();
    if (threadIdx.x < g.P) atomicAdd(&dpoly[threadIdx.x], pacc[threadIdx.x]);
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
static int warp_grid(long items) { return (int)std::max(1L, std::min((items + 7) / 8, 148L * 16)); }
static int elem_grid(long items) { return (int)std::max(1L, std::min((items + 255) / 256, 148L * 16)); }

static int check(const AtlasLayerParams* p) {
  if (!p) return report_error(ATLAS_ERR_INVALID_ARGUMENT, "params is NULL");
  if (p->abi_version != ATLAS_ABI_VERSION)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "abi_version mismatch");
  if (p->B <= 0 || p->T <= 0 || p->H <= 0 || p->D <= 0)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "B, T, H and D must be positive");
  if (p->D > 32 * MAXL) return report_error(ATLAS_ERR_UNSUPPORTED, "head_dim must be <= 256");
  if (p->conv_kernel < 1 || p->conv_kernel > MAXK)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "conv_kernel must be in 1..8");
  if (p->poly_degree < 0 || p->poly_degree > MAXP)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "poly_degree must be in 0..4");
  if (p->proj_stride != 0 && p->proj_stride < 3 * p->H * p->D + (3 + !!p->has_gamma + !!p->has_retrieve) * p->H)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "proj_stride is smaller than the projection's width");
  if (p->act_dtype != ATLAS_F32 && p->act_dtype != ATLAS_BF16)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "act_dtype must be ATLAS_F32 or ATLAS_BF16");
  clear_error();
  return ATLAS_OK;
}

static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return ATLAS_OK;
  return report_error(ATLAS_ERR_CUDA, cudaGetErrorString(e));
}

template <typename TA>
static cudaError_t prologue_fwd_t(const Geo& g, const void* proj, const float* cw, const float* cb, const float* poly,
                                  const float* gb, void* q, void* k, void* v, GatePtrs gp, cudaStream_t s) {
  if (vec_ok(g, sizeof(TA))) {
    const VecMap m = vec_map(g);
    qkv_fwd_vec_kernel<TA><<<warp_grid((long)g.B * g.T * 3 * m.ngroups), 256, 0, s>>>(
        g, m, (const TA*)proj, cw, cb, poly, (TA*)q, (TA*)k, (TA*)v);
  } else {
    const long witems = (long)g.B * g.T * 3 * g.H;
    qkv_fwd_kernel<TA><<<warp_grid(witems), 256, 0, s>>>(g, (const TA*)proj, cw, cb, poly, (TA*)q, (TA*)k, (TA*)v);
  }
  const long gitems = (long)g.B * g.T * g.G * g.H;
  gates_fwd_kernel<TA><<<elem_grid(gitems), 256, 0, s>>>(g, (const TA*)proj, gb, gp);
  return cudaGetLastError();
}

template <typename TA>
static cudaError_t prologue_bwd_t(const Geo& g, const void* proj, const float* cw, const float* cb, const float* poly,
                                  const float* gb, const void* dq, const void* dk, const void* dv, GateGrads dg,
                                  void* dproj, float* dcw, float* dcb, float* dpoly, float* dgb, float* dc,
                                  cudaStream_t s) {
  cudaError_t e;
  if ((e = cudaMemsetAsync(dcw, 0, (size_t)3 * g.di * g.K * sizeof(float), s)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(dcb, 0, (size_t)3 * g.di * sizeof(float), s)) != cudaSuccess) return e;
  if (g.P > 0 && (e = cudaMemsetAsync(dpoly, 0, (size_t)g.P * sizeof(float), s)) != cudaSuccess) return e;
  const int nb = (g.G - g.has_ret) * g.H;
  if ((e = cudaMemsetAsync(dgb, 0, (size_t)nb * sizeof(float), s)) != cudaSuccess) return e;
  if (vec_ok(g, sizeof(TA))) {
    const VecMap m = vec_map(g);
    qkv_bwd1_vec_kernel<TA><<<warp_grid((long)g.B * g.T * 3 * m.ngroups), 256, 0, s>>>(
        g, m, (const TA*)proj, cw, cb, poly, (const TA*)dq, (const TA*)dk, (const TA*)dv, dc, dpoly);
  } else {
    const long witems = (long)g.B * g.T * 3 * g.H;
    qkv_bwd1_kernel<TA><<<warp_grid(witems), 256, 0, s>>>(g, (const TA*)proj, cw, cb, poly, (const TA*)dq,
                                                           (const TA*)dk, (const TA*)dv, dc, dpoly);
  }
  const int tiles = (g.T + TT - 1) / TT;
  qkv_bwd2_kernel<TA><<<dim3((3 * g.di + 255) / 256, g.B * tiles), 256, 0, s>>>(g, (const TA*)proj, cw, dc,
                                                                                 (TA*)dproj, dcw, dcb);
  const long gitems = (long)g.B * g.T * g.G * g.H;
  gates_bwd_kernel<TA><<<elem_grid(gitems), 256, g.G * g.H * sizeof(float), s>>>(g, (const TA*)proj, gb, dg,
                                                                                  (TA*)dproj, dgb);
  return cudaGetLastError();
}

}  // namespace lio
}  // namespace atlas

using namespace atlas;
using namespace atlas::lio;

extern "C" size_t atlas_layer_prologue_workspace_bytes(const AtlasLayerParams* p) {
  if (check(p) != ATLAS_OK) return 0;
  const Geo g = geo(*p);
  return (size_t)g.B * g.T * 3 * g.di * sizeof(float);
}

extern "C" int atlas_layer_prologue_fwd(const AtlasLayerParams* p, const void* proj, const float* conv_w,
                                        const float* conv_b, const float* poly, const float* gate_bias, void* q,
                                        void* k, void* v, float* alpha, float* eta, float* theta, float* gamma,
                                        float* retrieve, void* stream) {
  int rc = check(p);
  if (rc) return rc;
  const Geo g = geo(*p);
  if (!proj || !conv_w || !conv_b || !gate_bias || !q || !k || !v || !alpha || !eta || !theta ||
      (g.P > 0 && !poly) || (g.has_gamma && !gamma) || (g.has_ret && !retrieve))
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  GatePtrs gp{{alpha, eta, theta, g.has_gamma ? gamma : retrieve, retrieve}};
  cudaStream_t s = (cudaStream_t)stream;
  return cuda_status(p->act_dtype == ATLAS_BF16
                         ? prologue_fwd_t<__nv_bfloat16>(g, proj, conv_w, conv_b, poly, gate_bias, q, k, v, gp, s)
                         : prologue_fwd_t<float>(g, proj, conv_w, conv_b, poly, gate_bias, q, k, v, gp, s));
}

extern "C" int atlas_layer_prologue_bwd(const AtlasLayerParams* p, const void* proj, const float* conv_w,
                                        const float* conv_b, const float* poly, const float* gate_bias,
                                        const void* dq, const void* dk, const void* dv, const float* dalpha,
                                        const float* deta, const float* dtheta, const float* dgamma,
                                        const float* dretrieve, void* dproj, float* dconv_w, float* dconv_b,
                                        float* dpoly, float* dgate_bias, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  int rc = check(p);
  if (rc) return rc;
  const Geo g = geo(*p);
  if (!proj || !conv_w || !conv_b || !gate_bias || !dproj || !dconv_w || !dconv_b || !dgate_bias ||
      (g.P > 0 && (!poly || !dpoly)))
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  const size_t need = (size_t)g.B * g.T * 3 * g.di * sizeof(float);
  if (!workspace || workspace_bytes < need)
    return report_error(ATLAS_ERR_WORKSPACE, "workspace smaller than atlas_layer_prologue_workspace_bytes()");
  GateGrads dg{{dalpha, deta, dtheta, g.has_gamma ? dgamma : dretrieve, dretrieve}};
  cudaStream_t s = (cudaStream_t)stream;
  float* dc = (float*)workspace;
  return cuda_status(p->act_dtype == ATLAS_BF16
                         ? prologue_bwd_t<__nv_bfloat16>(g, proj, conv_w, conv_b, poly, gate_bias, dq, dk, dv, dg,
                                                         dproj, dconv_w, dconv_b, dpoly, dgate_bias, dc, s)
                         : prologue_bwd_t<float>(g, proj, conv_w, conv_b, poly, gate_bias, dq, dk, dv, dg, dproj,
                                                 dconv_w, dconv_b, dpoly, dgate_bias, dc, s));
}

extern "C" int atlas_layer_retrieve_fwd(const AtlasLayerParams* p, const void* y, const float* retrieve, void* yg,
                                        void* stream) {
  int rc = check(p);
  if (rc) return rc;
  if (!y || !retrieve || !yg) return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  const Geo g = geo(*p);
  const long items = (long)g.B * g.T * g.H * g.D;
  cudaStream_t s = (cudaStream_t)stream;
  if (p->act_dtype == ATLAS_BF16)
    retrieve_fwd_kernel<__nv_bfloat16><<<elem_grid(items), 256, 0, s>>>(g, (const __nv_bfloat16*)y, retrieve,
                                                                         (__nv_bfloat16*)yg);
  else
    retrieve_fwd_kernel<float><<<elem_grid(items), 256, 0, s>>>(g, (const float*)y, retrieve, (float*)yg);
  return cuda_status(cudaGetLastError());
}

extern "C" int atlas_layer_retrieve_bwd(const AtlasLayerParams* p, const void* y, const float* retrieve,
                                        const void* dyg, void* dy, float* dretrieve, void* stream) {
  int rc = check(p);
  if (rc) return rc;
  if (!y || !retrieve || !dyg || !dy || !dretrieve)
    return report_error(ATLAS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  const Geo g = geo(*p);
  const long items = (long)g.B * g.T * g.H;
  cudaStream_t s = (cudaStream_t)stream;
  if (p->act_dtype == ATLAS_BF16)
    retrieve_bwd_kernel<__nv_bfloat16><<<warp_grid(items), 256, 0, s>>>(
        g, (const __nv_bfloat16*)y, retrieve, (const __nv_bfloat16*)dyg, (__nv_bfloat16*)dy, dretrieve);
  else
    retrieve_bwd_kernel<float><<<warp_grid(items), 256, 0, s>>>(g, (const float*)y, retrieve, (const float*)dyg,
                                                                 (float*)dy, dretrieve);
  return cuda_status(cudaGetLastError());
}
