// Shape-generic tensor-path forward scan: any head_dim D in {32, 64, 128, 256}, any
// memory width E (deep memory) and any chunk size, plus the linear-memory variant.
// It covers what the fused 2-CTA kernels (scan_tc.cu, D = 64, E = 256, chunk <= 64)
// do not: the long-context sweep's head_dim 128 and chunk 128, D == E, and the
// linear memory of atlas_jax/memory_layer.py:468-494.  Forward only.
//
// The chunk is processed token-parallel, the way the reference batches it
// (memory_layer.py:496-597): every token's momentum S_t is formed first, then the
// Polar Express of all of the chunk's matrices runs as ONE batched tensor-core call
// (atlas_polar_express_batched's tcgen05 GEMMs, pe_tc.cu), then the decayed memory
// recurrence and the read-out.  Per chunk, stream-ordered:
//   frozen_kernel   frozen-state pass on CUDA cores (memory_layer.py:504-520 / 471-477):
//                   the rank-1 factors F_t (rows) and G_t (columns) of each token's
//                   gradient, per matrix;
//   mom_kernel      one thread per matrix element: Omega window sum (233-253), momentum
//                   S_t = theta_t S_{t-1} - eta_t (2/D) sum (256-299), S_t -> PE input;
//   tcpe::launch    Polar Express of chains x chunk x matrices problems (43-71);
//   deep_w2_kernel  W2_t = alpha_t W2_{t-1} + O2_t and gelu(W2_t q_t), one warp per row;
//   deep_w1_kernel  W1_t scan and the read-out sum W1_t gelu(.) (592-595);
//   lin_out_kernel  linear memory: M_t scan and y_t = M_t q_t (490-492).
//
// State is kept in the workspace as E x D "tiles" per matrix: W1 and S_W1 transposed
// (W1^T), W2 and S_W2 as they are; linear memory M and S as they are (D x D).  In that
// orientation every per-token update is  tile[r][c] += coef * F_t[r] * G_t[c]:
//   W1^T: F = act (E), G = err (D);  W2: F = (W1^T err) * gelu'(h) (E), G = k (D);
//   M:    F = err (D), G = k (D);
// and Polar Express of a tile equals the tile-orientation of Polar Express of the
// matrix (PE(X^T) = PE(X)^T), so the deep tiles are PE'd as tall E x D matrices.
#include <algorithm>

#include "common.cuh"
#include "scan_internal.h"

namespace atlas {
namespace gen {

constexpr int NTH = 256;
constexpr int TB = 8;  // tokens per frozen_kernel CTA

struct Geo {
  int D, E, R, C, nm, cs, nch, chains;
  size_t RC;
};

__host__ __device__ inline Geo geo(const AtlasScanParams& p, int kind) {
  Geo g;
  g.D = p.D;
  g.E = kind == KIND_LINEAR ? p.D : p.E;
  g.R = g.E;
  g.C = p.D;
  g.nm = kind == KIND_LINEAR ? 1 : 2;
  g.cs = p.chunk;
  g.nch = n_chunks(p);
  g.chains = p.B * p.H;
  g.RC = (size_t)g.R * g.C;
  return g;
}

// workspace carve (floats unless noted)
struct WS {
  float *st;     // [chain][m][W, S][R x C]
  float *F, *G;  // [chain][m][t][R] and [chain][m][t][C]
  float *pin, *pout;  // [chain][t][m][R x C]
  float *gq;     // [chain][t][E]   gelu(W2_t q_t) (deep)
  float *yacc;   // [chain][t][D]   read-out sums (deep)
  void* pe_ws;
};

inline size_t al256(size_t b) { return (b + 255) & ~size_t(255); }

static WS carve(void* base, const Geo& g, size_t* total) {
  uint8_t* p = (uint8_t*)base;
  size_t off = 0;
  WS w;
  auto take = [&](size_t floats) {
    float* r = (float*)(p + off);
    off += al256(floats * sizeof(float));
    return r;
  };
  w.st = take((size_t)g.chains * g.nm * 2 * g.RC);
  w.F = take((size_t)g.chains * g.nm * g.cs * g.R);
  w.G = take((size_t)g.chains * g.nm * g.cs * g.C);
  w.pin = take((size_t)g.chains * g.cs * g.nm * g.RC);
  w.pout = take((size_t)g.chains * g.cs * g.nm * g.RC);
  w.gq = take((size_t)g.chains * g.cs * g.E);
  w.yacc = take((size_t)g.chains * g.cs * g.D);
  w.pe_ws = p + off;
  off += al256(tcpe::workspace_bytes((int64_t)g.chains * g.cs * g.nm, g.R, g.C));
  if (total) *total = off;
  return w;
}

// ---------------------------------------------------------------------------
// state in / out (tile orientation <-> the reference layout)
// ---------------------------------------------------------------------------
__global__ void state_in_kernel(Geo g, int kind, const float* W1, const float* W2, const float* S1,
                                const float* S2, float* st) {
  const size_t per = g.RC, total = (size_t)g.chains * g.nm * 2 * per;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t q = i / (g.nm * 2 * per);
    const int m = (int)((i / (2 * per)) % g.nm), ws = (int)((i / per) % 2);
    const size_t j = i % per;
    const int r = (int)(j / g.C), c = (int)(j % g.C);
    float v;
    if (kind == KIND_LINEAR) {  // M[v][k], S[v][k]
      const float* src = ws ? S1 : W1;
      v = src ? src[q * per + j] : 0.f;
    } else if (m == 0) {  // W1^T tile [e][d] from W1 (D x E)
      const float* src = ws ? S1 : W1;
      v = src ? src[q * per + (size_t)c * g.E + r] : 0.f;  // LM init: W1 = 0, S = 0
    } else {  // W2 (E x D)
      const float* src = ws ? S2 : W2;
      v = src ? src[q * per + j] : (ws == 0 && r == c ? 1.f : 0.f);  // LM init W2 = [I; 0]
    }
    st[i] = v;
  }
}

__global__ void state_out_kernel(Geo g, int kind, const float* st, float* W1, float* W2, float* S1, float* S2) {
  const size_t per = g.RC, total = (size_t)g.chains * g.nm * 2 * per;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t q = i / (g.nm * 2 * per);
    const int m = (int)((i / (2 * per)) % g.nm), ws = (int)((i / per) % 2);
    const size_t j = i % per;
    const int r = (int)(j / g.C), c = (int)(j % g.C);
    if (kind == KIND_LINEAR) {
      float* dst = ws ? S1 : W1;
      if (dst) dst[q * per + j] = st[i];
    } else if (m == 0) {
      float* dst = ws ? S1 : W1;
      if (dst) dst[q * per + (size_t)c * g.E + r] = st[i];
    } else {
      float* dst = ws ? S2 : W2;
      if (dst) dst[q * per + j] = st[i];
    }
  }
}

// ---------------------------------------------------------------------------
// frozen-state pass: rank-1 factors of every token's gradient (TB tokens per CTA)
// ---------------------------------------------------------------------------
template <typename TA>
__global__ void __launch_bounds__(NTH) frozen_kernel(FwdArgs a, Geo g, int kind, WS w, int c) {
  extern __shared__ float sm[];
  const AtlasScanParams& P = a.p;
  const int T = P.T, H = P.H, D = g.D, E = g.E, cs = g.cs;
  const int q = blockIdx.x, j0 = blockIdx.y * TB, tid = threadIdx.x;
  const int b = q / H, hh = q % H;
  float* kv = sm;             // [TB][D]
  float* vv = kv + TB * D;    // [TB][D]
  float* act = vv + TB * D;   // [TB][E]
  float* gp = act + TB * E;   // [TB][E]
  float* err = gp + TB * E;   // [TB][D]
  float* red = err + TB * D;  // [NTH / D][TB][D]
  for (int i = tid; i < TB * D; i += NTH) {
    const int j = i / D, d = i % D, t = c * cs + j0 + j;
    const bool ok = j0 + j < cs && t < T;
    const size_t o = (((size_t)b * T + t) * H + hh) * D + d;
    kv[i] = ok ? ld_act((const TA*)a.k, o) : 0.f;
    vv[i] = ok ? ld_act((const TA*)a.v, o) : 0.f;
  }
  __syncthreads();
  const float* st = w.st + (size_t)q * g.nm * 2 * g.RC;
  const int nj = min(TB, cs - j0);
  if (kind == KIND_LINEAR) {  // pred = M k, err = pred - v  (memory_layer.py:471-472)
    for (int v = tid; v < D; v += NTH) {
      float acc[TB];
#pragma unroll
      for (int j = 0; j < TB; ++j) acc[j] = 0.f;
      for (int k = 0; k < D; ++k) {
        const float m = st[(size_t)v * D + k];
#pragma unroll
        for (int j = 0; j < TB; ++j) acc[j] = fmaf(m, kv[j * D + k], acc[j]);
      }
      for (int j = 0; j < nj; ++j) {
        const size_t row = (size_t)q * cs + j0 + j;  // [chain][m = 0][t]
        w.F[row * D + v] = acc[j] - vv[j * D + v];
        w.G[row * D + v] = kv[j * D + v];
      }
    }
    return;
  }
  const float* W1t = st;               // E x D
  const float* W2 = st + 2 * g.RC;     // E x D
  // h = W2 k, act = gelu_tanh(h), gp = gelu'_erf(h)  (memory_layer.py:505-506, 517-518)
  for (int e = tid; e < E; e += NTH) {
    float acc[TB];
#pragma unroll
    for (int j = 0; j < TB; ++j) acc[j] = 0.f;
    for (int d = 0; d < D; ++d) {
      const float m = W2[(size_t)e * D + d];
#pragma unroll
      for (int j = 0; j < TB; ++j) acc[j] = fmaf(m, kv[j * D + d], acc[j]);
    }
#pragma unroll
    for (int j = 0; j < TB; ++j) {
      act[j * E + e] = gelu_tanh(acc[j]);
      gp[j * E + e] = gelu_erf_prime(acc[j]);
    }
  }
  __syncthreads();
  {  // err = k + W1 act - v  (507-508); NTH / D threads per column d split the E sum
    const int nsplit = NTH / D, d = tid % D, part = tid / D;
    float acc[TB];
#pragma unroll
    for (int j = 0; j < TB; ++j) acc[j] = 0.f;
    for (int e = part; e < E; e += nsplit) {
      const float m = W1t[(size_t)e * D + d];
#pragma unroll
      for (int j = 0; j < TB; ++j) acc[j] = fmaf(m, act[j * E + e], acc[j]);
    }
#pragma unroll
    for (int j = 0; j < TB; ++j) red[(part * TB + j) * D + d] = acc[j];
  }
  __syncthreads();
  for (int i = tid; i < TB * D; i += NTH) {
    const int j = i / D, d = i % D;
    float s = 0.f;
    for (int p2 = 0; p2 < NTH / D; ++p2) s += red[(p2 * TB + j) * D + d];
    err[i] = kv[i] - vv[i] + s;
  }
  __syncthreads();
  // chain = (W1^T err) * gelu'(h)  (516-519); write both matrices' factors
  for (int e = tid; e < E; e += NTH) {
    float acc[TB];
#pragma unroll
    for (int j = 0; j < TB; ++j) acc[j] = 0.f;
    for (int d = 0; d < D; ++d) {
      const float m = W1t[(size_t)e * D + d];
#pragma unroll
      for (int j = 0; j < TB; ++j) acc[j] = fmaf(m, err[j * D + d], acc[j]);
    }
    for (int j = 0; j < nj; ++j) {
      const size_t t0 = (size_t)j0 + j;
      w.F[(((size_t)q * 2 + 0) * cs + t0) * E + e] = act[j * E + e];
      w.F[(((size_t)q * 2 + 1) * cs + t0) * E + e] = acc[j] * gp[j * E + e];
    }
  }
  for (int i = tid; i < nj * D; i += NTH) {
    const int j = i / D, d = i % D;
    const size_t t0 = (size_t)j0 + j;
    w.G[(((size_t)q * 2 + 0) * cs + t0) * D + d] = err[j * D + d];
    w.G[(((size_t)q * 2 + 1) * cs + t0) * D + d] = kv[j * D + d];
  }
}

// ---------------------------------------------------------------------------
// momentum: one thread per tile element, every token of the chunk
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NTH) mom_kernel(FwdArgs a, Geo g, WS w, int c) {
  extern __shared__ float gs[];  // eta, theta, gamma of the chunk
  const AtlasScanParams& P = a.p;
  const int cs = g.cs, qm = blockIdx.y, q = qm / g.nm, m = qm % g.nm;
  const int b = q / P.H, hh = q % P.H;
  for (int t = threadIdx.x; t < cs; t += NTH) {
    const Gates G = load_gates(a.alpha, a.eta, a.theta, a.gamma, P.T, P.H, b, hh, c * cs + t);
    gs[t] = G.e;
    gs[cs + t] = G.t;
    gs[2 * cs + t] = G.g;
  }
  __syncthreads();
  const size_t idx = (size_t)blockIdx.x * NTH + threadIdx.x;
  if (idx >= g.RC) return;
  const int r = (int)(idx / g.C), cc = (int)(idx % g.C);
  float* Sp = w.st + ((size_t)q * g.nm + m) * 2 * g.RC + g.RC + idx;
  const float* __restrict__ F = w.F + ((size_t)q * g.nm + m) * cs * g.R + r;
  const float* __restrict__ Gc = w.G + ((size_t)q * g.nm + m) * cs * g.C + cc;
  float* __restrict__ out = w.pin + (size_t)m * g.RC + idx;
  const size_t ostride = (size_t)g.nm * g.RC, obase = (size_t)q * cs * ostride;
  const float s = 2.0f / g.D;
  const int om = P.omega;
  const bool win = om > 1;
  float S = *Sp;
  // G_t = sum_{i = t-om+1..t} gamma_i u_i (restarting at the chunk start), slid one token at
  // a time in float64 so the running sum does not drift over long chunks
  double acc = 0.0;
#pragma unroll 4
  for (int t = 0; t < cs; ++t) {
    const float u = __ldg(&F[(size_t)t * g.R]) * __ldg(&Gc[(size_t)t * g.C]);
    float gt;
    if (win) {
      acc = fma((double)gs[2 * cs + t], (double)u, acc);
      if (t >= om)
        acc = fma(-(double)gs[2 * cs + t - om],
                  (double)(__ldg(&F[(size_t)(t - om) * g.R]) * __ldg(&Gc[(size_t)(t - om) * g.C])), acc);
      gt = (float)acc;
    } else {
      gt = u;
    }
    S = fmaf(gs[cs + t], S, -gs[t] * s * gt);
    __stcs(&out[obase + (size_t)t * ostride], S);
  }
  *Sp = S;
}

// ---------------------------------------------------------------------------
// memory recurrence and read-out
// ---------------------------------------------------------------------------
constexpr int MAXL = 8;  // D / 32 <= 8

// W2_t = alpha_t W2_{t-1} + O2_t (memory_layer.py:583-584) and gq_t = gelu(W2_t q_t)
// (593-594); one warp per row e of the W2 tile, 8 rows per CTA.
template <typename TA>
__global__ void __launch_bounds__(NTH) deep_w2_kernel(FwdArgs a, Geo g, WS w, int c) {
  const AtlasScanParams& P = a.p;
  const int q = blockIdx.x, e = blockIdx.y * 8 + (threadIdx.x >> 5), l = threadIdx.x & 31;
  if (e >= g.E) return;
  const int b = q / P.H, hh = q % P.H, L = g.D / 32, cs = g.cs;
  float* Wr = w.st + ((size_t)q * 2 + 1) * 2 * g.RC + (size_t)e * g.D;
  float wv[MAXL];
#pragma unroll
  for (int i = 0; i < MAXL; ++i) wv[i] = i < L ? Wr[l + 32 * i] : 0.f;
  for (int t = 0; t < cs; ++t) {
    const int tok = c * cs + t;
    const bool ok = tok < P.T;
    const float al = ok ? a.alpha[((size_t)b * P.T + tok) * P.H + hh] : 1.f;
    const float* O = w.pout + (((size_t)q * cs + t) * 2 + 1) * g.RC + (size_t)e * g.D;
    const size_t qo = (((size_t)b * P.T + tok) * P.H + hh) * g.D;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L) {
        wv[i] = fmaf(al, wv[i], O[l + 32 * i]);
        if (ok) dot = fmaf(wv[i], ld_act((const TA*)a.q, qo + l + 32 * i), dot);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (l == 0) w.gq[((size_t)q * cs + t) * g.E + e] = gelu_tanh(dot);
  }
#pragma unroll
  for (int i = 0; i < MAXL; ++i)
    if (i < L) Wr[l + 32 * i] = wv[i];
}

// W1_t scan (tile W1^T, one warp per row e, 16 rows per CTA) and the read-out sum
// sum_e W1_t[d][e] gq_t[e]: the 16 warps' terms are reduced in shared memory, then one
// atomic add per (token, d) and CTA into the chunk's read-out accumulator.
__global__ void __launch_bounds__(512) deep_w1_kernel(FwdArgs a, Geo g, WS w, int c) {
  extern __shared__ float red[];  // [16][D]
  const AtlasScanParams& P = a.p;
  const int q = blockIdx.x, wp = threadIdx.x >> 5, e = blockIdx.y * 16 + wp, l = threadIdx.x & 31;
  const bool row = e < g.E;
  const int b = q / P.H, hh = q % P.H, L = g.D / 32, cs = g.cs;
  float* Wr = w.st + (size_t)q * 2 * 2 * g.RC + (size_t)(row ? e : 0) * g.D;
  float wv[MAXL];
#pragma unroll
  for (int i = 0; i < MAXL; ++i) wv[i] = row && i < L ? Wr[l + 32 * i] : 0.f;
  for (int t = 0; t < cs; ++t) {
    const int tok = c * cs + t;
    const float al = tok < P.T ? a.alpha[((size_t)b * P.T + tok) * P.H + hh] : 1.f;
    const float* O = w.pout + ((size_t)q * cs + t) * 2 * g.RC + (size_t)(row ? e : 0) * g.D;
    const float gv = row ? w.gq[((size_t)q * cs + t) * g.E + e] : 0.f;
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L) {
        if (row) wv[i] = fmaf(al, wv[i], O[l + 32 * i]);
        red[wp * g.D + l + 32 * i] = wv[i] * gv;
      }
    __syncthreads();
    for (int d = threadIdx.x; d < g.D; d += 512) {
      float s = 0.f;
#pragma unroll 4
      for (int k = 0; k < 16; ++k) s += red[k * g.D + d];
      atomicAdd(&w.yacc[((size_t)q * cs + t) * g.D + d], s);
    }
    __syncthreads();
  }
  if (row)
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L) Wr[l + 32 * i] = wv[i];
}

// y = q + read-out sum (deep memory), cropped to T (memory_layer.py:595, 718)
template <typename TA>
__global__ void deep_y_kernel(FwdArgs a, Geo g, WS w, int c) {
  const AtlasScanParams& P = a.p;
  const size_t total = (size_t)g.chains * g.cs * g.D;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % g.D), t = (int)((i / g.D) % g.cs), q = (int)(i / ((size_t)g.D * g.cs));
    const int tok = c * g.cs + t;
    if (tok >= P.T) continue;
    const int b = q / P.H, hh = q % P.H;
    const size_t o = (((size_t)b * P.T + tok) * P.H + hh) * g.D + d;
    st_act((TA*)a.y, o, ld_act((const TA*)a.q, o) + w.yacc[i]);
  }
}

// Linear memory: M_t = alpha_t M_{t-1} + O_t and y_t = M_t q_t (memory_layer.py:489-492),
// one warp per row v.
template <typename TA>
__global__ void __launch_bounds__(NTH) lin_out_kernel(FwdArgs a, Geo g, WS w, int c) {
  const AtlasScanParams& P = a.p;
  const int q = blockIdx.x, v = blockIdx.y * 8 + (threadIdx.x >> 5), l = threadIdx.x & 31;
  if (v >= g.D) return;
  const int b = q / P.H, hh = q % P.H, L = g.D / 32, cs = g.cs;
  float* Wr = w.st + (size_t)q * 2 * g.RC + (size_t)v * g.D;
  float wv[MAXL];
#pragma unroll
  for (int i = 0; i < MAXL; ++i) wv[i] = i < L ? Wr[l + 32 * i] : 0.f;
  for (int t = 0; t < cs; ++t) {
    const int tok = c * cs + t;
    const bool ok = tok < P.T;
    const float al = ok ? a.alpha[((size_t)b * P.T + tok) * P.H + hh] : 1.f;
    const float* O = w.pout + ((size_t)q * cs + t) * g.RC + (size_t)v * g.D;
    const size_t qo = (((size_t)b * P.T + tok) * P.H + hh) * g.D;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < MAXL; ++i)
      if (i < L) {
        wv[i] = fmaf(al, wv[i], O[l + 32 * i]);
        if (ok) dot = fmaf(wv[i], ld_act((const TA*)a.q, qo + l + 32 * i), dot);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (l == 0 && ok) st_act((TA*)a.y, qo + v, dot);
  }
#pragma unroll
  for (int i = 0; i < MAXL; ++i)
    if (i < L) Wr[l + 32 * i] = wv[i];
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
static int grid_for(size_t n) { return (int)std::min<size_t>((n + 255) / 256, 148 * 16); }

template <typename TA>
static cudaError_t launch_t(const FwdArgs& a, int kind, cudaStream_t s) {
  const Geo g = geo(a.p, kind);
  const WS w = carve(a.ws, g, nullptr);
  cudaError_t e;
  const size_t nst = (size_t)g.chains * g.nm * 2 * g.RC;
  state_in_kernel<<<grid_for(nst), 256, 0, s>>>(g, kind, a.W1_in, a.W2_in, a.S1_in, a.S2_in, w.st);
  const size_t fsm = (size_t)(3 * TB * g.D + 2 * TB * g.E + NTH * TB) * sizeof(float);
  if ((e = cudaFuncSetAttribute(frozen_kernel<TA>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsm)) !=
      cudaSuccess)
    return e;
  const size_t msm = (size_t)3 * g.cs * sizeof(float);
  if ((e = cudaFuncSetAttribute(mom_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msm)) !=
      cudaSuccess)
    return e;
  const int64_t npe = (int64_t)g.chains * g.cs * g.nm;
  for (int c = 0; c < g.nch; ++c) {
    frozen_kernel<TA><<<dim3(g.chains, (g.cs + TB - 1) / TB), NTH, fsm, s>>>(a, g, kind, w, c);
    mom_kernel<<<dim3((unsigned)((g.RC + NTH - 1) / NTH), g.chains * g.nm), NTH, msm, s>>>(a, g, w, c);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = tcpe::launch(w.pin, w.pout, npe, g.R, g.C, a.p.ns_steps, 1e-12f, w.pe_ws, s)) != cudaSuccess)
      return e;
    if (kind == KIND_LINEAR) {
      lin_out_kernel<TA><<<dim3(g.chains, (g.D + 7) / 8), NTH, 0, s>>>(a, g, w, c);
    } else {
      if ((e = cudaMemsetAsync(w.yacc, 0, (size_t)g.chains * g.cs * g.D * sizeof(float), s)) != cudaSuccess)
        return e;
      deep_w2_kernel<TA><<<dim3(g.chains, (g.E + 7) / 8), NTH, 0, s>>>(a, g, w, c);
      deep_w1_kernel<<<dim3(g.chains, (g.E + 15) / 16), 512, 16 * g.D * sizeof(float), s>>>(a, g, w, c);
      deep_y_kernel<TA><<<grid_for((size_t)g.chains * g.cs * g.D), 256, 0, s>>>(a, g, w, c);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  state_out_kernel<<<grid_for(nst), 256, 0, s>>>(g, kind, w.st, a.W1_out, a.W2_out, a.S1_out, a.S2_out);
  return cudaGetLastError();
}

bool supported(const AtlasScanParams& p, int kind, const char** why) {
  if (p.D % 32 != 0 || p.D > 256 || 256 % p.D != 0) {
    *why = "head_dim must be 32, 64, 128 or 256";
    return false;
  }
  if (kind == KIND_DEEP && (p.E < 1 || p.E > 2048)) {
    *why = "memory width E must be in 1..2048";
    return false;
  }
  if (p.chunk > 4096) {
    *why = "chunk must be <= 4096";
    return false;
  }
  return true;
}

size_t workspace_bytes(const AtlasScanParams& p, int kind) {
  size_t total = 0;
  carve(nullptr, geo(p, kind), &total);
  return total;
}

cudaError_t launch_fwd(const FwdArgs& a, int kind, cudaStream_t s) {
  return a.p.act_dtype == ATLAS_BF16 ? launch_t<__nv_bfloat16>(a, kind, s) : launch_t<float>(a, kind, s);
}

}  // namespace gen
}  // namespace atlas
