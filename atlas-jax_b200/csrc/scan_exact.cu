// Exact (float64 CUDA-core) Atlas scan: forward, backward and batched Polar
// Express.  One CTA per (b, h) pair walks the sequence token by token with the
// carry in a per-CTA float64 workspace.  It is the parity path: its rounding
// sits far below the reference's own float32 noise, so it reproduces the
// mathematics of atlas_jax/memory_layer.py:496-718 to ~1e-7 after the float32
// cast.  Speed is not its job (the tcgen05 path is the production path).
//
// Storage: both memory matrices are kept "wide" (D x E).  W1 and S1 are stored
// as is; W2 and S2 (E x D, tall) are stored transposed.  Polar Express of a
// tall matrix equals the transpose of Polar Express of its transpose
// (memory_layer.py:60-69: X^T X / X B on the tall side is X X^T / B X on the
// wide side), so one wide routine serves both.
#include "common.cuh"
#include "scan_internal.h"

namespace atlas {
namespace exact {

constexpr int kThreads = 256;

__device__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double s = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
  __syncthreads();
  return s;
}

// C[i,j] = alpha * sum_k opA(i,k) opB(k,j) + beta * C[i,j]   (row-major, C not aliased)
__device__ void gemm(double* C, int ldc, const double* A, int lda, bool ta, const double* B, int ldb,
                     bool tb, int M, int N, int K, double alpha, double beta) {
  for (int idx = threadIdx.x; idx < M * N; idx += blockDim.x) {
    int i = idx / N, j = idx % N;
    double s = 0;
    for (int k = 0; k < K; ++k) {
      double a = ta ? A[(size_t)k * lda + i] : A[(size_t)i * lda + k];
      double b = tb ? B[(size_t)j * ldb + k] : B[(size_t)k * ldb + j];
      s += a * b;
    }
    C[(size_t)i * ldc + j] = alpha * s + (beta == 0.0 ? 0.0 : beta * C[(size_t)i * ldc + j]);
  }
  __syncthreads();
}

// Workspace for one wide Polar Express on a D x E matrix.
struct PEWork {
  double *X, *Xn, *A, *AA, *Bm;
};

// Y = PE(S) (wide, D x E).  If hist != nullptr the per-step X, A, B are kept
// (hist layout per step: X (D*E), A (D*D), B (D*D)) for the VJP.  Returns the
// Frobenius norm n (memory_layer.py:55).
__device__ double pe_forward(const double* S, double* Y, int D, int E, int steps, double eps_sqrt, PEWork w,
                             double* hist, double* red) {
  const int DE = D * E;
  double ss = 0;
  for (int i = threadIdx.x; i < DE; i += blockDim.x) ss += S[i] * S[i];
  ss = block_sum(ss, red);
  double n = sqrt(ss + eps_sqrt);
  double kappa = n * 1.01 + 1e-6;
  double* X = w.X;
  for (int i = threadIdx.x; i < DE; i += blockDim.x) X[i] = S[i] / kappa;
  __syncthreads();
  for (int st = 0; st < steps; ++st) {
    double a = kPE[st][0], b = kPE[st][1], c = kPE[st][2];
    gemm(w.A, D, X, E, false, X, E, true, D, D, E, 1.0, 0.0);        // A = X X^T
    gemm(w.AA, D, w.A, D, false, w.A, D, false, D, D, D, 1.0, 0.0);  // A A
    for (int i = threadIdx.x; i < D * D; i += blockDim.x) w.Bm[i] = b * w.A[i] + c * w.AA[i];
    __syncthreads();
    if (hist) {
      double* h = hist + (size_t)st * (DE + 2 * D * D);
      for (int i = threadIdx.x; i < DE; i += blockDim.x) h[i] = X[i];
      for (int i = threadIdx.x; i < D * D; i += blockDim.x) {
        h[DE + i] = w.A[i];
        h[DE + D * D + i] = w.Bm[i];
      }
    }
    double* out = (st == steps - 1) ? Y : w.Xn;
    for (int i = threadIdx.x; i < DE; i += blockDim.x) out[i] = a * X[i];
    __syncthreads();
    gemm(out, E, w.Bm, D, false, X, E, false, D, E, D, 1.0, 1.0);    // X' = a X + B X
    if (st != steps - 1) {
      double* t = X;
      X = w.Xn;
      w.Xn = t;
    }
  }
  if (steps == 0) {
    for (int i = threadIdx.x; i < DE; i += blockDim.x) Y[i] = X[i];
    __syncthreads();
  }
  return n;
}

struct VJPWork {
  double *G, *dX, *dB, *dA, *T;
};

// dS (+)= PE_vjp(S, dO); hist from pe_forward.  accumulate: dS += result.
__device__ void pe_vjp(const double* S, const double* dO, double* dS, int D, int E, int steps, double n,
                       const double* hist, VJPWork w, double* red) {
  const int DE = D * E;
  const int DD = D * D;
  double* G = w.G;
  for (int i = threadIdx.x; i < DE; i += blockDim.x) G[i] = dO[i];
  __syncthreads();
  for (int st = steps - 1; st >= 0; --st) {
    double a = kPE[st][0], b = kPE[st][1], c = kPE[st][2];
    const double* X = hist + (size_t)st * (DE + 2 * DD);
    const double* A = X + DE;
    const double* Bm = A + DD;
    // dX = a G + B^T G
    for (int i = threadIdx.x; i < DE; i += blockDim.x) w.dX[i] = a * G[i];
    __syncthreads();
    gemm(w.dX, E, Bm, D, true, G, E, false, D, E, D, 1.0, 1.0);
    // dB = G X^T
    gemm(w.dB, D, G, E, false, X, E, true, D, D, E, 1.0, 0.0);
    // dA = b dB + c (dB A^T + A^T dB)
    gemm(w.dA, D, w.dB, D, false, A, D, true, D, D, D, c, 0.0);
    gemm(w.T, D, A, D, true, w.dB, D, false, D, D, D, c, 0.0);
    for (int i = threadIdx.x; i < DD; i += blockDim.x) w.dA[i] += w.T[i] + b * w.dB[i];
    __syncthreads();
    // T = dA + dA^T ; dX += T X
    for (int i = threadIdx.x; i < DD; i += blockDim.x) {
      int r = i / D, cc = i % D;
      w.T[i] = w.dA[i] + w.dA[cc * D + r];
    }
    __syncthreads();
    gemm(w.dX, E, w.T, D, false, X, E, false, D, E, D, 1.0, 1.0);
    double* t = G;
    G = w.dX;
    w.dX = t;
  }
  double kappa = n * 1.01 + 1e-6;
  double dot = 0;
  for (int i = threadIdx.x; i < DE; i += blockDim.x) dot += G[i] * S[i];
  dot = block_sum(dot, red);
  double coef = dot / (kappa * kappa) * 1.01 / n;
  for (int i = threadIdx.x; i < DE; i += blockDim.x) dS[i] += G[i] / kappa - coef * S[i];
  __syncthreads();
}

}  // namespace exact
}  // namespace atlas

namespace atlas {
namespace exact {

template <typename T> __device__ __forceinline__ const T* cptr(const void* p) { return (const T*)p; }

// Per-CTA float64 workspace of the forward.
struct FwdWS {
  double *W1, *W2, *S1, *S2, *O;
  PEWork pe;
  double *h, *act, *chain, *err, *kd, *z, *p, *red;
};

__host__ __device__ inline size_t fwd_ws_doubles(int D, int E, int cs) {
  size_t DE = (size_t)D * E;
  return 7 * DE + 3 * (size_t)D * D + 3 * (size_t)cs * E + 2 * (size_t)cs * D + 2 * (size_t)E + 32;
}

__device__ FwdWS carve_fwd(double* base, int D, int E, int cs) {
  size_t DE = (size_t)D * E;
  FwdWS w;
  double* p = base;
  w.W1 = p; p += DE;
  w.W2 = p; p += DE;
  w.S1 = p; p += DE;
  w.S2 = p; p += DE;
  w.O = p; p += DE;
  w.pe.X = p; p += DE;
  w.pe.Xn = p; p += DE;
  w.pe.A = p; p += D * D;
  w.pe.AA = p; p += D * D;
  w.pe.Bm = p; p += D * D;
  w.h = p; p += (size_t)cs * E;
  w.act = p; p += (size_t)cs * E;
  w.chain = p; p += (size_t)cs * E;
  w.err = p; p += (size_t)cs * D;
  w.kd = p; p += (size_t)cs * D;
  w.z = p; p += E;
  w.p = p; p += E;
  w.red = p;
  return w;
}

// Load the carry (wide storage) from the caller's float32 state or the LM init.
__device__ void load_state(const float* W1, const float* W2, const float* S1, const float* S2, size_t bh,
                           int D, int E, double* dW1, double* dW2, double* dS1, double* dS2) {
  size_t DE = (size_t)D * E;
  for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
    int d = (int)(i / E), e = (int)(i % E);
    size_t tall = bh * DE + (size_t)e * D + d;  // (E, D) element [e][d]
    dW1[i] = W1 ? (double)W1[bh * DE + i] : 0.0;
    dW2[i] = W2 ? (double)W2[tall] : (d == e ? 1.0 : 0.0);  // model.py:251-264: W2 = [I; 0]
    dS1[i] = S1 ? (double)S1[bh * DE + i] : 0.0;
    dS2[i] = S2 ? (double)S2[tall] : 0.0;
  }
  __syncthreads();
}

__device__ void store_state(float* W1, float* W2, float* S1, float* S2, size_t bh, int D, int E,
                            const double* dW1, const double* dW2, const double* dS1, const double* dS2) {
  size_t DE = (size_t)D * E;
  for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
    int d = (int)(i / E), e = (int)(i % E);
    size_t tall = bh * DE + (size_t)e * D + d;
    if (W1) W1[bh * DE + i] = (float)dW1[i];
    if (W2) W2[tall] = (float)dW2[i];
    if (S1) S1[bh * DE + i] = (float)dS1[i];
    if (S2) S2[tall] = (float)dS2[i];
  }
}

// Frozen-state pass over one chunk's keys (memory_layer.py:504-520):
// h = W2 k, act = gelu_tanh(h), err = k + W1 act - v, chain = (W1^T err) * gelu'(h).
template <typename TA>
__device__ void frozen_forward(const FwdArgs& a, int b, int hh, int c, const double* W1, const double* W2t,
                               double* h, double* act, double* err, double* chain, double* kd) {
  const AtlasScanParams& P = a.p;
  const int D = P.D, E = P.E, cs = P.chunk, T = P.T, H = P.H;
  const TA* k = cptr<TA>(a.k);
  const TA* v = cptr<TA>(a.v);
  for (int i = threadIdx.x; i < cs * D; i += blockDim.x) {
    int t = c * cs + i / D, d = i % D;
    kd[i] = t < T ? (double)ld_act(k, (((size_t)b * T + t) * H + hh) * D + d) : 0.0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < cs * E; i += blockDim.x) {
    int r = i / E, e = i % E;
    double s = 0;
    for (int d = 0; d < D; ++d) s += W2t[(size_t)d * E + e] * kd[r * D + d];
    h[i] = s;
    act[i] = gelu_tanh(s);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < cs * D; i += blockDim.x) {
    int r = i / D, d = i % D;
    int t = c * cs + r;
    double s = kd[i];
    for (int e = 0; e < E; ++e) s += W1[(size_t)d * E + e] * act[r * E + e];
    double vv = t < T ? (double)ld_act(v, (((size_t)b * T + t) * H + hh) * D + d) : 0.0;
    err[i] = s - vv;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < cs * E; i += blockDim.x) {
    int r = i / E, e = i % E;
    double s = 0;
    for (int d = 0; d < D; ++d) s += W1[(size_t)d * E + e] * err[r * D + d];
    chain[i] = s * gelu_erf_prime(h[i]);
  }
  __syncthreads();
}

// S <- theta S - eta * sum_{i in window(t)} w_i * s * f_i g_i^T  for both matrices
// (memory_layer.py:522-533 + linear_scan 256-299 for one token).
__device__ void momentum_step(const FwdArgs& a, int b, int hh, int c, int r, double* S1, double* S2t,
                              const double* err, const double* act, const double* chain, const double* kd,
                              double theta, double eta) {
  const AtlasScanParams& P = a.p;
  const int D = P.D, E = P.E;
  const double s = 2.0 / D;
  int i0 = P.omega > 1 ? max(0, r - P.omega + 1) : r;
  for (size_t idx = threadIdx.x; idx < (size_t)D * E; idx += blockDim.x) {
    int d = (int)(idx / E), e = (int)(idx % E);
    double g1 = 0, g2 = 0;
    for (int i = i0; i <= r; ++i) {
      double wgt = 1.0;
      if (P.omega > 1) wgt = load_gates(a.alpha, a.eta, a.theta, a.gamma, P.T, P.H, b, hh, c * P.chunk + i).g;
      g1 += wgt * err[i * D + d] * act[i * E + e];
      g2 += wgt * chain[i * E + e] * kd[i * D + d];
    }
    S1[idx] = theta * S1[idx] - eta * s * g1;
    S2t[idx] = theta * S2t[idx] - eta * s * g2;
  }
  __syncthreads();
}

// y_t = q_t + W1_t gelu_tanh(W2_t q_t)   (memory_layer.py:592-595)
template <typename TA>
__device__ void readout(const FwdArgs& a, int b, int hh, int t, const double* W1, const double* W2t, double* qd,
                        double* z, double* p) {
  const AtlasScanParams& P = a.p;
  const int D = P.D, E = P.E;
  const TA* q = cptr<TA>(a.q);
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    qd[d] = t < P.T ? (double)ld_act(q, (((size_t)b * P.T + t) * P.H + hh) * D + d) : 0.0;
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    double s = 0;
    for (int d = 0; d < D; ++d) s += W2t[(size_t)d * E + e] * qd[d];
    z[e] = s;
    p[e] = gelu_tanh(s);
  }
  __syncthreads();
  if (t < P.T) {
    TA* y = (TA*)a.y;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      double s = qd[d];
      for (int e = 0; e < E; ++e) s += W1[(size_t)d * E + e] * p[e];
      st_act(y, (((size_t)b * P.T + t) * P.H + hh) * D + d, (float)s);
    }
  }
  __syncthreads();
}

template <typename TA>
__global__ void __launch_bounds__(kThreads) fwd_kernel(FwdArgs a) {
  const AtlasScanParams& P = a.p;
  const int D = P.D, E = P.E, cs = P.chunk;
  const size_t DE = (size_t)D * E;
  const int bh = blockIdx.x;
  const int b = bh / P.H, hh = bh % P.H;
  double* base = (double*)a.ws + (size_t)bh * (fwd_ws_doubles(D, E, cs) + 2 * D);
  FwdWS w = carve_fwd(base, D, E, cs);
  double* qd = base + fwd_ws_doubles(D, E, cs);
  load_state(a.W1_in, a.W2_in, a.S1_in, a.S2_in, bh, D, E, w.W1, w.W2, w.S1, w.S2);
  const int nc = n_chunks(P);
  for (int c = 0; c < nc; ++c) {
    if (a.saved) {
      double* sv = (double*)a.saved + ((size_t)bh * nc + c) * 4 * DE;
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
        sv[i] = w.W1[i];
        sv[DE + i] = w.W2[i];
        sv[2 * DE + i] = w.S1[i];
        sv[3 * DE + i] = w.S2[i];
      }
    }
    frozen_forward<TA>(a, b, hh, c, w.W1, w.W2, w.h, w.act, w.err, w.chain, w.kd);
    for (int r = 0; r < cs; ++r) {
      const int t = c * cs + r;
      Gates g = load_gates(a.alpha, a.eta, a.theta, a.gamma, P.T, P.H, b, hh, t);
      momentum_step(a, b, hh, c, r, w.S1, w.S2, w.err, w.act, w.chain, w.kd, g.t, g.e);
      pe_forward(w.S1, w.O, D, E, P.ns_steps, 1e-12, w.pe, nullptr, w.red);
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) w.W1[i] = g.a * w.W1[i] + w.O[i];
      __syncthreads();
      pe_forward(w.S2, w.O, D, E, P.ns_steps, 1e-12, w.pe, nullptr, w.red);
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) w.W2[i] = g.a * w.W2[i] + w.O[i];
      __syncthreads();
      readout<TA>(a, b, hh, t, w.W1, w.W2, qd, w.z, w.p);
    }
  }
  store_state(a.W1_out, a.W2_out, a.S1_out, a.S2_out, bh, D, E, w.W1, w.W2, w.S1, w.S2);
}

}  // namespace exact
}  // namespace atlas

namespace atlas {
namespace exact {

__host__ __device__ inline size_t bwd_extra_doubles(int D, int E, int cs, int steps) {
  size_t DE = (size_t)D * E, DD = (size_t)D * D;
  return (size_t)(cs + 1) * 4 * DE   // per-token states
         + 4 * DE                     // dW1 dW2 dS1 dS2
         + 2 * DE + 3 * DD            // VJP work
         + (size_t)steps * (DE + 2 * DD)  // PE history
         + 3 * (size_t)cs * E + 2 * (size_t)cs * D  // dact dchain dh derr dkd
         + 4 * (size_t)cs                           // dalpha deta dtheta dgamma
         + 4 * (size_t)E + 4 * (size_t)D + 32;      // dp dz wv1 wv2 | dyv qd w1 w2
}

__device__ double block_dot(const double* x, const double* y, size_t n, double* red) {
  double s = 0;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) s += x[i] * y[i];
  return block_sum(s, red);
}
// out[d] = sum_e M[d][e] x[e]
__device__ void mv(const double* M, const double* x, double* out, int D, int E) {
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    double s = 0;
    for (int e = 0; e < E; ++e) s += M[(size_t)d * E + e] * x[e];
    out[d] = s;
  }
}
// out[e] = sum_d M[d][e] y[d]
__device__ void mvt(const double* M, const double* y, double* out, int D, int E) {
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    double s = 0;
    for (int d = 0; d < D; ++d) s += M[(size_t)d * E + e] * y[d];
    out[e] = s;
  }
}

template <typename TA>
__global__ void __launch_bounds__(kThreads) bwd_kernel(BwdArgs a) {
  const AtlasScanParams& P = a.p;
  const int D = P.D, E = P.E, cs = P.chunk, T = P.T, H = P.H, steps = P.ns_steps;
  const size_t DE = (size_t)D * E, DD = (size_t)D * D;
  const int bh = blockIdx.x;
  const int b = bh / H, hh = bh % H;
  const double s = 2.0 / D;
  const bool win = P.omega > 1;
  double* base = (double*)a.ws + (size_t)bh * (fwd_ws_doubles(D, E, cs) + bwd_extra_doubles(D, E, cs, steps));
  FwdWS w = carve_fwd(base, D, E, cs);
  double* p = base + fwd_ws_doubles(D, E, cs);
  double* HS = p; p += (size_t)(cs + 1) * 4 * DE;
  double* dW1 = p; p += DE;
  double* dW2 = p; p += DE;
  double* dS1 = p; p += DE;
  double* dS2 = p; p += DE;
  VJPWork vw;
  vw.G = p; p += DE;
  vw.dX = p; p += DE;
  vw.dB = p; p += DD;
  vw.dA = p; p += DD;
  vw.T = p; p += DD;
  double* hist = p; p += (size_t)steps * (DE + 2 * DD);
  double* dact = p; p += (size_t)cs * E;
  double* dchain = p; p += (size_t)cs * E;
  double* dh = p; p += (size_t)cs * E;
  double* derr = p; p += (size_t)cs * D;
  double* dkd = p; p += (size_t)cs * D;
  double* dal = p; p += cs;
  double* det = p; p += cs;
  double* dth = p; p += cs;
  double* dga = p; p += cs;
  double* dp = p; p += E;
  double* dz = p; p += E;
  double* v1 = p; p += E;
  double* v2 = p; p += E;
  double* dyv = p; p += D;
  double* qd = p; p += D;
  double* w1 = p; p += D;
  double* w2 = p; p += D;

  FwdArgs fa;
  fa.p = P; fa.q = a.q; fa.k = a.k; fa.v = a.v;
  fa.alpha = a.alpha; fa.eta = a.eta; fa.theta = a.theta; fa.gamma = a.gamma;

  load_state(a.dW1_out, a.dW2_out, a.dS1_out, a.dS2_out, bh, D, E, dW1, dW2, dS1, dS2);
  if (!a.dW2_out)  // load_state puts the LM identity into a missing W2; a missing cotangent is zero
    for (size_t i = threadIdx.x; i < DE; i += blockDim.x) dW2[i] = 0.0;
  __syncthreads();
  const TA* q = (const TA*)a.q;
  const TA* dy = (const TA*)a.dy;
  const int nc = n_chunks(P);
  for (int c = nc - 1; c >= 0; --c) {
    const double* sv = (const double*)a.saved + ((size_t)bh * nc + c) * 4 * DE;
    for (size_t i = threadIdx.x; i < 4 * DE; i += blockDim.x) HS[i] = sv[i];
    __syncthreads();
    frozen_forward<TA>(fa, b, hh, c, HS, HS + DE, w.h, w.act, w.err, w.chain, w.kd);
    // forward recompute of the per-token states
    for (int r = 0; r < cs; ++r) {
      Gates g = load_gates(a.alpha, a.eta, a.theta, a.gamma, T, H, b, hh, c * cs + r);
      double* prv = HS + (size_t)r * 4 * DE;
      double* cur = prv + 4 * DE;
      for (size_t i = threadIdx.x; i < 4 * DE; i += blockDim.x) cur[i] = prv[i];
      __syncthreads();
      momentum_step(fa, b, hh, c, r, cur + 2 * DE, cur + 3 * DE, w.err, w.act, w.chain, w.kd, g.t, g.e);
      pe_forward(cur + 2 * DE, w.O, D, E, steps, 1e-12, w.pe, nullptr, w.red);
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) cur[i] = g.a * cur[i] + w.O[i];
      __syncthreads();
      pe_forward(cur + 3 * DE, w.O, D, E, steps, 1e-12, w.pe, nullptr, w.red);
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) cur[DE + i] = g.a * cur[DE + i] + w.O[i];
      __syncthreads();
    }
    for (int i = threadIdx.x; i < cs * E; i += blockDim.x) dact[i] = dchain[i] = 0.0;
    for (int i = threadIdx.x; i < cs * D; i += blockDim.x) derr[i] = dkd[i] = 0.0;
    for (int i = threadIdx.x; i < cs; i += blockDim.x) dal[i] = det[i] = dth[i] = dga[i] = 0.0;
    __syncthreads();
    for (int r = cs - 1; r >= 0; --r) {
      const int t = c * cs + r;
      Gates g = load_gates(a.alpha, a.eta, a.theta, a.gamma, T, H, b, hh, t);
      const double* prv = HS + (size_t)r * 4 * DE;
      const double* cur = prv + 4 * DE;
      // --- read-out backward (memory_layer.py:592-595) ---
      for (int d = threadIdx.x; d < D; d += blockDim.x) {
        size_t o = (((size_t)b * T + t) * H + hh) * D + d;
        qd[d] = t < T ? (double)ld_act(q, o) : 0.0;
        dyv[d] = t < T ? (double)ld_act(dy, o) : 0.0;
      }
      __syncthreads();
      mvt(cur + DE, qd, w.z, D, E);     // z = W2 q
      mvt(cur, dyv, dp, D, E);          // dp = W1^T dy
      __syncthreads();
      for (int e = threadIdx.x; e < E; e += blockDim.x) {
        w.p[e] = gelu_tanh(w.z[e]);
        dz[e] = dp[e] * gelu_tanh_grad(w.z[e]);
      }
      __syncthreads();
      if (t < T) {
        TA* dq = (TA*)a.dq;
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
          double sacc = dyv[d];
          for (int e = 0; e < E; ++e) sacc += cur[DE + (size_t)d * E + e] * dz[e];
          st_act(dq, (((size_t)b * T + t) * H + hh) * D + d, (float)sacc);
        }
      }
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
        int d = (int)(i / E), e = (int)(i % E);
        dW1[i] += dyv[d] * w.p[e];
        dW2[i] += qd[d] * dz[e];
      }
      __syncthreads();
      // --- memory scan W_t = alpha W_{t-1} + O_t ---
      double da = block_dot(dW1, prv, DE, w.red) + block_dot(dW2, prv + DE, DE, w.red);
      if (P.pe_ste) {
        for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
          dS1[i] += dW1[i];
          dS2[i] += dW2[i];
        }
        __syncthreads();
      } else {
        double n1 = pe_forward(cur + 2 * DE, w.O, D, E, steps, 1e-12, w.pe, hist, w.red);
        pe_vjp(cur + 2 * DE, dW1, dS1, D, E, steps, n1, hist, vw, w.red);
        double n2 = pe_forward(cur + 3 * DE, w.O, D, E, steps, 1e-12, w.pe, hist, w.red);
        pe_vjp(cur + 3 * DE, dW2, dS2, D, E, steps, n2, hist, vw, w.red);
      }
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
        dW1[i] *= g.a;
        dW2[i] *= g.a;
      }
      __syncthreads();
      // --- momentum scan S_t = theta S_{t-1} + m_t, m_t = -eta G_t ---
      double dt_ = block_dot(dS1, prv + 2 * DE, DE, w.red) + block_dot(dS2, prv + 3 * DE, DE, w.red);
      double de_ = 0;
      int i0 = win ? max(0, r - P.omega + 1) : r;
      for (int i = i0; i <= r; ++i) {
        double gi = win ? (double)load_gates(a.alpha, a.eta, a.theta, a.gamma, T, H, b, hh, c * cs + i).g : 1.0;
        mv(dS1, w.act + (size_t)i * E, w1, D, E);      // dS1 act_i
        mv(dS2, w.chain + (size_t)i * E, w2, D, E);    // dS2^T-stored . chain_i
        mvt(dS1, w.err + (size_t)i * D, v1, D, E);     // dS1^T err_i
        mvt(dS2, w.kd + (size_t)i * D, v2, D, E);      // dS2 k_i
        __syncthreads();
        double ip = 0;
        for (int d = threadIdx.x; d < D; d += blockDim.x) ip += w.err[i * D + d] * w1[d] + w.kd[i * D + d] * w2[d];
        ip = block_sum(ip, w.red);  // <dS, u_i> / s
        de_ += -gi * s * ip;
        if (threadIdx.x == 0 && win) dga[i] += -g.e * s * ip;
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
          derr[i * D + d] += -g.e * s * gi * w1[d];
          dkd[i * D + d] += -g.e * s * gi * w2[d];
        }
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
          dact[i * E + e] += -g.e * s * gi * v1[e];
          dchain[i * E + e] += -g.e * s * gi * v2[e];
        }
        __syncthreads();
      }
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
        dS1[i] *= g.t;
        dS2[i] *= g.t;
      }
      if (threadIdx.x == 0) {
        dal[r] = da;
        dth[r] = dt_;
        det[r] = de_;
      }
      __syncthreads();
    }
    // --- frozen-state pass backward (memory_layer.py:504-520) ---
    const double* W1_0 = HS;
    const double* W2_0 = HS + DE;
    for (int i = threadIdx.x; i < cs * E; i += blockDim.x) {
      int r = i / E, e = i % E;
      double w1t = 0;
      for (int d = 0; d < D; ++d) w1t += W1_0[(size_t)d * E + e] * w.err[r * D + d];
      double hv = w.h[i];
      dh[i] = dchain[i] * w1t * gelu_erf_second(hv);
      dchain[i] = dchain[i] * gelu_erf_prime(hv);  // now d(W1^T err)
    }
    __syncthreads();
    for (int i = threadIdx.x; i < cs * D; i += blockDim.x) {
      int r = i / D, d = i % D;
      double sacc = 0;
      for (int e = 0; e < E; ++e) sacc += W1_0[(size_t)d * E + e] * dchain[r * E + e];
      derr[i] += sacc;
    }
    __syncthreads();
    for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
      int d = (int)(i / E), e = (int)(i % E);
      double s1 = 0;
      for (int r = 0; r < cs; ++r)
        s1 += w.err[r * D + d] * dchain[r * E + e] + derr[r * D + d] * w.act[r * E + e];
      dW1[i] += s1;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < cs * E; i += blockDim.x) {
      int r = i / E, e = i % E;
      double sacc = 0;
      for (int d = 0; d < D; ++d) sacc += W1_0[(size_t)d * E + e] * derr[r * D + d];
      dh[i] += (dact[i] + sacc) * gelu_tanh_grad(w.h[i]);
    }
    __syncthreads();
    for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
      int d = (int)(i / E), e = (int)(i % E);
      double s2 = 0;
      for (int r = 0; r < cs; ++r) s2 += w.kd[r * D + d] * dh[r * E + e];
      dW2[i] += s2;
    }
    TA* dkp = (TA*)a.dk;
    TA* dvp = (TA*)a.dv;
    for (int i = threadIdx.x; i < cs * D; i += blockDim.x) {
      int r = i / D, d = i % D;
      int t = c * cs + r;
      if (t >= T) continue;
      double sacc = dkd[i] + derr[i];
      for (int e = 0; e < E; ++e) sacc += W2_0[(size_t)d * E + e] * dh[r * E + e];
      size_t o = (((size_t)b * T + t) * H + hh) * D + d;
      st_act(dkp, o, (float)sacc);
      st_act(dvp, o, (float)(-derr[i]));
    }
    for (int r = threadIdx.x; r < cs; r += blockDim.x) {
      int t = c * cs + r;
      if (t >= T) continue;
      size_t o = ((size_t)b * T + t) * H + hh;
      if (a.dalpha) a.dalpha[o] = (float)dal[r];
      if (a.deta) a.deta[o] = (float)det[r];
      if (a.dtheta) a.dtheta[o] = (float)dth[r];
      if (a.dgamma) a.dgamma[o] = (float)dga[r];
    }
    __syncthreads();
    if (P.stop_grad_chunks) {
      for (size_t i = threadIdx.x; i < DE; i += blockDim.x) dW1[i] = dW2[i] = dS1[i] = dS2[i] = 0.0;
      __syncthreads();
    }
  }
  store_state(a.dW1_in, a.dW2_in, a.dS1_in, a.dS2_in, bh, D, E, dW1, dW2, dS1, dS2);
}

// ---- standalone batched Polar Express (one CTA per matrix) -------------------
__global__ void __launch_bounds__(kThreads) pe_kernel(const float* X, float* Y, int rows, int cols, int steps,
                                                      float eps, double* ws) {
  const bool tall = rows > cols;
  const int D = tall ? cols : rows, E = tall ? rows : cols;
  const size_t DE = (size_t)D * E, DD = (size_t)D * D;
  double* base = ws + (size_t)blockIdx.x * (4 * DE + 3 * DD + 32);
  double* S = base;
  double* O = S + DE;
  PEWork w;
  w.X = O + DE;
  w.Xn = w.X + DE;
  w.A = w.Xn + DE;
  w.AA = w.A + DD;
  w.Bm = w.AA + DD;
  double* red = w.Bm + DD;
  const float* x = X + (size_t)blockIdx.x * DE;
  for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
    int r = (int)(i / cols), cc = (int)(i % cols);
    // wide storage: tall inputs are transposed
    S[tall ? (size_t)cc * E + r : i] = (double)x[i];
  }
  __syncthreads();
  pe_forward(S, O, D, E, steps, (double)eps, w, nullptr, red);
  float* y = Y + (size_t)blockIdx.x * DE;
  for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
    int r = (int)(i / cols), cc = (int)(i % cols);
    y[i] = (float)O[tall ? (size_t)cc * E + r : i];
  }
}

// ---- linear memory (memory_layer.py:468-494), forward and backward ----------------
// One CTA per chain, float64, the square memory M and momentum S (reference layout
// M[v][k]) in the workspace.  Square Polar Express goes through the wide routine
// (memory_layer.py:65-69: A = X X^T, X' = a X + B X).
__host__ __device__ inline size_t lin_ws_doubles(int D, int cs, int nch, int steps) {
  const size_t DD = (size_t)D * D;
  return DD * (2 + 5 + 1 + 3 * (size_t)steps + 5 + 3 + 2 * (size_t)nch + 3 * (size_t)cs + 1) +
         4 * (size_t)cs * D + 4 * (size_t)D + 4 * (size_t)cs + 32;
}

// err_r = M0 k_r - v_r (memory_layer.py:471-472) for the chunk's tokens (0 on padding)
template <typename TA>
__device__ void lin_frozen(const LinArgs& a, int b, int hh, int c, const double* M0, double* kd, double* err) {
  const AtlasScanParams& P = a.p;
  const int D = P.D, cs = P.chunk;
  for (int i = threadIdx.x; i < cs * D; i += blockDim.x) {
    const int t = c * cs + i / D, d = i % D;
    kd[i] = t < P.T ? (double)ld_act((const TA*)a.k, (((size_t)b * P.T + t) * P.H + hh) * D + d) : 0.0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < cs * D; i += blockDim.x) {
    const int r = i / D, vv = i % D, t = c * cs + r;
    double sum = 0;
    for (int k = 0; k < D; ++k) sum += M0[(size_t)vv * D + k] * kd[r * D + k];
    err[i] = sum - (t < P.T ? (double)ld_act((const TA*)a.v, (((size_t)b * P.T + t) * P.H + hh) * D + vv) : 0.0);
  }
  __syncthreads();
}

// window weight of token i in G_r (1 without the Omega window), memory_layer.py:233-253
__device__ __forceinline__ double lin_w(const LinArgs& a, int b, int hh, int tok) {
  return a.p.omega > 1 ? (double)load_gates(a.alpha, a.eta, a.theta, a.gamma, a.p.T, a.p.H, b, hh, tok).g : 1.0;
}

// S <- theta S - eta G_r, G_r = sum_{i in window(r)} w_i (2/D) err_i k_i^T  (523-533)
__device__ void lin_momentum(const LinArgs& a, int b, int hh, int c, int r, double* S, const double* err,
                             const double* kd, double th, double et) {
  const int D = a.p.D;
  const double s = 2.0 / D;
  const int i0 = a.p.omega > 1 ? max(0, r - a.p.omega + 1) : r;
  for (int idx = threadIdx.x; idx < D * D; idx += blockDim.x) {
    const int vv = idx / D, k = idx % D;
    double g = 0;
    for (int i = i0; i <= r; ++i) g += lin_w(a, b, hh, c * a.p.chunk + i) * err[i * D + vv] * kd[i * D + k];
    S[idx] = th * S[idx] - et * s * g;
  }
  __syncthreads();
}

template <typename TA>
__global__ void __launch_bounds__(kThreads) lin_kernel(LinArgs a) {
  const AtlasScanParams& P = a.p;
  const int D = P.D, cs = P.chunk, T = P.T, H = P.H, steps = P.ns_steps, nc = n_chunks(P);
  const size_t DD = (size_t)D * D;
  const int bh = blockIdx.x, b = bh / H, hh = bh % H;
  const double s = 2.0 / D;
  const bool win = P.omega > 1;
  double* p = (double*)a.ws + (size_t)bh * lin_ws_doubles(D, cs, nc, steps);
  double* M = p; p += DD;
  double* S = p; p += DD;
  PEWork pw;
  pw.X = p; p += DD;
  pw.Xn = p; p += DD;
  pw.A = p; p += DD;
  pw.AA = p; p += DD;
  pw.Bm = p; p += DD;
  double* O = p; p += DD;
  double* hist = p; p += 3 * (size_t)steps * DD;
  VJPWork vw;
  vw.G = p; p += DD;
  vw.dX = p; p += DD;
  vw.dB = p; p += DD;
  vw.dA = p; p += DD;
  vw.T = p; p += DD;
  double* dM = p; p += DD;
  double* dS = p; p += DD;
  double* dSt = p; p += DD;
  double* carry = p; p += 2 * DD * nc;
  double* Sall = p; p += (size_t)cs * DD;
  double* Mall = p; p += (size_t)(cs + 1) * DD;
  double* R = p; p += (size_t)cs * DD;
  double* kd = p; p += (size_t)cs * D;
  double* err = p; p += (size_t)cs * D;
  double* tR = p; p += (size_t)cs * D;
  double* dkd = p; p += (size_t)cs * D;
  double* qd = p; p += D;
  double* dyv = p; p += D;
  p += 2 * D;
  double* gsc = p; p += 4 * cs;  // dalpha, deta, dtheta, dgamma of the chunk
  double* red = p;
  const size_t off = (size_t)bh * DD;
  for (size_t i = threadIdx.x; i < DD; i += blockDim.x) {
    M[i] = a.M_in ? (double)a.M_in[off + i] : 0.0;  // memory_layer.py:138-140: zeros
    S[i] = a.S_in ? (double)a.S_in[off + i] : 0.0;
  }
  __syncthreads();
  // ---- forward (the whole output in forward mode; the chunk carries in backward mode) ----
  for (int c = 0; c < nc; ++c) {
    if (a.bwd)
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) {
        carry[2 * DD * c + i] = M[i];
        carry[2 * DD * c + DD + i] = S[i];
      }
    lin_frozen<TA>(a, b, hh, c, M, kd, err);
    for (int r = 0; r < cs; ++r) {
      const int t = c * cs + r;
      const Gates g = load_gates(a.alpha, a.eta, a.theta, a.gamma, T, H, b, hh, t);
      lin_momentum(a, b, hh, c, r, S, err, kd, g.t, g.e);
      pe_forward(S, O, D, D, steps, 1e-12, pw, nullptr, red);
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) M[i] = g.a * M[i] + O[i];
      __syncthreads();
      if (!a.bwd && t < T) {  // y_t = M_t q_t (490-492)
        for (int vv = threadIdx.x; vv < D; vv += blockDim.x) {
          double sum = 0;
          for (int k = 0; k < D; ++k)
            sum += M[(size_t)vv * D + k] * (double)ld_act((const TA*)a.q, (((size_t)b * T + t) * H + hh) * D + k);
          st_act((TA*)a.y, (((size_t)b * T + t) * H + hh) * D + vv, (float)sum);
        }
      }
    }
  }
  if (!a.bwd) {
    for (size_t i = threadIdx.x; i < DD; i += blockDim.x) {
      if (a.M_out) a.M_out[off + i] = (float)M[i];
      if (a.S_out) a.S_out[off + i] = (float)S[i];
    }
    return;
  }
  // ---- backward, chunks in reverse ----
  for (size_t i = threadIdx.x; i < DD; i += blockDim.x) {
    dM[i] = a.dM_out ? (double)a.dM_out[off + i] : 0.0;
    dS[i] = a.dS_out ? (double)a.dS_out[off + i] : 0.0;
  }
  __syncthreads();
  for (int c = nc - 1; c >= 0; --c) {
    const double* M0 = carry + 2 * DD * c;
    const double* S0 = M0 + DD;
    for (size_t i = threadIdx.x; i < DD; i += blockDim.x) {
      Mall[i] = M0[i];
      S[i] = S0[i];
    }
    for (size_t i = threadIdx.x; i < (size_t)cs * DD; i += blockDim.x) R[i] = 0.0;
    __syncthreads();
    lin_frozen<TA>(a, b, hh, c, M0, kd, err);
    for (int r = 0; r < cs; ++r) {  // recompute S_t and M_t of the chunk
      const Gates g = load_gates(a.alpha, a.eta, a.theta, a.gamma, T, H, b, hh, c * cs + r);
      lin_momentum(a, b, hh, c, r, S, err, kd, g.t, g.e);
      double* Sr = Sall + r * DD;
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) Sr[i] = S[i];
      pe_forward(S, O, D, D, steps, 1e-12, pw, nullptr, red);
      const double* Mp = Mall + r * DD;
      double* Mr = Mall + (r + 1) * DD;
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) Mr[i] = g.a * Mp[i] + O[i];
      __syncthreads();
    }
    for (int r = cs - 1; r >= 0; --r) {
      const int t = c * cs + r;
      const Gates g = load_gates(a.alpha, a.eta, a.theta, a.gamma, T, H, b, hh, t);
      for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const size_t o = (((size_t)b * T + t) * H + hh) * D + d;
        qd[d] = t < T ? (double)ld_act((const TA*)a.q, o) : 0.0;
        dyv[d] = t < T && a.dy ? (double)ld_act((const TA*)a.dy, o) : 0.0;
      }
      __syncthreads();
      const double* Mr = Mall + (r + 1) * DD;
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) dM[i] += dyv[i / D] * qd[i % D];
      if (t < T)  // dq = M_t^T dy
        for (int k = threadIdx.x; k < D; k += blockDim.x) {
          double sum = 0;
          for (int vv = 0; vv < D; ++vv) sum += Mr[(size_t)vv * D + k] * dyv[vv];
          st_act((TA*)a.dq, (((size_t)b * T + t) * H + hh) * D + k, (float)sum);
        }
      __syncthreads();
      double acc = 0;
      const double* Mp = Mall + r * DD;
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) acc += dM[i] * Mp[i];
      const double dal = block_sum(acc, red);
      // dS_t = theta_{t+1} dS_{t+1} + PE_vjp(S_t, dO_t = dM_t)
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) dSt[i] = dS[i];
      __syncthreads();
      const double* Sr = Sall + r * DD;
      const double n = pe_forward(Sr, O, D, D, steps, 1e-12, pw, hist, red);
      pe_vjp(Sr, dM, dSt, D, D, steps, n, hist, vw, red);
      const double* Sp = r > 0 ? Sall + (r - 1) * DD : S0;
      const int i0 = win ? max(0, r - P.omega + 1) : r;
      double ath = 0, aet = 0;
      for (size_t idx = threadIdx.x; idx < DD; idx += blockDim.x) {
        const int vv = (int)(idx / D), k = (int)(idx % D);
        ath += dSt[idx] * Sp[idx];
        double gsum = 0;
        for (int i = i0; i <= r; ++i) {
          gsum += lin_w(a, b, hh, c * cs + i) * s * err[i * D + vv] * kd[i * D + k];
          R[(size_t)i * DD + idx] -= g.e * dSt[idx];  // dG_r = -eta dS_t, to every token of the window
        }
        aet += dSt[idx] * gsum;
      }
      const double dth = block_sum(ath, red);
      const double det = -block_sum(aet, red);
      if (threadIdx.x == 0) {
        gsc[r] = dal;
        gsc[cs + r] = det;
        gsc[2 * cs + r] = dth;
      }
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) {
        dM[i] *= g.a;
        dS[i] = g.t * dSt[i];
      }
      __syncthreads();
    }
    // u_i = (2/D) err_i k_i^T with du_i = w_i R_i: tR_i = (2/D) R_i k_i, derr_i = w_i tR_i
    for (int i2 = threadIdx.x; i2 < cs * D; i2 += blockDim.x) {
      const int i = i2 / D, vv = i2 % D;
      double sum = 0;
      for (int k = 0; k < D; ++k) sum += R[(size_t)i * DD + (size_t)vv * D + k] * kd[i * D + k];
      tR[i2] = s * sum;
    }
    for (int i2 = threadIdx.x; i2 < cs * D; i2 += blockDim.x) {
      const int i = i2 / D, k = i2 % D;
      const double wi = lin_w(a, b, hh, c * cs + i);
      double sum = 0;
      for (int vv = 0; vv < D; ++vv) sum += R[(size_t)i * DD + (size_t)vv * D + k] * err[i * D + vv];
      dkd[i2] = wi * s * sum;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < cs; i += blockDim.x) {  // dgamma_i = <u_i, R_i>
      double sum = 0;
      for (int vv = 0; vv < D; ++vv) sum += err[i * D + vv] * tR[i * D + vv];
      gsc[3 * cs + i] = sum;
    }
    __syncthreads();
    for (int i2 = threadIdx.x; i2 < cs * D; i2 += blockDim.x) tR[i2] *= lin_w(a, b, hh, c * cs + i2 / D);  // derr
    __syncthreads();
    for (int i2 = threadIdx.x; i2 < cs * D; i2 += blockDim.x) {  // err = M0 k - v
      const int i = i2 / D, k = i2 % D, t = c * cs + i;
      double sum = dkd[i2];
      for (int vv = 0; vv < D; ++vv) sum += M0[(size_t)vv * D + k] * tR[i * D + vv];
      if (t < T) {
        const size_t o = (((size_t)b * T + t) * H + hh) * D + k;
        st_act((TA*)a.dk, o, (float)sum);
        st_act((TA*)a.dv, (((size_t)b * T + t) * H + hh) * D + k, (float)-tR[i2]);
      }
    }
    for (size_t idx = threadIdx.x; idx < DD; idx += blockDim.x) {
      const int vv = (int)(idx / D), k = (int)(idx % D);
      double sum = 0;
      for (int i = 0; i < cs; ++i) sum += tR[i * D + vv] * kd[i * D + k];
      dM[idx] += sum;
    }
    for (int r = threadIdx.x; r < cs; r += blockDim.x) {
      const int t = c * cs + r;
      if (t >= T) continue;
      const size_t gi = ((size_t)b * T + t) * H + hh;
      a.dalpha[gi] = (float)gsc[r];
      a.deta[gi] = (float)gsc[cs + r];
      a.dtheta[gi] = (float)gsc[2 * cs + r];
      if (a.dgamma) a.dgamma[gi] = win ? (float)gsc[3 * cs + r] : 0.f;
    }
    __syncthreads();
    if (P.stop_grad_chunks) {  // memory_layer.py:665: the incoming carry is detached
      for (size_t i = threadIdx.x; i < DD; i += blockDim.x) dM[i] = dS[i] = 0.0;
      __syncthreads();
    }
  }
  for (size_t i = threadIdx.x; i < DD; i += blockDim.x) {
    if (a.dM_in) a.dM_in[off + i] = (float)dM[i];
    if (a.dS_in) a.dS_in[off + i] = (float)dS[i];
  }
}

// ---- host side ----------------------------------------------------------------
size_t saved_bytes(const AtlasScanParams& p) {
  return (size_t)p.B * p.H * n_chunks(p) * 4 * (size_t)p.D * p.E * sizeof(double);
}
size_t workspace_bytes(const AtlasScanParams& p) {
  size_t per = fwd_ws_doubles(p.D, p.E, p.chunk) + bwd_extra_doubles(p.D, p.E, p.chunk, p.ns_steps) + 2 * p.D;
  return (size_t)p.B * p.H * per * sizeof(double);
}
cudaError_t launch_fwd(const FwdArgs& a, cudaStream_t s) {
  dim3 grid(a.p.B * a.p.H);
  if (a.p.act_dtype == ATLAS_BF16)
    fwd_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(a);
  else
    fwd_kernel<float><<<grid, kThreads, 0, s>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_bwd(const BwdArgs& a, cudaStream_t s) {
  dim3 grid(a.p.B * a.p.H);
  if (a.p.act_dtype == ATLAS_BF16)
    bwd_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(a);
  else
    bwd_kernel<float><<<grid, kThreads, 0, s>>>(a);
  return cudaGetLastError();
}
size_t lin_workspace_bytes(const AtlasScanParams& p) {
  return (size_t)p.B * p.H * lin_ws_doubles(p.D, p.chunk, n_chunks(p), p.ns_steps) * sizeof(double);
}
cudaError_t lin_launch(const LinArgs& a, cudaStream_t s) {
  dim3 grid(a.p.B * a.p.H);
  if (a.p.act_dtype == ATLAS_BF16)
    lin_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(a);
  else
    lin_kernel<float><<<grid, kThreads, 0, s>>>(a);
  return cudaGetLastError();
}
size_t pe_workspace_bytes(int64_t batch, int rows, int cols, int) {
  size_t D = rows < cols ? rows : cols;
  size_t DE = (size_t)rows * cols;
  return (size_t)batch * (4 * DE + 3 * D * D + 32) * sizeof(double);
}
cudaError_t launch_pe(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps, void* ws,
                      cudaStream_t s) {
  for (int64_t off = 0; off < batch; off += 65535) {
    int n = (int)((batch - off) < 65535 ? (batch - off) : 65535);
    size_t DE = (size_t)rows * cols;
    size_t D = rows < cols ? rows : cols;
    pe_kernel<<<n, kThreads, 0, s>>>(X + off * DE, Y + off * DE, rows, cols, steps, eps,
                                     (double*)ws + off * (4 * DE + 3 * D * D + 32));
  }
  return cudaGetLastError();
}

}  // namespace exact
}  // namespace atlas
