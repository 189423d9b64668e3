// tcgen05 (sm_100a) batched Polar Express for large matrices: the Muon
// orthogonalisation of stacked parameter gradients (atlas_jax/optim.py:56-108,
// Polar Express at 68-83; same iteration as memory_layer.py:43-71), e.g. the 170M
// model's (12, 768, 768), (12, 4096, 768), (12, 768, 2048) stacks.
//
// Matrices are held "wide" (D = min(rows, cols) rows, E = max columns; tall inputs
// are transposed on the way in and out), so every step is
//   A = X X^T,   B = b A + c A A,   X <- a X + B X
// as three launches of one batched GEMM kernel.  The GEMM reads float32 operands,
// splits them into fp16 hi/lo parts (of 256 x the value) while staging them in shared
// memory, and accumulates hi*hi + hi*lo + lo*hi on the tensor cores in float32 in TMEM
// (about 22 significant bits per operand; a single 16-bit pass loses the near-null
// directions that Polar Express amplifies).  The epilogue fuses alpha * product + beta * addend.
//
// GEMM kernel: one CTA of 4 warps per 128 x 128 output tile and batch entry; K in
// chunks of 32, two shared-memory stages (the next chunk's coalesced global loads are
// in flight while the current chunk's MMAs run); one elected thread issues the MMAs
// and commits them to the stage's mbarrier; every wait is bounded and records
// ATLAS_ERR_DEVICE_TIMEOUT instead of hanging.
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "pe_tma.h"
#include "scan_internal.h"
#include "tc_ops.cuh"

namespace atlas {
namespace pet {
using namespace tcx;

constexpr int TM = 128, TN = 128, TK = 32, NTH = 128;
constexpr int TILE = 128 * TK * 2;  // bytes of one 16-bit 128 x 32 (or 32 x 128) tile

struct __align__(1024) Smem {
  uint8_t a[2][2][TILE];  // [stage][hi, lo]: 128 (m) x 32 (k), K-major
  uint8_t b[2][2][TILE];  // [stage][hi, lo]: 128 (n) x 32 (k) K-major, or 32 (k) x 128 (n) MN-major
  uint64_t bar[2];
  uint32_t tmem;
  int bad;
};

// C[m][n] = alpha * sum_k A[m][k] B(n, k) + beta * Dm[m][n] for one batch entry
// (blockIdx.z), B(n, k) = Bp[n * ldb + k] (b_kn = 0) or Bp[k * ldb + n] (b_kn = 1).
// alpha / beta come from the Polar Express step `st` by mode: 0 -> (1, 0), 1 -> (c, b),
// 2 -> (1, a).
struct GemmArgs {
  const float* A;
  const float* B;
  const float* Dm;
  float* C;
  int64_t sA, sB, sD, sC;  // batch strides (floats)
  int lda, ldb, ldd, ldc;
  int M, N, K;
  int b_kn, mode, st;
  float sa, sb;  // operand split scales (powers of two)
  int* status;
};

// Operand split: 4 consecutive values v -> fp16 hi = fp16(sc v), lo = fp16(sc v - hi),
// 8 bytes into each tile.  hi + lo keeps about 22 significant bits as long as the lo
// parts stay above the fp16 subnormal floor, so each operand gets a power-of-two
// scale sc that lifts its typical entry to about 1 (operand_scale): large matrices
// have small entries (a normalised 768 x 4096 X has entries near 5e-4).  Every operand
// is bounded (normalised X <= 1.2, A <= 1.44, B <= 64), and the scales are capped so
// that sc * |v| stays below the fp16 maximum.  A product accumulates sa * sb times
// its value; the epilogue divides it out.
__device__ __forceinline__ void split4(uint8_t* th, uint8_t* tl, uint32_t off, const float* v, float sc) {
  uint32_t h[2], l[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float y0 = v[2 * k] * sc, y1 = v[2 * k + 1] * sc;
    const __half2 hv = __floats2half2_rn(y0, y1);
    const float2 hf = __half22float2(hv);
    const __half2 lv = __floats2half2_rn(y0 - hf.x, y1 - hf.y);
    h[k] = *reinterpret_cast<const uint32_t*>(&hv);
    l[k] = *reinterpret_cast<const uint32_t*>(&lv);
  }
  *(uint2*)(th + off) = make_uint2(h[0], h[1]);
  *(uint2*)(tl + off) = make_uint2(l[0], l[1]);
}

__global__ void __launch_bounds__(NTH) gemm3_kernel(GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int t = threadIdx.x, w = t >> 5;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN, z = blockIdx.z;
  const float* A = g.A + z * g.sA;
  const float* Bp = g.B + z * g.sB;
  if (w == 0) {
    tmem_alloc(&s.tmem, 128);
    tmem_relinquish();
  }
  if (t == 0) {
    mbar_init(&s.bar[0], 1);
    mbar_init(&s.bar[1], 1);
    fence_mbar_init();
    s.bad = 0;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = s.tmem;
  const bool vecA = (g.lda & 3) == 0, vecB = (g.ldb & 3) == 0;
  const int nk = (g.K + TK - 1) / TK;
  // Coalesced staging: per pass, 8 threads cover one 128-byte row segment of a K-major
  // tile (32 k) and a warp reads 4 whole segments; for the MN-major B tile a warp
  // reads one 512-byte row of 128 n.  Each thread holds 8 passes x 4 floats; the next
  // chunk's loads are issued right after this chunk is staged, so they are in flight
  // while its MMAs run.
  float ra0[32], rb0[32];
  auto ld4 = [&](const float* p, int valid, bool vec, float* v) {
    if (vec && valid >= 4) {
      const float4 x = *(const float4*)p;
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = j < valid ? p[j] : 0.f;
    }
  };
  auto load = [&](int i, float* ra, float* rb) {
    const int k0 = i * TK, kq = 4 * (t & 7);
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const int m = m0 + 16 * p + (t >> 3);
      if (m < g.M)
        ld4(A + (size_t)m * g.lda + k0 + kq, g.K - k0 - kq, vecA, ra + 4 * p);
      else
        ra[4 * p] = ra[4 * p + 1] = ra[4 * p + 2] = ra[4 * p + 3] = 0.f;
      if (!g.b_kn) {
        const int n = n0 + 16 * p + (t >> 3);
        if (n < g.N)
          ld4(Bp + (size_t)n * g.ldb + k0 + kq, g.K - k0 - kq, vecB, rb + 4 * p);
        else
          rb[4 * p] = rb[4 * p + 1] = rb[4 * p + 2] = rb[4 * p + 3] = 0.f;
      } else {
        const int k = k0 + 4 * p + (t >> 5), nq = 4 * (t & 31);
        if (k < g.K)
          ld4(Bp + (size_t)k * g.ldb + n0 + nq, g.N - n0 - nq, vecB, rb + 4 * p);
        else
          rb[4 * p] = rb[4 * p + 1] = rb[4 * p + 2] = rb[4 * p + 3] = 0.f;
      }
    }
  };
  const uint32_t idesc = idesc_f16(128, 128, false, g.b_kn != 0);
  auto chunk = [&](int i, float* ra, float* rb) {
    const int st = i & 1;
    if (i >= 2 && !s.bad && !mbar_wait(&s.bar[st], ((i - 2) >> 1) & 1)) {  // MMAs of chunk i-2 read this stage
      s.bad = 1;
      set_status(g.status, ATLAS_ERR_DEVICE_TIMEOUT);
    }
    uint8_t *ah = s.a[st][0], *al = s.a[st][1], *bh = s.b[st][0], *bl = s.b[st][1];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      split4(ah, al, cm_off(16 * p + (t >> 3), 4 * (t & 7), TK), ra + 4 * p, g.sa);
      if (!g.b_kn)
        split4(bh, bl, cm_off(16 * p + (t >> 3), 4 * (t & 7), TK), rb + 4 * p, g.sb);
      else
        split4(bh, bl, cm_off(4 * p + (t >> 5), 4 * (t & 31), TN), rb + 4 * p, g.sb);
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    if (i + 1 < nk) load(i + 1, ra, rb);
    if (w == 0 && !__shfl_sync(0xffffffffu, s.bad, 0)) {  // warp-uniform: elect.sync needs the whole warp
      fence_after();
      const uint64_t da[2] = {desc_kmajor(smem_u32(ah), TK), desc_kmajor(smem_u32(al), TK)};
      uint64_t db[2];
      uint64_t sb;
      if (!g.b_kn) {
        db[0] = desc_kmajor(smem_u32(bh), TK);
        db[1] = desc_kmajor(smem_u32(bl), TK);
        sb = 256 >> 4;  // two core matrices along K
      } else {
        db[0] = desc_mnmajor(smem_u32(bh), TN);
        db[1] = desc_mnmajor(smem_u32(bl), TN);
        sb = (uint64_t)(2 * 16 * TN) >> 4;  // two 8-row blocks of k
      }
      constexpr uint64_t sa = 256 >> 4;
      const int ta[3] = {0, 0, 1}, tb[3] = {0, 1, 0};  // hi*hi, hi*lo, lo*hi
#pragma unroll
      for (int term = 0; term < 3; ++term)
#pragma unroll
        for (int ks = 0; ks < TK / 16; ++ks)
          mma_kf16(tm, da[ta[term]] + ks * sa, db[tb[term]] + ks * sb, idesc, (i || term || ks) ? 1u : 0u);
      mma_commit(&s.bar[st]);
    }
  };
  load(0, ra0, rb0);
  for (int i = 0; i < nk; ++i) chunk(i, ra0, rb0);
  // the last commit covers every MMA of the tile
  if (!s.bad && !mbar_wait(&s.bar[(nk - 1) & 1], ((nk - 1) >> 1) & 1)) {
    s.bad = 1;
    set_status(g.status, ATLAS_ERR_DEVICE_TIMEOUT);
  }
  fence_after();
  const float unsc = 1.f / (g.sa * g.sb);
  float alpha = unsc, beta = 0.f;
  if (g.mode == 1) {
    alpha = (float)kPE[g.st][2] * unsc;
    beta = (float)kPE[g.st][1];
  } else if (g.mode == 2) {
    beta = (float)kPE[g.st][0];
  }
  const int m = m0 + t;
  float* C = g.C + z * g.sC;
  const float* Dm = g.Dm ? g.Dm + z * g.sD : nullptr;
#pragma unroll 1
  for (int cb = 0; cb < TN / 32; ++cb) {
    float v[32];
    tmem_ld16(tm + ((uint32_t)(32 * w) << 16) + 32 * cb, v);
    tmem_ld16(tm + ((uint32_t)(32 * w) << 16) + 32 * cb + 16, v + 16);
    tmem_wait_ld();
    if (m < g.M && !s.bad) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + 32 * cb + j;
        if (n < g.N) {
          float r = alpha * v[j];
          if (Dm) r = fmaf(beta, Dm[(size_t)m * g.ldd + n], r);
          C[(size_t)m * g.ldc + n] = r;
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(tm, 128);
}

// X (wide, D x E) = S / (1.01 * sqrt(sum S^2 + eps) + 1e-6); one CTA per matrix.
__global__ void __launch_bounds__(256) normalize_kernel(const float* S, float* X, int rows, int cols, float eps) {
  __shared__ double red[8];
  const size_t DE = (size_t)rows * cols;
  const float* s = S + blockIdx.x * DE;
  float* x = X + blockIdx.x * DE;
  double ss = 0;
  for (size_t i = threadIdx.x; i < DE; i += blockDim.x) ss += (double)s[i] * s[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = (float)(1.0 / (sqrt(tot + (double)eps) * 1.01 + 1e-6));
  const bool tall = rows > cols;
  const int E = tall ? rows : cols;
  for (size_t i = threadIdx.x; i < DE; i += blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    x[tall ? (size_t)c * E + r : i] = s[i] * inv;
  }
}

// Y (rows x cols) from the wide X; grid-stride over every batch entry.
__global__ void unwide_kernel(const float* X, float* Y, int64_t batch, int rows, int cols) {
  const size_t DE = (size_t)rows * cols;
  const bool tall = rows > cols;
  const int E = tall ? rows : cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)batch * DE;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t z = i / DE, j = i % DE;
    const int r = (int)(j / cols), c = (int)(j % cols);
    Y[i] = X[z * DE + (tall ? (size_t)c * E + r : j)];
  }
}

static cudaError_t gemm(const GemmArgs& g, int64_t batch, cudaStream_t s) {
  const size_t smem = sizeof(Smem) + 1024;
  // per device (and cheap): set on every launch
  cudaError_t e = cudaFuncSetAttribute(gemm3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  for (int64_t z0 = 0; z0 < batch; z0 += 65535) {
    const int nz = (int)std::min<int64_t>(65535, batch - z0);
    GemmArgs h = g;
    h.A += z0 * g.sA;
    h.B += z0 * g.sB;
    h.C += z0 * g.sC;
    if (h.Dm) h.Dm += z0 * g.sD;
    dim3 grid((g.N + TN - 1) / TN, (g.M + TM - 1) / TM, nz);
    gemm3_kernel<<<grid, NTH, smem, s>>>(h);
  }
  return cudaGetLastError();
}

}  // namespace pet

namespace tcpe {

// Matrices with a short side >= 128 take the TMA path (pe_tma.cu): float32 A, and
// split operands X (ping-pong), A and B; float32 X only when there are no
// Newton-Schulz steps.
size_t workspace_bytes(int64_t batch, int rows, int cols) {
  const size_t D = std::min(rows, cols), DE = (size_t)rows * cols;
  if (pecl::usable(rows, cols) || pecta::usable(rows, cols)) return 256;  // on-chip kernels: no workspace
  if (pet2::usable(rows, cols)) return (size_t)batch * ((3 * DE + 3 * D * D) * sizeof(float) + 64 * sizeof(double));
  if (pet2::usable_packed(rows, cols))
    return (size_t)batch * ((3 * DE + 2 * D * D + D * 128) * sizeof(float) + 64 * sizeof(double));
  return (size_t)batch * (2 * DE + 2 * D * D) * sizeof(float);
}

// typical |entry| of a unit-Frobenius n-element matrix is n^-1/2: scale it to ~2
static float operand_scale(double n, float cap) {
  float sc = 256.f;
  while (sc < cap && sc * sc < 4.0 * n) sc *= 2.f;
  return sc;
}

// Polar Express on pre-split operands: per step A = X X^T (float32 A and split A),
// B = c A A + b A (split B only), X' = B X + a X (X' split, read K-major by the next Gram
// and MN-major by the next B X; a X read from the split of X).  The last step writes
// the result in the caller's orientation.
static cudaError_t launch_tma(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps,
                              void* ws, cudaStream_t s) {
  const int D = std::min(rows, cols), E = std::max(rows, cols);
  const size_t DE = (size_t)D * E, DD = (size_t)D * D;
  float* Af = (float*)ws;
  float* xf = Af + batch * DD;  // steps == 0 only
  __half* xs[2];
  xs[0] = (__half*)(xf + batch * DE);  // each split array is 2 x n halves = n floats of space
  xs[1] = xs[0] + 2 * batch * DE;
  __half* as = xs[1] + 2 * batch * DE;
  __half* bs = as + 2 * batch * DD;
  double* part = (double*)(bs + 2 * batch * DD);
  const float sx = operand_scale((double)DE, 16384.f), sa = operand_scale((double)DD, 16384.f),
              sbm = operand_scale((double)DD, 512.f);
  cudaError_t e =
      pet2::normalize_split(X, steps == 0 ? xf : nullptr, xs[0], nullptr, part, batch, rows, cols, eps, sx, s);
  if (e != cudaSuccess) return e;
  int* status = device_status_ptr();
  int cur = 0;
  for (int st = 0; st < steps; ++st) {
    const float ca = (float)kPEHost[st][0], cb = (float)kPEHost[st][1], cc = (float)kPEHost[st][2];
    const bool last = st + 1 == steps;
    pet2::EpiArgs g{};
    g.status = status;
    // A = X X^T (D x D, K = E)
    g.M = D; g.N = D; g.K = E;
    g.alpha = 1.f / (sx * sx); g.beta = 0.f; g.so = sa;
    g.Cf = Af; g.sC = DD; g.ldc = D; g.Cs = as;
    if ((e = pet2::gemm(xs[cur], xs[cur], g, batch, s)) != cudaSuccess) return e;
    // B = c A A + b A (A symmetric, so A itself is its K-major B operand)
    g = pet2::EpiArgs{};
    g.status = status;
    g.M = D; g.N = D; g.K = D;
    g.alpha = cc / (sa * sa); g.beta = cb; g.so = sbm;
    g.Dm = Af; g.sD = DD; g.ldd = D; g.Cs = bs;
    if ((e = pet2::gemm(as, as, g, batch, s)) != cudaSuccess) return e;
    // X' = B X + a X (D x E, K = D; B symmetric; X read MN-major as the B operand)
    g = pet2::EpiArgs{};
    g.status = status;
    g.M = D; g.N = E; g.K = D;
    g.alpha = 1.f / (sbm * sx); g.beta = ca; g.so = sx;
    g.Ds = xs[cur]; g.dscale_inv = 1.f / sx;
    if (last) {  // the result, in the caller's orientation
      g.Cf = rows > cols ? nullptr : Y;
      g.sC = DE; g.ldc = E;
      g.CfT = rows > cols ? Y : nullptr;
    } else {
      g.Cs = xs[cur ^ 1];
    }
    if ((e = pet2::gemm(bs, xs[cur], g, batch, s, true)) != cudaSuccess) return e;
    cur ^= 1;
  }
  if (steps > 0) return cudaSuccess;
  const size_t total = (size_t)batch * DE;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  pet::unwide_kernel<<<blocks, 256, 0, s>>>(xf, Y, batch, rows, cols);
  return cudaGetLastError();
}

// D = 64: the same three products with two matrices per 128-row tile (pe_tma.cu's packed
// mode): the Gram and A A keep the block diagonal of a 128 x 128 product, and
// B' = a I + b A + c A A times X runs as one K = 128 product of the block-diagonal
// [B'_z 0; 0 B'_z+1] with the stacked X's (the a X term rides in B', as in the fused scan).
static cudaError_t launch_packed(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps,
                                 void* ws, cudaStream_t s) {
  const int D = std::min(rows, cols), E = std::max(rows, cols);
  const size_t DE = (size_t)D * E, DD = (size_t)D * D;
  float* Af = (float*)ws;
  float* xf = Af + batch * DD;  // steps == 0 only
  __half* xs[2];
  xs[0] = (__half*)(xf + batch * DE);
  xs[1] = xs[0] + 2 * batch * DE;
  __half* as = xs[1] + 2 * batch * DE;
  __half* bpad = as + 2 * batch * DD;
  double* part = (double*)(bpad + 2 * batch * D * 128);
  const float sx = operand_scale((double)DE, 16384.f), sa = operand_scale((double)DD, 16384.f),
              sbm = operand_scale((double)DD, 512.f);
  cudaError_t e = pet2::normalize_split(X, steps == 0 ? xf : nullptr, xs[0], nullptr, part, batch, rows, cols, eps,
                                        sx, s, true);
  if (e != cudaSuccess) return e;
  int* status = device_status_ptr();
  int cur = 0;
  for (int st = 0; st < steps; ++st) {
    const float ca = (float)kPEHost[st][0], cb = (float)kPEHost[st][1], cc = (float)kPEHost[st][2];
    const bool last = st + 1 == steps;
    pet2::EpiArgs g{};
    g.status = status;
    g.pack = 128 / D;
    g.diag = 1;
    g.M = D; g.N = D; g.K = E;  // A = X X^T
    g.alpha = 1.f / (sx * sx); g.beta = 0.f; g.so = sa;
    g.Cf = Af; g.Cs = as;
    if ((e = pet2::gemm(xs[cur], xs[cur], g, batch, s)) != cudaSuccess) return e;
    g.Cf = nullptr; g.Cs = nullptr;
    g.K = D;  // B = c A A + b A, block-diagonal padded
    g.alpha = cc / (sa * sa); g.beta = cb; g.so = sbm;
    g.Dm = Af; g.Cpad = bpad;
    g.diag_add = ca;  // B' = a I + b A + c A A, so X' = B' X needs no addend
    if ((e = pet2::gemm(as, as, g, batch, s)) != cudaSuccess) return e;
    g = pet2::EpiArgs{};
    g.status = status;
    g.pack = 128 / D;
    g.diag = 0;
    g.M = D; g.N = E; g.K = 128;  // X' = B' X
    g.alpha = 1.f / (sbm * sx); g.so = sx;
    if (last) {
      g.Cf = rows > cols ? nullptr : Y;
      g.CfT = rows > cols ? Y : nullptr;
    } else {
      g.Cs = xs[cur ^ 1];
    }
    if ((e = pet2::gemm(bpad, xs[cur], g, batch, s, true)) != cudaSuccess) return e;
    cur ^= 1;
  }
  if (steps > 0) return cudaSuccess;
  const size_t total = (size_t)batch * DE;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  pet::unwide_kernel<<<blocks, 256, 0, s>>>(xf, Y, batch, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps, void* ws,
                   cudaStream_t s) {
  using pet::GemmArgs;
  if (pecl::usable(rows, cols)) return pecl::launch(X, Y, batch, rows, cols, steps, eps, s);
  if (pecta::usable(rows, cols)) return pecta::launch(X, Y, batch, rows, cols, steps, eps, s);
  if (pet2::usable(rows, cols)) return launch_tma(X, Y, batch, rows, cols, steps, eps, ws, s);
  if (pet2::usable_packed(rows, cols)) return launch_packed(X, Y, batch, rows, cols, steps, eps, ws, s);
  const int D = std::min(rows, cols), E = std::max(rows, cols);
  const size_t DE = (size_t)D * E, DD = (size_t)D * D;
  float* xa = (float*)ws;
  float* xb = xa + batch * DE;
  float* A = xb + batch * DE;
  float* Bm = A + batch * DD;
  for (int64_t z0 = 0; z0 < batch; z0 += 65535) {
    const int nz = (int)std::min<int64_t>(65535, batch - z0);
    pet::normalize_kernel<<<nz, 256, 0, s>>>(X + z0 * DE, xa + z0 * DE, rows, cols, eps);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int* status = device_status_ptr();
  const float sx = operand_scale((double)DE, 16384.f), sa = operand_scale((double)DD, 16384.f),
              sbm = operand_scale((double)DD, 512.f);
  for (int st = 0; st < steps; ++st) {
    GemmArgs g{};
    g.status = status;
    g.st = st;
    // A = X X^T  (D x D, K = E; B(n, k) = X[n][k])
    g.A = xa; g.sA = DE; g.lda = E;
    g.B = xa; g.sB = DE; g.ldb = E; g.b_kn = 0;
    g.C = A; g.sC = DD; g.ldc = D;
    g.Dm = nullptr; g.M = D; g.N = D; g.K = E; g.mode = 0;
    g.sa = sx; g.sb = sx;
    if ((e = pet::gemm(g, batch, s)) != cudaSuccess) return e;
    // B = c A A + b A  (A symmetric: B(n, k) = A[n][k])
    g.A = A; g.sA = DD; g.lda = D;
    g.B = A; g.sB = DD; g.ldb = D; g.b_kn = 0;
    g.C = Bm; g.sC = DD; g.ldc = D;
    g.Dm = A; g.sD = DD; g.ldd = D; g.M = D; g.N = D; g.K = D; g.mode = 1;
    g.sa = sa; g.sb = sa;
    if ((e = pet::gemm(g, batch, s)) != cudaSuccess) return e;
    // X' = B X + a X  (D x E, K = D; B(n, k) = X[k][n])
    g.A = Bm; g.sA = DD; g.lda = D;
    g.B = xa; g.sB = DE; g.ldb = E; g.b_kn = 1;
    g.C = xb; g.sC = DE; g.ldc = E;
    g.Dm = xa; g.sD = DE; g.ldd = E; g.M = D; g.N = E; g.K = D; g.mode = 2;
    g.sa = sbm; g.sb = sx;
    if ((e = pet::gemm(g, batch, s)) != cudaSuccess) return e;
    std::swap(xa, xb);
  }
  const size_t total = (size_t)batch * DE;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  pet::unwide_kernel<<<blocks, 256, 0, s>>>(xa, Y, batch, rows, cols);
  return cudaGetLastError();
}

}  // namespace tcpe
}  // namespace atlas
