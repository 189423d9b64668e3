// tcgen05 (sm_100a) batched Polar Express for large matrices: the Muon
// orthogonalisation of stacked parameter gradients (atlas_jax/optim.py:56-108,
// Polar Express at 68-83; same iteration as memory_layer.py:43-71), e.g. the 170M
// model's (12, 768, 768), (12, 4096, 768), (12, 768, 2048) stacks.
//
// Matrices are held "wide" (D = min(rows, cols) rows, E = max columns; tall inputs
// are transposed on the way in and out), so every step is
//   A = X X^T,   B = b A + c A A,   X <- a X + B X
// as three launches of one batched GEMM kernel.  The GEMM reads float32 operands,
// splits them into bf16 hi/lo parts while staging them in shared memory, and
// accumulates hi*hi + hi*lo + lo*hi on the tensor cores in float32 in TMEM (about 16
// mantissa bits per operand; a single bf16 pass loses the near-null directions that
// Polar Express amplifies).  The epilogue fuses alpha * product + beta * addend.
//
// GEMM kernel: one CTA of 4 warps per 128 x 128 output tile and batch entry; K in
// chunks of 32, two shared-memory stages (the next chunk's global loads are in
// flight while the current chunk's MMAs run); one elected thread issues the MMAs
// and commits them to the stage's mbarrier; every wait is bounded and records
// ATLAS_ERR_DEVICE_TIMEOUT instead of hanging.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "scan_internal.h"
#include "tc_ops.cuh"

namespace atlas {
namespace pet {
using namespace tcx;

constexpr int TM = 128, TN = 128, TK = 32, NTH = 128;
constexpr int TILE = 128 * TK * 2;  // bytes of one bf16 128 x 32 (or 32 x 128) tile

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
  int* status;
};

__device__ __forceinline__ void ld_row32(const float* p, int valid, bool vec, float* v) {
  if (vec && valid >= 32) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 x = ((const float4*)p)[j];
      v[4 * j] = x.x; v[4 * j + 1] = x.y; v[4 * j + 2] = x.z; v[4 * j + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = j < valid ? p[j] : 0.f;
  }
}

__device__ __forceinline__ void split8(uint8_t* th, uint8_t* tl, uint32_t off, const float* v) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    const uint32_t hb = *reinterpret_cast<uint32_t*>(&hv);
    const float r0 = v[2 * k] - __uint_as_float(hb << 16);
    const float r1 = v[2 * k + 1] - __uint_as_float(hb & 0xFFFF0000u);
    __nv_bfloat162 lv = __floats2bfloat162_rn(r0, r1);
    h[k] = hb;
    l[k] = *reinterpret_cast<uint32_t*>(&lv);
  }
  *(uint4*)(th + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *(uint4*)(tl + off) = make_uint4(l[0], l[1], l[2], l[3]);
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
  float ra[32], rb[32];
  auto load = [&](int i) {
    const int k0 = i * TK;
    const int m = m0 + t;
    if (m < g.M)
      ld_row32(A + (size_t)m * g.lda + k0, g.K - k0, vecA, ra);
    else
#pragma unroll
      for (int j = 0; j < 32; ++j) ra[j] = 0.f;
    if (!g.b_kn) {  // row n of B, k0..k0+31
      const int n = n0 + t;
      if (n < g.N)
        ld_row32(Bp + (size_t)n * g.ldb + k0, g.K - k0, vecB, rb);
      else
#pragma unroll
        for (int j = 0; j < 32; ++j) rb[j] = 0.f;
    } else {  // row k of B, 32 columns of n
      const int k = k0 + (t >> 2), nc = n0 + 32 * (t & 3);
      if (k < g.K)
        ld_row32(Bp + (size_t)k * g.ldb + nc, g.N - nc, vecB, rb);
      else
#pragma unroll
        for (int j = 0; j < 32; ++j) rb[j] = 0.f;
    }
  };
  const uint32_t idesc = idesc_bf16(128, 128, false, g.b_kn != 0);
  load(0);
  for (int i = 0; i < nk; ++i) {
    const int st = i & 1;
    if (i >= 2 && !s.bad && !mbar_wait(&s.bar[st], ((i - 2) >> 1) & 1)) {  // MMAs of chunk i-2 read this stage
      s.bad = 1;
      set_status(g.status, ATLAS_ERR_DEVICE_TIMEOUT);
    }
    uint8_t *ah = s.a[st][0], *al = s.a[st][1], *bh = s.b[st][0], *bl = s.b[st][1];
#pragma unroll
    for (int j = 0; j < 4; ++j) split8(ah, al, cm_off(t, 8 * j, TK), ra + 8 * j);
    if (!g.b_kn) {
#pragma unroll
      for (int j = 0; j < 4; ++j) split8(bh, bl, cm_off(t, 8 * j, TK), rb + 8 * j);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) split8(bh, bl, cm_off(t >> 2, 32 * (t & 3) + 8 * j, TN), rb + 8 * j);
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    if (i + 1 < nk) load(i + 1);  // next chunk's global loads overlap this chunk's MMAs
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
          mma_bf16(tm, da[ta[term]] + ks * sa, db[tb[term]] + ks * sb, idesc, (i || term || ks) ? 1u : 0u);
      mma_commit(&s.bar[st]);
    }
  }
  // the last commit covers every MMA of the tile
  if (!s.bad && !mbar_wait(&s.bar[(nk - 1) & 1], ((nk - 1) >> 1) & 1)) {
    s.bad = 1;
    set_status(g.status, ATLAS_ERR_DEVICE_TIMEOUT);
  }
  fence_after();
  float alpha = 1.f, beta = 0.f;
  if (g.mode == 1) {
    alpha = (float)kPE[g.st][2];
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
  static bool attr_set = false;
  const size_t smem = sizeof(Smem) + 1024;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
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

size_t workspace_bytes(int64_t batch, int rows, int cols) {
  const size_t D = std::min(rows, cols), DE = (size_t)rows * cols;
  return (size_t)batch * (2 * DE + 2 * D * D) * sizeof(float);
}

cudaError_t launch(const float* X, float* Y, int64_t batch, int rows, int cols, int steps, float eps, void* ws,
                   cudaStream_t s) {
  using pet::GemmArgs;
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
  for (int st = 0; st < steps; ++st) {
    GemmArgs g{};
    g.status = status;
    g.st = st;
    // A = X X^T  (D x D, K = E; B(n, k) = X[n][k])
    g.A = xa; g.sA = DE; g.lda = E;
    g.B = xa; g.sB = DE; g.ldb = E; g.b_kn = 0;
    g.C = A; g.sC = DD; g.ldc = D;
    g.Dm = nullptr; g.M = D; g.N = D; g.K = E; g.mode = 0;
    if ((e = pet::gemm(g, batch, s)) != cudaSuccess) return e;
    // B = c A A + b A  (A symmetric: B(n, k) = A[n][k])
    g.A = A; g.sA = DD; g.lda = D;
    g.B = A; g.sB = DD; g.ldb = D; g.b_kn = 0;
    g.C = Bm; g.sC = DD; g.ldc = D;
    g.Dm = A; g.sD = DD; g.ldd = D; g.M = D; g.N = D; g.K = D; g.mode = 1;
    if ((e = pet::gemm(g, batch, s)) != cudaSuccess) return e;
    // X' = B X + a X  (D x E, K = D; B(n, k) = X[k][n])
    g.A = Bm; g.sA = DD; g.lda = D;
    g.B = xa; g.sB = DE; g.ldb = E; g.b_kn = 1;
    g.C = xb; g.sC = DE; g.ldc = E;
    g.Dm = xa; g.sD = DE; g.ldd = E; g.M = D; g.N = E; g.K = D; g.mode = 2;
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
