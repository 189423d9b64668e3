// TMA-fed tcgen05 GEMM over pre-split fp16 hi / lo operands (pe_tma.cu), used by the
// batched Polar Express for matrices whose short side is >= 128.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace atlas {
namespace pet2 {

// C = alpha * sum_k A[m][k] B[n][k] + beta * Dm[m][n] for every batch entry, with A and B
// given as split arrays [batch][hi, lo][rows][K] (K-major, rows M resp. N; B may also be
// MN-major, see gemm()).  Outputs (each
// may be null): Cf float32 (ldc, batch stride sC); Cs split [batch][part][M][N] and
// Ct split [batch][part][N][M], both of so * C.
struct EpiArgs {
  int M, N, K;
  float alpha, beta, so;
  const float* Dm;
  int64_t sD;
  int ldd;
  const __half* Ds;  // addend as a split [batch][part][M][N] of dscale * Dm (used when Dm is null)
  float dscale_inv;
  float* Cf;
  int64_t sC;
  int ldc;
  __half* Cs;
  __half* Ct;
  float* CfT;  // float32 transposed [batch][N][M]
  int* status;
  // Packed mode for matrices of D = 128 / pack rows (pack > 0): operands are split
  // arrays [part][batch * rows][K] and tiles hold `pack` matrices.  diag: the product of
  // each matrix with itself over K (A = X X^T, A A), keeping the block diagonal; M = N = D.
  // Otherwise the row product X' = B X: A is the block-diagonal padded B (K = 128),
  // B is X read MN-major, M = D, N = E.  Cpad: packed block-diagonal output (row length 128).
  int pack, diag;
  __half* Cpad;
  float diag_add;  // added to the diagonal of each D x D block (diagonal products)
};

bool usable(int rows, int cols);
bool usable_packed(int rows, int cols);  // D = 64: two matrices per 128-row tile
// b_mn: B given as a split array [batch][part][K][N] (MN-major) instead of [batch][part][N][K]
cudaError_t gemm(const __half* As, const __half* Bs, const EpiArgs& g, int64_t batch, cudaStream_t s,
                 bool b_mn = false);
// Frobenius normalisation of the Polar Express input, X = S / (1.01 sqrt(sum S^2 + eps) + 1e-6),
// S given as rows x cols (wide X = S, tall X = S^T, D x E): writes X as float32 (Xf, may be
// null) and as splits of sx * X, row-major (Xs, D x E) and transposed (Xt, E x D; may be null).  part: batch * 64
// doubles of scratch.  packed: Xs as [part][batch * D][E] (pe_tma's packed mode).
cudaError_t normalize_split(const float* S, float* Xf, __half* Xs, __half* Xt, double* part, int64_t batch, int rows,
                            int cols, float eps, float sx, cudaStream_t s, bool packed = false);

}  // namespace pet2
}  // namespace atlas
