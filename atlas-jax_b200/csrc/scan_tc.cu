// tcgen05 (sm_100a) Atlas scan, forward.
//
// Work decomposition
//   A (b, h) pair is a "chain" of chunks that must run in order.  A 2-CTA
//   cluster processes one (chain, chunk) item at a time: CTA rank 0 owns the
//   memory matrix W1 (and its momentum S1), rank 1 owns W2 / S2.  Items are
//   taken by a persistent grid of clusters from a ticket counter in chunk-major
//   order (ticket k -> chain k % NC, chunk k / NC), so a chain migrates between
//   clusters from chunk to chunk and every SM stays busy even when the number
//   of chains is not a multiple of the number of clusters.  The carry between
//   chunks goes through global memory (it is the `saved` buffer the backward
//   needs anyway); a per-chain counter released after the carry is written
//   orders the items of one chain.
//
// Per chunk (memory_layer.py:496-597)
//   * frozen-state pass on CUDA cores in float32, both CTAs reading the carry
//     from global memory: h = W2 k, act = gelu(h), err = k + W1 act - v and, on
//     rank 1, chain = (W1^T err) * gelu'(h).  Each CTA keeps the rank-1 factors
//     of its own per-token gradient: rank 0 u1^T = act err^T, rank 1 u2 = chain k^T.
//   * per token: S <- theta S - eta * (2/D) sum_{i in window} gamma_i f_i g_i^T in
//     float32 registers; X0 = S / (1.01 ||S|| + 1e-6); five Polar Express steps on
//     the tensor cores; W <- alpha W + X5; read-out y = q + W1 gelu(W2 q) with the
//     gelu(W2 q) vector exchanged through distributed shared memory.
//   * tokens go through Polar Express in pairs: two operand-tile sets and two TMEM
//     regions let one token's epilogue overlap the other token's MMAs.  A
//     dedicated producer warp issues every MMA (pe_produce); the 8 epilogue warps
//     (pe_consume) hand tiles to it through mbarriers.  The momentum / memory
//     recurrences stay in token order.
//
// Numerics: every Polar Express product runs on split fp16 operands (hi + lo of
// 256 x the value, ~22 significant bits; hi*hi + hi*lo + lo*hi, plus lo*lo in the
// stacked products, float32 accumulation in TMEM).  A single 16-bit pass is not
// enough: Polar Express amplifies noise in the near-null directions of the
// low-rank momentum by ~1e3.  With this split the scan's error matches the
// reference's own float32 arithmetic.
//
// Storage: each CTA keeps its matrix in the E x D orientation ("tile"): rank 0
// holds W1^T and S1^T, rank 1 holds W2 and S2.  Polar Express of the wide D x E
// matrix then reads  A = X~^T X~ (Gram over E),  X~' = X~ B'^T  with
// B' = a I + b A + c A^2.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "scan_internal.h"
#include "tc_ops.cuh"
#include "tc_common.cuh"

namespace atlas {
namespace tc {
using namespace tcx;

// Chunks of up to MAXCS_F tokens: a chunk longer than MAXCS runs its frozen pass in
// MAXCS-token parts (the frozen state is the chunk's entry carry for every part) and
// keeps its column factors in global scratch beside the row factors.
constexpr int MAXCS_F = 2 * MAXCS;

struct __align__(1024) Smem {
  uint8_t slot[2][NS_TILE_BYTES];  // per in-flight token: stacked X~, stacked A, B' hi/lo (frozen pass: scratch)
  float G[MAXCS * D];              // per-token column factor: err (rank 0) or k (rank 1), chunks <= MAXCS
  float gate[4][MAXCS_F];          // alpha, eta, theta, gamma
  float qv[D];
  float zbuf[2][E];
  float pbuf[2][E];                // gelu(W2 q) written by rank 1 into rank 0
  float ybuf[4][D];
  float red[8];
  uint64_t bar[2];    // done[s]: MMAs of slot s complete
  uint64_t ready[2];  // ready[s]: slot s operand tiles published by the 8 epilogue warps
  uint32_t tmem;
  int bad;
  int item;  // current work item (next_item)
};

__device__ __forceinline__ PESlot make_slot(Smem& s, int j, uint32_t tmem) {
  PESlot p;
  uint8_t* b = s.slot[j];
  p.Xh = b;
  p.Xl = b + XLO;
  p.Ah = b + 2 * XT_BYTES;
  p.Al = p.Ah + XLO;
  p.Bh = p.Ah + 2 * AT_BYTES;
  p.Bl = p.Bh + AT_BYTES;
  p.bar = &s.bar[j];
  p.tm = tmem + 256u * j;
  p.phase = 0;
  p.ns = nullptr;
  p.save_last = 0;
  return p;
}

// Carry slot entering chunk c of chain q: [matrix m][W, S][E x D tile].
__device__ __forceinline__ float* carry_slot(const FwdArgs& a, float* carries, int q, int c, int nch) {
  return a.saved ? (float*)a.saved + ((size_t)q * nch + c) * 4 * DE : carries + (size_t)q * 4 * DE;
}

// Frozen-state pass of one chunk (memory_layer.py:504-520), float32 CUDA cores.
// Writes this CTA's row factor (act on rank 0, chain on rank 1) to Fg (cs x E,
// global scratch) and its column factor (err / k) to s.G, or to Gg (cs x D, global
// scratch) when the chunk is longer than MAXCS; such a chunk is processed in parts of
// MAXCS tokens, all against the chunk's entry carry.
template <typename TA>
__device__ void frozen_pass(const FwdArgs& a, Smem& s, const float* slot, float* Fg, float* Gg, int b, int hh,
                            int c, int cs, uint32_t rank) {
  const AtlasScanParams& P = a.p;
  const int T = P.T, H = P.H;
  const TA* kp = (const TA*)a.k;
  const TA* vp = (const TA*)a.v;
  const float* W1t = slot;            // W1^T: [e][d]
  const float* W2 = slot + 2 * DE;    // W2:   [e][d]
  float* actb = (float*)s.slot[0];                     // E x MAXCS, tsw layout (64 KB)
  float* kbuf = (float*)s.slot[1];                     // cs x D  (16 KB)
  float* errb = (float*)(s.slot[1] + MAXCS * D * 4);   // cs x D  (16 KB)
  float* W1s = (float*)(s.slot[1] + 2 * MAXCS * D * 4); // W1^T staged (64 KB)
  const int tid = threadIdx.x;
  const uint64_t pol = l2_evict_last_policy();  // Fg is re-read by every token of the chunk
  for (int i = tid; i < DE / 4; i += NT) ((float4*)W1s)[i] = ((const float4*)W1t)[i];
  for (int r = tid; r < cs; r += NT) {
    Gates g = load_gates(a.alpha, a.eta, a.theta, a.gamma, T, H, b, hh, c * cs + r);
    s.gate[0][r] = g.a;
    s.gate[1][r] = g.e;
    s.gate[2][r] = g.t;
    s.gate[3][r] = g.g;
  }
  for (int rb = 0; rb < cs; rb += MAXCS) {  // parts of at most MAXCS tokens
  const int n = min(MAXCS, cs - rb);
  float* Fp = Fg + (size_t)rb * E;
  for (int i = tid; i < n * D; i += NT) {
    int r = i / D, d = i % D, t = c * cs + rb + r;
    kbuf[i] = t < T ? ld_act(kp, (((size_t)b * T + t) * H + hh) * D + d) : 0.f;
  }
  epi_sync();
  {  // h = W2 k ; thread e
    const int e = tid;
    float w[D];
#pragma unroll
    for (int d = 0; d < D; ++d) w[d] = W2[e * D + d];
    for (int r = 0; r < n; ++r) {
      float hv = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) hv = fmaf(w[d], kbuf[r * D + d], hv);
      const float av = gelu_tanh(hv);
      actb[tsw(e, r)] = av;
      st_hint(&Fp[r * E + e], rank ? hv : av, pol);  // rank 1 keeps h for gelu'(h)
    }
  }
  epi_sync();
  {  // err = k + W1 act - v ; 4 x 4 (token x d) tile per thread
    const int dq = tid & 15, iq = tid >> 4;
    float acc[4][4];
    tile_tok_d(W1s, actb, dq, iq, acc);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = 4 * iq + u, t = c * cs + rb + r;
      if (r < n)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int d = 4 * dq + v;
          const float vv = t < T ? ld_act(vp, (((size_t)b * T + t) * H + hh) * D + d) : 0.f;
          errb[r * D + d] = kbuf[r * D + d] + acc[u][v] - vv;
        }
    }
  }
  epi_sync();
  if (rank) {  // chain = (W1^T err) * gelu'(h) ; thread e
    const int e = tid;
    float w[D];
#pragma unroll
    for (int d = 0; d < D; ++d) w[d] = W1t[e * D + d];
    for (int r = 0; r < n; ++r) {
      float rv = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) rv = fmaf(w[d], errb[r * D + d], rv);
      st_hint(&Fp[r * E + e], rv * gelu_erf_prime(Fp[r * E + e]), pol);
    }
  }
  float* Gd = Gg ? Gg + (size_t)rb * D : s.G;
  for (int i = tid; i < n * D; i += NT) Gd[i] = rank ? kbuf[i] : errb[i];
  epi_sync();
  }  // parts
}

size_t bwd_workspace_bytes(const AtlasScanParams& p);

struct KArgs {
  FwdArgs a;
  int nchains, nch;
  float* carries;  // used when a.saved == nullptr: one slot per chain
  int* flags;      // chunks completed per chain (zeroed before launch)
  int* ticket;     // next work item (zeroed before launch)
  WaitHooks hooks;
  float* fscr;     // per cluster, per rank: the chunk's row factors (cs x E) [, column factors (cs x D)]
  size_t fstride;  // floats of fscr per cluster rank
};

#ifdef ATLAS_PHASE_PROF
__device__ unsigned long long g_prof_fwd[32];
#endif

// LONGC: chunks longer than MAXCS (column factors in global scratch)
template <typename TA, bool LONGC>
__global__ void __launch_bounds__(NT + 128, 1) fwd_kernel(KArgs K) {
  PROF_DECL
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const FwdArgs& a = K.a;
  const AtlasScanParams& P = a.p;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int qd = w & 3, ch = w >> 2;
  const int e0 = 32 * qd + l, e1 = e0 + 128, dc = 32 * ch;
  const uint32_t rank = cluster_rank();
  const int cluster = blockIdx.x >> 1;  // indexes this cluster's scratch
  const int cs = P.chunk, T = P.T, H = P.H, nch = K.nch;
  const float sc = 2.0f / D;
  const bool win = P.omega > 1;
  const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
  float* Fg = K.fscr + ((size_t)cluster * 2 + rank) * K.fstride;
  float* Gg = LONGC ? Fg + (size_t)MAXCS_F * E : nullptr;  // column factors of a long chunk
  const float* Gsrc = LONGC ? Gg : s.G;

  if (w == 0) {
    tmem_alloc(&s.tmem, TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.bar[0], 1);  // done[0]
    mbar_init(&s.bar[1], 1);  // done[1]
    mbar_init(&s.ready[0], 8);
    mbar_init(&s.ready[1], 8);
    fence_mbar_init();
    s.bad = 0;
  }
  fence_before();
  __syncthreads();
  fence_after();
  PESlot sl[2] = {make_slot(s, 0, s.tmem), make_slot(s, 1, s.tmem)};
  PEBars B;
  B.ready[0] = &s.ready[0];
  B.ready[1] = &s.ready[1];
  B.done[0] = &s.bar[0];
  B.done[1] = &s.bar[1];
  B.ready_phase[0] = B.ready_phase[1] = B.done_phase[0] = B.done_phase[1] = 0;
  PROF_INIT
  const long total = (long)K.nchains * nch;
  const int npair = P.ns_steps > 0 ? 2 : 1;

  // Register split (launch: 384 threads x 168 = 64512): the two epilogue
  // warpgroups take 240 each, the producer warpgroup keeps 24:
  // 2 * 128 * 240 + 128 * 24 = 64512.
  if (w >= 8) {  // ---- producer warpgroup: warp 8 issues every MMA; all four mirror the cluster barriers ----
    asm volatile("setmaxnreg.dec.sync.aligned.u32 24;");
    for (;;) {
      const long k = next_item(K.ticket, &s.item);
      if (k >= total) break;
      cluster_sync();
      cluster_sync();
      for (int r0 = 0; r0 < cs; r0 += npair) {
        const int n = min(npair, cs - r0);
        if (w == 8 && P.ns_steps > 0) pe_produce(sl, B, n, P.ns_steps, &s.bad);
        for (int j = 0; j < n; ++j) cluster_sync();
      }
      cluster_sync();
    }
  } else {  // ---- 8 epilogue warps ----
  asm volatile("setmaxnreg.inc.sync.aligned.u32 240;");
  float Sv[2][32], Wv[2][32];
  for (;;) {
    const long k = next_item(K.ticket, &s.item);
    if (k >= total) break;
    const int q = (int)(k % K.nchains), c = (int)(k / K.nchains);
    const int b = q / H, hh = q % H;
    PROF_T(titem)
    PROF_T(twait)
    // ---- wait for the previous chunk of this chain ----
    if (c > 0 && tid == 0 && !s.bad) {
      int spins = 0;
      while (ld_acquire(&K.flags[q]) < c + K.hooks.flag_bias) {
        __nanosleep(200);
        if (++spins > K.hooks.spin_limit) {
          set_status(a.status, ATLAS_ERR_DEVICE_TIMEOUT);
          s.bad = 1;
          break;
        }
      }
    }
    epi_sync();
    PROF_ADD(13, twait)
    float* slot = carry_slot(a, K.carries, q, c, nch);
    float* mine = slot + 2 * rank * DE;  // [W, S] of this CTA's matrix
    if (c == 0) {  // initial carry: caller's state or the LM init (model.py:251-264)
      for (int i = tid; i < DE; i += NT) {
        int e = i / D, d = i % D;
        size_t bh = (size_t)q * DE;
        float wv, sv;
        if (rank == 0) {  // W1, S1 are (D, E): tile holds the transpose
          wv = a.W1_in ? a.W1_in[bh + (size_t)d * E + e] : 0.f;
          sv = a.S1_in ? a.S1_in[bh + (size_t)d * E + e] : 0.f;
        } else {
          wv = a.W2_in ? a.W2_in[bh + i] : (e == d ? 1.f : 0.f);
          sv = a.S2_in ? a.S2_in[bh + i] : 0.f;
        }
        mine[i] = wv;
        mine[DE + i] = sv;
      }
      __threadfence();
    }
    cluster_sync();
    PROF_T(tfz)
    frozen_pass<TA>(a, s, slot, Fg, Gg, b, hh, c, cs, rank);
    PROF_ADD(5, tfz)
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      Wv[0][j] = mine[e0 * D + dc + j];
      Wv[1][j] = mine[e1 * D + dc + j];
      Sv[0][j] = mine[DE + e0 * D + dc + j];
      Sv[1][j] = mine[DE + e1 * D + dc + j];
    }
    cluster_sync();  // both CTAs are done reading the carry slot

    for (int r0 = 0; r0 < cs; r0 += npair) {
      PROF_T(tpair)
      const int n = min(npair, cs - r0);
      float inv0 = 0.f;
      float Gv[2][32];  // Omega-window gradient sum, slid from the pair's first token to its second
      for (int j = 0; j < n; ++j) {
        PROF_T(ttok)
        const int r = r0 + j;
        const float et = s.gate[1][r], th = s.gate[2][r];
        // ---- momentum: S <- theta S - eta * s * sum_i gamma_i f_i g_i^T ----
        window_sum(Gv, Fg, Gsrc, s.gate[3], r, P.omega, win, j > 0, e0, e1, dc);
        const float wg = -et * sc;
        axpby<32>(Sv[0], th, Gv[0], wg);
        axpby<32>(Sv[1], th, Gv[1], wg);
        PROF_ADD(2, ttok)
        PROF_T(tnorm)
        // ---- Frobenius normalisation (memory_layer.py:55-56) ----
        float ss = 0.f;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) ss = fmaf(Sv[0][jj], Sv[0][jj], fmaf(Sv[1][jj], Sv[1][jj], ss));
        ss = block_sum_epi(ss, s.red);
        const float inv = 1.0f / (sqrtf(ss + 1e-12f) * 1.01f + 1e-6f);
        inv0 = inv;
        if (P.ns_steps > 0) {
          float xv[32];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) xv[jj] = Sv[0][jj] * inv;
          store_stk<32>(sl[j].Xh, e0, dc, xv);
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) xv[jj] = Sv[1][jj] * inv;
          store_stk<32>(sl[j].Xh, e1, dc, xv);
        }
        PROF_ADD(3, tnorm)
      }
      // q of the pair, loaded before Polar Express so the read-out does not wait on it
      float pq[2] = {0.f, 0.f};
      if (tid < D)
        for (int j = 0; j < n; ++j) {
          const int t = c * cs + r0 + j;
          if (t < T) pq[j] = ld_act((const TA*)a.q, (((size_t)b * T + t) * H + hh) * D + tid);
        }
      // ---- Polar Express (memory_layer.py:43-71) for the pair, interleaved ----
      if (P.ns_steps > 0 && !pe_consume(sl, B, n, P.ns_steps, &s.bad, PROF_PTR) && !s.bad) {
        set_status(a.status, ATLAS_ERR_DEVICE_TIMEOUT);
        s.bad = 1;
      }
      for (int j = 0; j < n; ++j) {
        PROF_T(tro)
        const int r = r0 + j, t = c * cs + r;
        const float al = s.gate[0][r];
        if (P.ns_steps > 0) {
          float x0[32], x1[32];
          tmem_ld32(sl[j].tm + lane_off + TM_X + dc, x0);
          tmem_ld32(sl[j].tm + lane_off + TM_X + 64 + dc, x1);
          tmem_wait_ld();
          axpby<32>(Wv[0], al, x0, KUNSC2);  // TMEM holds KSPLIT^2 X_ns
          axpby<32>(Wv[1], al, x1, KUNSC2);
        } else {  // PE with zero steps is the normalisation alone
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            Wv[0][jj] = al * Wv[0][jj] + Sv[0][jj] * inv0;
            Wv[1][jj] = al * Wv[1][jj] + Sv[1][jj] * inv0;
          }
        }
        // ---- read-out y = q + W1 gelu(W2 q)  (memory_layer.py:592-595) ----
        if (tid < D) s.qv[tid] = j ? pq[1] : pq[0];
        epi_sync();
        if (rank == 1) {
          float z0 = 0.f, z1 = 0.f;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            z0 = fmaf(Wv[0][jj], s.qv[dc + jj], z0);
            z1 = fmaf(Wv[1][jj], s.qv[dc + jj], z1);
          }
          s.zbuf[ch][e0] = z0;
          s.zbuf[ch][e1] = z1;
          epi_sync();
          const float z = s.zbuf[0][tid] + s.zbuf[1][tid];
          st_remote_f32(&s.pbuf[r & 1][tid], 0, gelu_tanh(z));
          cluster_sync();
        } else {
          cluster_sync();
          const float p0 = s.pbuf[r & 1][e0], p1 = s.pbuf[r & 1][e1];
          float yv[32];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) yv[jj] = fmaf(Wv[0][jj], p0, Wv[1][jj] * p1);
          float part = warp_reduce_scatter32(yv);
          s.ybuf[qd][dc + l] = part;
          epi_sync();
          if (tid < D && t < T) {
            float y = s.qv[tid] + s.ybuf[0][tid] + s.ybuf[1][tid] + s.ybuf[2][tid] + s.ybuf[3][tid];
            st_act((TA*)a.y, (((size_t)b * T + t) * H + hh) * D + tid, y);
          }
        }
        epi_sync();
        PROF_ADD(6, tro)
      }
      PROF_ADD(4, tpair)
    }
    // ---- carry out ----
    if (c + 1 < nch) {
      float* nxt = carry_slot(a, K.carries, q, c + 1, nch) + 2 * rank * DE;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        nxt[e0 * D + dc + j] = Wv[0][j];
        nxt[e1 * D + dc + j] = Wv[1][j];
        nxt[DE + e0 * D + dc + j] = Sv[0][j];
        nxt[DE + e1 * D + dc + j] = Sv[1][j];
      }
    } else {
      const size_t bh = (size_t)q * DE;
      float* Wo = rank ? a.W2_out : a.W1_out;
      float* So = rank ? a.S2_out : a.S1_out;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int e = h2 ? e1 : e0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int d = dc + j;
          const size_t o = rank ? bh + (size_t)e * D + d : bh + (size_t)d * E + e;
          if (Wo) Wo[o] = Wv[h2][j];
          if (So) So[o] = Sv[h2][j];
        }
      }
    }
    __threadfence();
    cluster_sync();
    if (rank == 0 && tid == 0) st_release(&K.flags[q], c + 1);
    PROF_ADD(14, titem)
  }
  }  // epilogue warps
  fence_before();
  __syncthreads();
  if (w == 0) tmem_dealloc(s.tmem, TMEM_COLS);
  PROF_FLUSH(g_prof_fwd)
}

// ---- host side ----------------------------------------------------------------
bool supported(const AtlasScanParams& p, const char** why) {
  if (p.D != D || p.E != E) {
    *why = "tcgen05 path is built for head_dim 64, memory hidden 256";
    return false;
  }
  if (p.chunk > MAXCS) {
    *why = "tcgen05 backward supports chunk <= 64";
    return false;
  }
  return true;
}
bool supported_fwd(const AtlasScanParams& p, const char** why) {
  if (p.D != D || p.E != E) {
    *why = "tcgen05 path is built for head_dim 64, memory hidden 256";
    return false;
  }
  if (p.chunk > MAXCS_F) {
    *why = "tcgen05 forward supports chunk <= 128";
    return false;
  }
  return true;
}
size_t saved_bytes(const AtlasScanParams& p) { return (size_t)p.B * p.H * n_chunks(p) * 4 * DE * sizeof(float); }

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// per-chain completion counters, then the item ticket
static size_t flags_bytes(const AtlasScanParams& p) { return align256(((size_t)p.B * p.H + 1) * sizeof(int)); }
static size_t fwd_clusters(const AtlasScanParams& p) {
  return std::min((size_t)p.B * p.H, (size_t)max_clusters_bound());
}
// factor scratch per cluster rank: row factors, plus column factors for chunks > MAXCS
static size_t fscr_floats(const AtlasScanParams& p) {
  return p.chunk > MAXCS ? (size_t)MAXCS_F * (E + D) : (size_t)MAXCS * E;
}
size_t fwd_workspace_bytes(const AtlasScanParams& p) {
  return flags_bytes(p) + (size_t)p.B * p.H * 4 * DE * sizeof(float) +
         fwd_clusters(p) * 2 * fscr_floats(p) * sizeof(float);
}
size_t workspace_bytes(const AtlasScanParams& p) {
  // one buffer serves the forward and the backward (chunks > MAXCS are forward-only)
  if (p.chunk > MAXCS) return fwd_workspace_bytes(p);
  return std::max(fwd_workspace_bytes(p), bwd_workspace_bytes(p));
}

static DeviceCache g_max_clusters;  // resident 2-CTA clusters, per device

template <typename TA, bool LONGC>
static cudaError_t launch_fwd_t(const KArgs& k, int nclusters, cudaStream_t st) {
  size_t smem = sizeof(Smem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(fwd_kernel<TA, LONGC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(NT + 128);  // 8 epilogue warps + a producer warpgroup (1 MMA warp, 3 idle)
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int maxc = g_max_clusters.get([&] {
    int n = 0;
    cfg.gridDim = dim3(2);
    if (cudaOccupancyMaxActiveClusters(&n, fwd_kernel<TA, LONGC>, &cfg) != cudaSuccess || n <= 0) n = 1;
    return n;
  });
  cfg.gridDim = dim3(2 * std::min(nclusters, maxc));
  return cudaLaunchKernelEx(&cfg, fwd_kernel<TA, LONGC>, k);
}

cudaError_t launch_fwd(const FwdArgs& a, cudaStream_t st) {
  KArgs k;
  k.a = a;
  k.nchains = a.p.B * a.p.H;
  k.nch = n_chunks(a.p);
  k.hooks = wait_hooks();
  uint8_t* ws = (uint8_t*)a.ws;
  k.flags = (int*)ws;
  k.ticket = k.flags + k.nchains;
  k.carries = (float*)(ws + flags_bytes(a.p));
  k.fscr = k.carries + (size_t)k.nchains * 4 * DE;
  k.fstride = fscr_floats(a.p);
  cudaError_t e = cudaMemsetAsync(k.flags, 0, flags_bytes(a.p), st);
  if (e != cudaSuccess) return e;
  const int ncl = (int)fwd_clusters(a.p);
  if (a.p.chunk > MAXCS)
    return a.p.act_dtype == ATLAS_BF16 ? launch_fwd_t<__nv_bfloat16, true>(k, ncl, st)
                                       : launch_fwd_t<float, true>(k, ncl, st);
  return a.p.act_dtype == ATLAS_BF16 ? launch_fwd_t<__nv_bfloat16, false>(k, ncl, st)
                                     : launch_fwd_t<float, false>(k, ncl, st);
}

}  // namespace tc
}  // namespace atlas

#ifdef ATLAS_PHASE_PROF
// Instrumented builds only: read and clear the forward kernel's phase cycle counters.
extern "C" int atlas_debug_prof_fwd(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, atlas::tc::g_prof_fwd, 32 * sizeof(unsigned long long));
  unsigned long long z[32] = {};
  return cudaMemcpyToSymbol(atlas::tc::g_prof_fwd, z, sizeof(z)) == cudaSuccess ? 0 : 3;
}
#endif
