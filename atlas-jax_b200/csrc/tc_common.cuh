// Shared pieces of the tcgen05 scan kernels (forward and backward).
#pragma once
#include <cuda_bf16.h>

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
constexpr int XT_BYTES = E * D * 2;  // bf16 E x D tile
constexpr int AT_BYTES = D * D * 2;  // bf16 D x D tile
constexpr int TMEM_COLS = 512;  // two in-flight problems of 256 columns each
// TMEM column map
constexpr uint32_t TM_X = 0;      // X~ update: rows 0-127 in cols [0,64), rows 128-255 in [64,128)
constexpr uint32_t TM_GRAM = 128; // Gram A (M=64 layout)
constexpr uint32_t TM_A2 = 192;   // A*A    (M=64 layout)

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
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Split 8 consecutive float32 values into bf16 hi and lo parts and store them
// as one 16-byte core-matrix row segment in each tile.
__device__ __forceinline__ void store_split8(uint8_t* th, uint8_t* tl, uint32_t off, const float* v) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    // packed conversions (one cvt.rn.bf16x2.f32 per pair); bf16 -> f32 is a bit shift
    __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    uint32_t hb = *reinterpret_cast<uint32_t*>(&hv);
    float r0 = v[2 * k] - __uint_as_float(hb << 16);
    float r1 = v[2 * k + 1] - __uint_as_float(hb & 0xFFFF0000u);
    __nv_bfloat162 lv = __floats2bfloat162_rn(r0, r1);
    h[k] = hb;
    l[k] = *reinterpret_cast<uint32_t*>(&lv);
  }
  *(uint4*)(th + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *(uint4*)(tl + off) = make_uint4(l[0], l[1], l[2], l[3]);
}
// 32 consecutive columns [c0, c0+32) of row r of a tile with C columns.
__device__ __forceinline__ void store_split32(uint8_t* th, uint8_t* tl, int r, int c0, int C, const float* v) {
#pragma unroll
  for (int k = 0; k < 4; ++k) store_split8(th, tl, cm_off(r, c0 + 8 * k, C), v + 8 * k);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + 16, v + 16);
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

// Three-term split product into TMEM column `tmd`:
//   D (+)= Ah*Bh + Ah*Bl + Al*Bh   (M x 64, contraction length K)
// Operand tiles have 64 columns (core-matrix tiles of C = 64).  amn / bmn pick
// the MN-major view (rows = K index) instead of the K-major view (rows = M/N).
// a_off is a byte offset into the A tiles (selects the 128-row half for M = 128).
// Descriptors are built once per term; stepping K by 16 adds to the 14-bit
// start-address field (shared-memory addresses < 256 KB never carry out of it).
template <int K>
__device__ __forceinline__ void mma3(uint32_t tmd, const uint8_t* ah, const uint8_t* al, bool amn,
                                     const uint8_t* bh, const uint8_t* bl, bool bmn, int M, uint32_t a_off,
                                     bool accumulate) {
  const uint32_t id = idesc_bf16(M, 64, amn, bmn);
  const uint64_t sa = amn ? (2048 >> 4) : (256 >> 4);
  const uint64_t sb = bmn ? (2048 >> 4) : (256 >> 4);
  const uint8_t* ta[3] = {ah, ah, al};
  const uint8_t* tb[3] = {bh, bl, bh};
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const uint32_t aa = smem_u32(ta[t]) + a_off, bb = smem_u32(tb[t]);
    const uint64_t da = amn ? desc_mnmajor(aa, 64) : desc_kmajor(aa, 64);
    const uint64_t db = bmn ? desc_mnmajor(bb, 64) : desc_kmajor(bb, 64);
#pragma unroll
    for (int ks = 0; ks < K / 16; ++ks)
      mma_bf16(tmd, da + ks * sa, db + ks * sb, id, (accumulate || t || ks) ? 1u : 0u);
  }
}

// Optional phase timers (build with -DATLAS_PHASE_PROF; thread 0 accumulates
// clock64() deltas into a shared array; off in the product build).
#ifdef ATLAS_PHASE_PROF
#define PROF_DECL __shared__ unsigned long long s_prof[16];
#define PROF_INIT if (threadIdx.x < 16) s_prof[threadIdx.x] = 0;
#define PROF_T(v) long long v = clock64();
#define PROF_ADD(slot, v) if (threadIdx.x == 0) s_prof[slot] += clock64() - v;
#define PROF_PTR s_prof
#define PROF_FLUSH(g) if (threadIdx.x < 16) atomicAdd(&g[threadIdx.x], s_prof[threadIdx.x]);
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
struct PESlot {
  uint8_t *Xh, *Xl, *Ah, *Al, *Bh, *Bl;
  uint64_t* bar;
  uint32_t tm;       // TMEM base of this slot: X~ at +TM_X (+64), Gram at +TM_GRAM, A*A at +TM_A2
  uint32_t phase;
  uint8_t* ns;       // global destination of step k's tiles at ns + k * NS_TILE_BYTES, or null
  int save_last;     // unused (every step is saved when ns is set)
};
constexpr size_t NS_TILE_BYTES = 2 * XT_BYTES + 4 * AT_BYTES;

__device__ __forceinline__ void pe_issue(const PESlot& p, int type) {
  if (type == 0) {         // Gram A = X~^T X~
    mma3<E>(p.tm + TM_GRAM, p.Xh, p.Xl, true, p.Xh, p.Xl, true, 64, 0, false);
  } else if (type == 1) {  // A * A
    mma3<D>(p.tm + TM_A2, p.Ah, p.Al, false, p.Ah, p.Al, true, 64, 0, false);
  } else {                 // X~ B'^T, two 128-row halves
    mma3<D>(p.tm + TM_X, p.Xh, p.Xl, false, p.Bh, p.Bl, false, 128, 0, false);
    mma3<D>(p.tm + TM_X + 64, p.Xh, p.Xl, false, p.Bh, p.Bl, false, 128, 16384, false);
  }
}

// Thread 0: copy the tile the epilogue of phase `type` of step `st` just produced
// to the slot's scratch (step k at ns + k * NS_TILE_BYTES: X hi, X lo, A hi, A lo,
// B' hi, B' lo).  type 0 -> A_st, 1 -> B'_st, 2 -> X_{st+1}.  Bulk copies are
// asynchronous; before issuing, all but the most recent earlier copy must have
// finished reading shared memory -- a tile is rewritten three phases after it was
// produced, so this never stalls on a copy whose source is still needed.
__device__ __forceinline__ void pe_save(const PESlot& q, int type, int st) {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
  if (type == 2) {
    uint8_t* o = q.ns + (size_t)(st + 1) * NS_TILE_BYTES;
    bulk_s2g(o, q.Xh, XT_BYTES);
    bulk_s2g(o + XT_BYTES, q.Xl, XT_BYTES);
  } else {
    uint8_t* o = q.ns + (size_t)st * NS_TILE_BYTES + 2 * XT_BYTES + (type == 0 ? 0 : 2 * AT_BYTES);
    bulk_s2g(o, type == 0 ? q.Ah : q.Bh, AT_BYTES);
    bulk_s2g(o + AT_BYTES, type == 0 ? q.Al : q.Bl, AT_BYTES);
  }
  bulk_commit();
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
// On return each slot's final X~ is in TMEM (tm + TM_X, + 64).
static __device__ __forceinline__ bool pe_consume(PESlot* sl, PEBars& B, int nslots, int steps, volatile int* bad,
                                                  unsigned long long* prof = nullptr) {
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, qd = w & 3, ch = w >> 2;
  const int dc = 32 * ch, e0 = 32 * qd + l, e1 = e0 + 128, ra = 16 * qd + l;
  const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
  const int P = 3 * steps;
  bool ok = true;
  for (int s = 0; s < nslots; ++s) pe_publish(B, s);
  for (int p = 0; p < P; ++p) {
    const int type = p % 3, st = p / 3;
    for (int s = 0; s < nslots; ++s) {
      PESlot& q = sl[s];
      long long tw = prof ? clock64() : 0;
      if (!*bad && !mbar_wait(B.done[s], B.done_phase[s])) ok = false;
      B.done_phase[s] ^= 1;
      fence_after();
      long long te = prof ? clock64() : 0;
      if (prof && threadIdx.x == 0) prof[11] += te - tw;
      if (type == 0) {
        float av[32];
        tmem_ld32(q.tm + lane_off + TM_GRAM + dc, av);
        tmem_wait_ld();
        if (l < 16) store_split32(q.Ah, q.Al, ra, dc, D, av);
      } else if (type == 1) {
        const float ca = (float)kPE[st][0], cb = (float)kPE[st][1], cc = (float)kPE[st][2];
        float av[32], a2[32];
        tmem_ld32(q.tm + lane_off + TM_GRAM + dc, av);
        tmem_ld32(q.tm + lane_off + TM_A2 + dc, a2);
        tmem_wait_ld();
        if (l < 16) {
#pragma unroll
          for (int j = 0; j < 32; ++j) a2[j] = fmaf(cc, a2[j], cb * av[j]) + (ra == dc + j ? ca : 0.f);
          store_split32(q.Bh, q.Bl, ra, dc, D, a2);  // B'[ra][c]
        }
      } else if (st + 1 < steps) {
        float x0[32], x1[32];
        tmem_ld32(q.tm + lane_off + TM_X + dc, x0);
        tmem_ld32(q.tm + lane_off + TM_X + 64 + dc, x1);
        tmem_wait_ld();
        store_split32(q.Xh, q.Xl, e0, dc, D, x0);
        store_split32(q.Xh, q.Xl, e1, dc, D, x1);
      }
      if (p + 1 < P) pe_publish(B, s);
      if (prof && threadIdx.x == 0) prof[12] += clock64() - te;
    }
  }
  return ok;
}

// Producer (one whole warp).  Mirrors pe_consume's schedule; saves the freshly
// published tiles (when q.ns is set) before issuing the next MMAs.
static __device__ __forceinline__ bool pe_produce(PESlot* sl, PEBars& B, int nslots, int steps, volatile int* bad) {
  const int P = 3 * steps;
  const bool lead = (threadIdx.x & 31) == 0;
  bool ok = true;
  for (int p = 0; p < P; ++p) {
    const int type = p % 3, st = p / 3;
    for (int s = 0; s < nslots; ++s) {
      PESlot& q = sl[s];
      if (!*bad && !mbar_wait(B.ready[s], B.ready_phase[s])) ok = false;
      B.ready_phase[s] ^= 1;
      fence_after();
      if (q.ns && lead) {  // tile published for this phase: X_st (type 0), A_st (1), B'_st (2)
        if (type == 0) {
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          uint8_t* o = q.ns + (size_t)st * NS_TILE_BYTES;
          bulk_s2g(o, q.Xh, XT_BYTES);
          bulk_s2g(o + XT_BYTES, q.Xl, XT_BYTES);
          bulk_commit();
        } else {
          pe_save(q, type - 1, st);
        }
      }
      __syncwarp();
      if (!*bad) {
        pe_issue(q, type);
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
