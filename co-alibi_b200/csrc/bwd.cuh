// Co-ALiBi attention backward for sm_100a: three kernels, no atomics, no
// O(S^2) scratch, deterministic.
//
// With p = scale q.k, s = sigmoid(p), z_ij = sum_{t>=j} s_it, a = p - slope z,
// P = exp(a - lse), the gradient of the penalised logits is
//   dA_ij = P_ij (dO_i.v_j - delta_i),        delta_i = dO_i . O_i
//   dp_ij = dA_ij - slope s_ij (1 - s_ij) c_ij, c_ij = sum_{t<=j} dA_it
//   dQ = scale dp K,  dK = scale dp^T Q,  dV = P^T dO
// (model.py:61-76 with the slope of co_alibi_attn/co_alibi_bwd_kernel.py:133).
// z and c are running sums along the key axis of each query row, so a
// key-major kernel cannot form them on its own.  The split is:
//
//  1. delta pre-pass: delta_i = dO_i . O_i (16-byte loads, D/8 lanes per row).
//  2. pass A, query-major (one CTA per 128-row query tile, 128-key sub-tiles
//     left to right): recomputes S = Q K^T and dP = dO V^T into TMEM, runs the
//     two scans (four warpgroups of 32 keys, running sums handed along the
//     row), accumulates dQ += dS K in TMEM, and records at every 32-key
//     boundary the pair (z suffix, c prefix) of each row -- 8 bytes per
//     (row, 32 keys).
//  3. pass B, key-major (one CTA per block of keys of one kv head): for every
//     query head of the GQA group and every query tile that sees the block it
//     recomputes S and dP, restarts both scans from pass A's carries, writes
//     P and dS to shared memory and accumulates dV += P^T dO and dK += dS^T Q
//     in TMEM.  The GQA group sum therefore happens in TMEM.
//
// D = 128 uses 128-key blocks in pass B with four warpgroups and transposed
// accumulators (dV^T = dO^T P, M = D); D = 64 uses 128-key blocks with one
// warpgroup (dV = P^T dO, M = keys).  Every MMA has M = 128.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include "coalibi.h"
#include "sm100.cuh"
#include "fwd.cuh"

namespace coalibi {

// Two ways to run passes A and B, chosen per call by the workspace it gets:
//  * stored (preferred while its scratch stays under kStoredCapBytes): pass A
//    also writes P and dS -- the 16-bit values its own dQ MMA consumes -- as
//    128 x 128 tiles, one per visible (query tile, key tile) pair, and pass B is
//    a streaming GEMM (dV = P^T dO, dK = dS^T Q) with no per-score maths;
//  * recompute (bounded scratch, O(S^2 / 32)): pass A records the running sums
//    (z suffix, c prefix) every 32 keys and pass B recomputes S, dP, P and dS.
struct BwdWorkspace {
  size_t delta_off, carry_off, p_off, ds_off, total;
  long long tiles_per_head;  // stored: visible tiles per (b, q head)
  bool stored;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// P / dS scratch of the stored path is used only while it stays below this size;
// larger problems recompute in pass B (their scratch grows as S^2 / 32 instead).
constexpr size_t kStoredCapBytes = (size_t)24 << 30;
constexpr size_t kTileBytes = 128 * 128 * 2;  // one 16-bit [128 rows][128 keys] tile

// Visible key tiles of query tile qt: top-left causal key tile kt is seen iff kt <= qt.
__host__ __device__ inline int tiles_in_row(int qt, int n_kv, bool causal) {
  return causal ? min(qt + 1, n_kv) : n_kv;
}
// Index of tile (qt, 0) among a head's visible tiles, rows in order.
__host__ __device__ inline long long tile_row_start(int qt, int n_kv, bool causal) {
  if (!causal) return (long long)qt * n_kv;
  if (qt <= n_kv) return (long long)qt * (qt + 1) / 2;
  return (long long)n_kv * (n_kv + 1) / 2 + (long long)(qt - n_kv) * n_kv;
}

// recompute: delta float [B*Hq][sq_pad]; carry float2 [B*Hq][n_kb32][sq_pad] (one pair per 32 keys)
inline BwdWorkspace bwd_workspace_recompute(int B, int Hq, int Sq, int Skv) {
  const size_t sq_pad = (size_t)((Sq + 127) / 128) * 128;
  const size_t nkb = (size_t)((Skv + 31) / 32);
  BwdWorkspace w{};
  w.stored = false;
  w.delta_off = 0;
  w.carry_off = align256((size_t)B * Hq * sq_pad * 4);
  w.total = w.carry_off + align256((size_t)B * Hq * nkb * sq_pad * 8);
  return w;
}

// stored: delta float [B*Hq][sq_pad]; then per visible tile a P tile and its dS tile, 16-bit
// [B*Hq][tiles_per_head][P, dS][16][128][8]: each tile in 8-key segments of all 128 rows
// (the no-swizzle core-matrix order the MMA reads)
inline BwdWorkspace bwd_workspace_stored(int B, int Hq, int Sq, int Skv, bool causal) {
  const int n_q = (Sq + 127) / 128, n_kv = (Skv + 127) / 128;
  const size_t sq_pad = (size_t)n_q * 128;
  BwdWorkspace w{};
  w.stored = true;
  w.tiles_per_head = tile_row_start(n_q, n_kv, causal);
  w.delta_off = 0;
  w.p_off = align256((size_t)B * Hq * sq_pad * 4);
  w.ds_off = w.p_off + kTileBytes;  // dS tile right after its P tile
  w.total = w.p_off + 2 * (size_t)B * Hq * (size_t)w.tiles_per_head * kTileBytes;
  return w;
}

// The layout a call uses: stored when the caller's workspace holds it, else
// recompute; total == 0 when neither fits.
inline BwdWorkspace bwd_workspace_for(int B, int Hq, int Sq, int Skv, bool causal, size_t provided) {
  const BwdWorkspace s = bwd_workspace_stored(B, Hq, Sq, Skv, causal);
  if (provided >= s.total) return s;
  BwdWorkspace r = bwd_workspace_recompute(B, Hq, Sq, Skv);
  if (provided < r.total) r.total = 0;
  return r;
}

// The size to allocate: the stored layout while its P / dS scratch is below the
// cap, else the recompute layout.
inline size_t bwd_workspace_preferred(int B, int Hq, int Sq, int Skv, bool causal) {
  const BwdWorkspace s = bwd_workspace_stored(B, Hq, Sq, Skv, causal);
  if (s.total - s.p_off <= kStoredCapBytes) return s.total;
  return bwd_workspace_recompute(B, Hq, Sq, Skv).total;
}

struct BwdParams {
  const void* o;
  const void* dout;
  const float* lse;
  const float* rowsig;
  const void* slopes;
  void* dq;
  void* dk;
  void* dv;
  float* delta;
  float2* carry;     // recompute path: pass A -> pass B running sums (null on the stored path)
  uint16_t* pstore;  // stored path: [B*Hq][tiles_per_head][P, dS][16][128][8] (null on the recompute path)
  long long tiles_per_head;
  int B, Hq, Hkv, Sq, Skv;
  int slopes_dtype;
  int causal;
  float sm_scale;
  int* status;
  unsigned long long timeout_ns;
  int n_qtiles;   // ceil(Sq / 128)
  int n_kvtiles;  // ceil(Skv / 128)
  int n_kb32;     // ceil(Skv / 32): carry entries per row
  int n_blocks;   // pass-B key blocks: ceil(Skv / KB)
  int sq_pad;
  // optional [B * Hq * Sq]: dA prefix carried in from keys left of this call's keys
  // (the call is one key shard of a longer row); null = 0
  const float* c_init;
};

// ---------------------------------------------------------------------------
// 1. delta pre-pass
// ---------------------------------------------------------------------------
template <int D, bool BF16>
__global__ void __launch_bounds__(256) coalibi_bwd_delta_kernel(const BwdParams p) {
  // 16-byte loads: D / 8 lanes per row, 32 / (D / 8) rows per warp
  constexpr int LPR = D / 8;
  constexpr int RPW = 32 / LPR;
  const long long nrows = (long long)p.B * p.Hq * p.sq_pad;
  const int lane = threadIdx.x & 31;
  const long long rg = ((long long)blockIdx.x * 8 + (threadIdx.x >> 5)) * RPW + lane / LPR;
  const int sub = lane % LPR;
  float acc = 0.f;
  int bh = 0, row = 0;
  grid_dep_wait();  // before any global-memory access
  grid_dep_launch();
  if (rg < nrows) {
    bh = (int)(rg / p.sq_pad);
    row = (int)(rg - (long long)bh * p.sq_pad);
    if (row < p.Sq) {
      const size_t base = ((size_t)bh * p.Sq + row) * D;
      const uint4 a = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.o) + base)[sub];
      const uint4 b = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.dout) + base)[sub];
      const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 x = unpack2<BF16>(av[i]), y = unpack2<BF16>(bv[i]);
        acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
      }
    }
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (sub == 0 && rg < nrows) p.delta[rg] = acc;
}

// ---------------------------------------------------------------------------
// Per-key maths of pass B: one 32-key chunk of a row, keys left
// to right.  zs = suffix sum of sigmoids from the current key on (inclusive),
// cacc = inclusive prefix of dA.  Writes 16 packed dp pairs and, if P_OUT, 16
// packed P pairs.  Keys >= lim are masked.
// ---------------------------------------------------------------------------
template <bool MASK, bool BF16, bool P_OUT>
__device__ __forceinline__ void bwd_chunk(const uint32_t* sreg, const uint32_t* dsreg, int key0, int lim,
                                          float c_t, float c_a, float slope, float slope2, float lse2,
                                          float delta, float& zs, float& cacc, uint32_t* dp_out,
                                          uint32_t* p_out) {
  // two keys per packed f32x2 instruction; sigmoid(p) = 1/2 + tanh(p / 2) / 2
#pragma unroll
  for (int j2 = 0; j2 < 16; ++j2) {
    const int j = 2 * j2;
    const float2 x = make_float2(__uint_as_float(sreg[j]), __uint_as_float(sreg[j + 1]));
    const float2 y = make_float2(__uint_as_float(dsreg[j]), __uint_as_float(dsreg[j + 1]));
    const float2 u = __fmul2_rn(x, make_float2(c_t, c_t));
    float2 sg = __ffma2_rn(make_float2(0.5f, 0.5f), make_float2(tanh_approx(u.x), tanh_approx(u.y)),
                           make_float2(0.5f, 0.5f));
    if (MASK && key0 + j >= lim) sg.x = 0.f;
    if (MASK && key0 + j + 1 >= lim) sg.y = 0.f;
    float2 z;  // sigmoid suffix from each key on (inclusive)
    z.x = zs;
    z.y = zs - sg.x;
    zs = z.y - sg.y;
    const float2 e = __ffma2_rn(make_float2(-slope2, -slope2), z,
                                __ffma2_rn(x, make_float2(c_a, c_a), make_float2(-lse2, -lse2)));
    float2 P = make_float2(ex2_approx(e.x), ex2_approx(e.y));
    if (MASK && key0 + j >= lim) P.x = 0.f;
    if (MASK && key0 + j + 1 >= lim) P.y = 0.f;
    const float2 dA = __fmul2_rn(P, __fadd2_rn(y, make_float2(-delta, -delta)));
    float2 c;  // dA prefix up to each key (inclusive)
    c.x = cacc + dA.x;
    c.y = c.x + dA.y;
    cacc = c.y;
    const float2 sp = __ffma2_rn(make_float2(-sg.x, -sg.y), sg, sg);  // s (1 - s)
    const float2 dp = __ffma2_rn(__fmul2_rn(sp, make_float2(-slope, -slope)), c, dA);
    dp_out[j2] = pack2<BF16>(dp.x, dp.y);
    if (P_OUT) p_out[j2] = pack2<BF16>(P.x, P.y);
  }
}

// ---------------------------------------------------------------------------
// 2. pass A: dQ and the per-32-key carries
//
// One 128-row query tile per CTA; key sub-tiles of 128, left to right, so every
// MMA has N = 128 (an N = 64 tile reads its A operand from shared memory for
// half the work).  Four softmax warpgroups split each sub-tile's keys 32 ways
// (warpgroup w: keys [32w, 32w+32)).  The running sums along a row (sigmoid
// suffix, dA prefix) are handed from warpgroup to warpgroup through shared
// memory and per-link mbarriers: w passes its running value to w+1 as soon as
// its own chunk total is known, and warpgroup 3 passes it on to warpgroup 0 for
// the next sub-tile.  No warpgroup waits for one to its right, so the four warps
// on a sub-partition drift apart and overlap their MUFU-bound and FMA-bound
// phases.  Each thread copies its S and dP columns to registers and
// releases them at once, so the MMA warp computes S/dP of the next sub-tile
// while this one is still in the softmax.  TMEM: S [0,128), dP [128,256),
// dS (packed 16-bit, two buffers so the softmax never waits for the previous
// sub-tile's dQ) [256,384), dQ [384,384+D).
// ---------------------------------------------------------------------------
#ifndef COALIBI_PASS_A_IDLE_NS
#define COALIBI_PASS_A_IDLE_NS 60
#endif
constexpr unsigned kPassAIdleNs = COALIBI_PASS_A_IDLE_NS;  // pass A MMA issuer: sleep when nothing is ready

template <int D>
struct BwdALayout {
  static constexpr int BM = 128, BN = 128;
  static constexpr int NWG = 4;                  // softmax warpgroups, 32 keys each
  static constexpr int KS = (D == 128) ? 3 : 4;  // K lives from S(n) to dQ(n): deeper ring
  static constexpr int VS = (D == 128) ? 1 : 2;  // V only feeds dP(n)
  static constexpr int KBOX = BN * 128;          // [128 rows][64 cols] box
  static constexpr int TILE = BN * D * 2;        // one K or V sub-tile
  static constexpr int QB = BM * D * 2;
  static constexpr int OFF_Q = 0, OFF_DO = QB;
  static constexpr int OFF_K = 2 * QB;
  static constexpr int OFF_V = OFF_K + KS * TILE;
  static constexpr int OFF_X = OFF_V + VS * TILE;  // float [2][NWG][128]: running sums handed to warpgroup w
  static constexpr int OFF_BAR = OFF_X + 2 * NWG * 128 * 4;
  static constexpr int NLINK = 4 * NWG;            // per (lane quarter, receiving warpgroup)
  static constexpr int NBAR = 1 + 2 * KS + 2 * VS + 9 + 2 * NLINK;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  // + a producer warpgroup (TMA warp, MMA warp, two idle).  640 threads put five
  // warps on each SM sub-partition (96 registers each at launch); setmaxnreg then
  // moves registers from the producer warpgroup to the softmax.
  static constexpr int THREADS = 128 * NWG + 128;
  static constexpr int WARP_TMA = 4 * NWG, WARP_MMA = 4 * NWG + 1;
  static constexpr int REGS_SOFTMAX = 104, REGS_PRODUCER = 64;
  static_assert(4 * REGS_SOFTMAX + REGS_PRODUCER <= 5 * 96, "register split exceeds the launch allocation");
  // the variant that also stores P and dS holds more per thread: 112 / 32
  static constexpr int REGS_SOFTMAX_ST = 112, REGS_PRODUCER_ST = 32;
  static_assert(4 * REGS_SOFTMAX_ST + REGS_PRODUCER_ST <= 5 * 96, "register split exceeds the launch allocation");
  static constexpr uint32_t TM_S = 0, TM_DP = 128, TM_DS = 256, TM_DQ = 384, TM_COLS = 512;
  static_assert(ALLOC <= 232448, "shared memory budget");
  static_assert(TM_DQ + D <= TM_COLS, "TMEM budget");
};

// Per-key maths of pass A, two keys per packed f32x2 instruction (one issue
// slot for two lanes of work; the softmax warps are issue-bound).
//
// Phase 1 of a 32-key chunk: sigmoids (kept in sg; the raw q.k values stay in
// sreg); returns the chunk's sigmoid total.
template <bool MASK>
__device__ __forceinline__ float bwd_a_sig(const uint32_t* sreg, float* sg, int key0, int lim, float c_t) {
  float2 tot = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float2 x = make_float2(__uint_as_float(sreg[j]), __uint_as_float(sreg[j + 1]));
    const float2 u = __fmul2_rn(x, make_float2(c_t, c_t));
    float2 sv = __ffma2_rn(make_float2(0.5f, 0.5f), make_float2(tanh_approx(u.x), tanh_approx(u.y)),
                           make_float2(0.5f, 0.5f));
    if (MASK && key0 + j >= lim) sv.x = 0.f;
    if (MASK && key0 + j + 1 >= lim) sv.y = 0.f;
    sg[j] = sv.x;
    sg[j + 1] = sv.y;
    tot = __fadd2_rn(tot, sv);
  }
  return tot.x + tot.y;
}

// Phase 2 on 16 keys: P = 2^(c_a x + Z) with the sigmoid suffix carried in
// exponent units, Z = -lse2 - slope2 * z (so each key adds slope2 * s to it and the
// exponent is one FMA of the raw q.k value x), dA = P (dP - delta) over the x
// registers; returns the sum of dA.  With STORE, also P packed to 16 bits in pk.
template <bool MASK, bool BF16, bool STORE>
__device__ __forceinline__ float bwd_a_da(uint32_t* xa, const float* sg, const uint32_t* dpr, int key0, int lim,
                                          float c_a, float slope2, float delta, float& zz, uint32_t* pk) {
  float2 tot = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    float2 z;
    z.x = zz;
    zz = fmaf(slope2, sg[j], zz);
    z.y = zz;
    zz = fmaf(slope2, sg[j + 1], zz);
    const float2 e = __ffma2_rn(make_float2(__uint_as_float(xa[j]), __uint_as_float(xa[j + 1])),
                                make_float2(c_a, c_a), z);
    float2 P;
    P.x = ex2_approx(e.x);
    P.y = ex2_approx(e.y);
    if (MASK && key0 + j >= lim) P.x = 0.f;
    if (MASK && key0 + j + 1 >= lim) P.y = 0.f;
    if (STORE) pk[j / 2] = pack2<BF16>(P.x, P.y);
    const float2 dA = __fmul2_rn(
        P, __fadd2_rn(make_float2(__uint_as_float(dpr[j]), __uint_as_float(dpr[j + 1])), make_float2(-delta, -delta)));
    xa[j] = __float_as_uint(dA.x);
    xa[j + 1] = __float_as_uint(dA.y);
    tot = __fadd2_rn(tot, dA);
  }
  return tot.x + tot.y;
}

template <int D, bool BF16, bool STORE>
__global__ void __launch_bounds__(BwdALayout<D>::THREADS, 1)
    coalibi_bwd_a_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                         const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         const BwdParams p) {
  using L = BwdALayout<D>;
  constexpr int BN = L::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sDO = smem + L::OFF_DO;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  float* xs = reinterpret_cast<float*>(smem + L::OFF_X);  // [NWG][128] sigmoid suffix at chunk start
  float* xd = xs + L::NWG * 128;                          // [NWG][128] dA prefix at chunk start
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + L::KS;
  uint64_t* v_full = k_empty + L::KS;
  uint64_t* v_empty = v_full + L::VS;
  uint64_t* s_full = v_empty + L::VS;
  uint64_t* s_free = s_full + 1;   // every softmax warp has S in registers
  uint64_t* dp_full = s_free + 1;
  uint64_t* dp_free = dp_full + 1;
  uint64_t* ds_full = dp_free + 1;  // [2] dS of sub-tile n written to TMEM buffer n & 1
  uint64_t* dq_done = ds_full + 2;  // [2] dQ(n) has read dS buffer n & 1
  uint64_t* mma_idle = dq_done + 2;
  uint64_t* zlink = mma_idle + 1;      // [quarter][receiving warpgroup]
  uint64_t* clink = zlink + L::NLINK;  // [quarter][receiving warpgroup]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  const int BH = p.B * p.Hq;
  int bh, qt;
  decode_tile(blockIdx.x, BH, p.n_qtiles, bh, qt);
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int zkv = b * p.Hkv + h / (p.Hq / p.Hkv);
  // 128-key sub-tiles this query tile sees (causal: those starting at or before its last row)
  const int N = p.causal ? min(p.n_kvtiles, qt + 1) : p.n_kvtiles;
  CtaGuard g{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < L::KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < L::VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4 * L::NWG);
    mbar_init(dp_full, 1);
    mbar_init(dp_free, 4 * L::NWG);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ds_full[i], 4 * L::NWG);
      mbar_init(&dq_done[i], 1);
    }
    mbar_init(mma_idle, 1);
    for (int i = 0; i < L::NLINK; ++i) {
      mbar_init(&zlink[i], 32);  // every lane of the sending warp arrives after its store
      mbar_init(&clink[i], 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == L::WARP_MMA) {
    tmem_alloc(tmem_slot, L::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // before any global-memory access
  grid_dep_launch();

  if (warp >= L::WARP_TMA) {
    regs_decrease<STORE ? L::REGS_PRODUCER_ST : L::REGS_PRODUCER>();
  if (warp == L::WARP_TMA) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, 2 * L::QB);
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) {
        tma_load_3d(sQ + bx * L::KBOX, &tmQ, q_full, bx * 64, qt * L::BM, bh);
        tma_load_3d(sDO + bx * L::KBOX, &tmDO, q_full, bx * 64, qt * L::BM, bh);
      }
      int nk = 0, nv = 0;
      for (int n = 0; n < N; ++n) {
        const int ks = n % L::KS;
        if (!mbar_wait(&k_empty[ks], ((n / L::KS) & 1) ^ 1, g)) break;
        mbar_arrive_expect_tx(&k_full[ks], L::TILE);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sK + ks * L::TILE + bx * L::KBOX, &tmK, &k_full[ks], bx * 64, n * BN, zkv);
        ++nk;
        const int vs = n % L::VS;
        if (!mbar_wait(&v_empty[vs], ((n / L::VS) & 1) ^ 1, g)) break;
        mbar_arrive_expect_tx(&v_full[vs], L::TILE);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sV + vs * L::TILE + bx * L::KBOX, &tmV, &v_full[vs], bx * 64, n * BN, zkv);
        ++nv;
      }
      mbar_drain(q_full, 0, g.timeout_ns);
      for (int s = 0; s < L::KS; ++s) {
        const int uses = (nk > s) ? (nk - 1 - s) / L::KS + 1 : 0;
        if (uses > 0) mbar_drain(&k_full[s], (uses - 1) & 1, g.timeout_ns);
      }
      for (int s = 0; s < L::VS; ++s) {
        const int uses = (nv > s) ? (nv - 1 - s) / L::VS + 1 : 0;
        if (uses > 0) mbar_drain(&v_full[s], (uses - 1) & 1, g.timeout_ns);
      }
    }
  } else if (warp == L::WARP_MMA) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_f16(BF16, 128, BN, false, false);
      constexpr uint32_t idQ = make_idesc_f16(BF16, 128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sDO);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      // Non-blocking issue loop.  S(n) once K(n) landed and every softmax warp
      // copied S(n-1) out; dP(n) once V(n) landed and dP(n-1) was copied out;
      // dQ(n) once the softmax wrote dS(n).
      bool ok = mbar_wait(q_full, 0, g);
      if (ok) tc_fence_after();
      int next_s = 0, next_p = 0, next_q = 0;
      int idle = 0;
      uint64_t t_idle = 0;
      while (ok && next_q < N) {
        bool progressed = false;
        if (next_q < next_p && mbar_test(&ds_full[next_q & 1], (next_q >> 1) & 1)) {
          tc_fence_after();
          const int ks = next_q % L::KS;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            // A = dS (TMEM, 16 keys = 8 packed columns), B = K_n as (N = d, K = keys): MN-major
            const uint64_t kdesc = make_sdesc_sw128(k_addr + ks * L::TILE + kk * 16 * 128, L::KBOX, 1024);
            umma_ts(tmem + L::TM_DQ, tmem + L::TM_DS + (next_q & 1) * 64 + kk * 8, kdesc, idQ,
                    (next_q > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&dq_done[next_q & 1]);
          umma_commit(&k_empty[ks]);
          ++next_q;
          progressed = true;
        }
        if (next_s < N && (next_s == 0 || mbar_test(s_free, (next_s - 1) & 1)) &&
            mbar_test(&k_full[next_s % L::KS], (next_s / L::KS) & 1)) {
          tc_fence_after();
          const uint32_t kb = k_addr + (next_s % L::KS) * L::TILE;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t o = (kk >> 2) * L::KBOX + (kk & 3) * 32;
            umma_ss(tmem + L::TM_S, make_sdesc_sw128(q_addr + o, 16, 1024), make_sdesc_sw128(kb + o, 16, 1024), idS,
                    kk > 0 ? 1u : 0u);
          }
          umma_commit(s_full);
          ++next_s;
          progressed = true;
        }
        if (next_p < next_s && (next_p == 0 || mbar_test(dp_free, (next_p - 1) & 1)) &&
            mbar_test(&v_full[next_p % L::VS], (next_p / L::VS) & 1)) {
          tc_fence_after();
          const int vs = next_p % L::VS;
          const uint32_t vb = v_addr + vs * L::TILE;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t o = (kk >> 2) * L::KBOX + (kk & 3) * 32;
            umma_ss(tmem + L::TM_DP, make_sdesc_sw128(do_addr + o, 16, 1024), make_sdesc_sw128(vb + o, 16, 1024),
                    idS, kk > 0 ? 1u : 0u);
          }
          umma_commit(dp_full);
          umma_commit(&v_empty[vs]);
          ++next_p;
          progressed = true;
        }
        if (progressed) {
          idle = 0;
          t_idle = 0;
        } else {
          // suspend briefly: a spinning issuer takes issue slots from the four softmax
          // warps that share its sub-partition
          if (kPassAIdleNs > 0) __nanosleep(kPassAIdleNs);
          if (++idle == 64) {
            idle = 0;
            const uint64_t now = global_timer_ns();
            if (t_idle == 0) t_idle = now;
            if (g.aborted()) ok = false;
            else if (now - t_idle > g.timeout_ns) {
              g.raise(kStatusTimeout);
              ok = false;
            }
          }
        }
      }
      umma_commit(mma_idle);
      mbar_drain(mma_idle, 0, g.timeout_ns);
    }
  }
  } else {
    regs_increase<STORE ? L::REGS_SOFTMAX_ST : L::REGS_SOFTMAX>();
    // ------------------------------------------------------------ softmax: 4 x 32 keys per row
    const int wg = warp >> 2;
    const int quarter = warp & 3;
    const int t_row = quarter * 32 + lane;
    const int nwg = (wg + 1) % L::NWG;  // warpgroup this one hands its running sums to
    const int row = qt * L::BM + t_row;
    const bool row_ok = row < p.Sq;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float slope = load_slope(p.slopes, p.slopes_dtype, h);
    const float c_t = 0.5f * p.sm_scale;  // sigmoid(p) = 1/2 + tanh(p / 2) / 2
    const float c_a = p.sm_scale * kLog2e;
    const float slope2 = slope * kLog2e;
    const size_t ri = (size_t)bh * p.Sq + row;
    const float lse2 = row_ok ? p.lse[ri] * kLog2e : 0.f;
    const float zs_row = row_ok ? p.rowsig[ri] : 0.f;  // sigmoid suffix sum from key 0 on
    const float delta = p.delta[(size_t)bh * p.sq_pad + row];
    const int lim = row_ok ? (p.causal ? min(row + 1, p.Skv) : p.Skv) : 0;
    const bool rows_partial = (qt * L::BM + L::BM > p.Sq);
    float2* carry_row = STORE ? nullptr : p.carry + (size_t)bh * p.n_kb32 * p.sq_pad + row;
    // stored path: row t_row of the (qt, n) P / dS tiles; a tile holds 16 segments of
    // 8 keys x 128 rows, so this thread's 32 keys are segments 4 wg .. 4 wg + 3 and a
    // warp (32 consecutive rows) writes 512 contiguous bytes per segment
    uint16_t* const pd_row =
        STORE ? p.pstore + ((size_t)bh * p.tiles_per_head + tile_row_start(qt, p.n_kvtiles, p.causal != 0)) *
                               (size_t)(2 * 128 * 128) + (4 * wg * 128 + t_row) * 8
              : nullptr;
    bool ok = true;
    for (int n = 0; n < N; ++n) {
      const int key0 = n * BN + 32 * wg;  // first key of this thread's chunk
      const bool masked = rows_partial || (key0 + 32 > p.Skv) || (p.causal && key0 + 31 > qt * L::BM);
      if (ok) ok = mbar_wait(s_full, n & 1, g);
      ok = __all_sync(0xffffffffu, ok);
      uint32_t xa[32];
      float sg[32];
      float tot = 0.f;
      if (ok) {
        tc_fence_after();
        tmem_ld32(lane_base + L::TM_S + 32 * wg, xa);
        tmem_ld_wait32(xa);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
        tot = masked ? bwd_a_sig<true>(xa, sg, key0, lim, c_t) : bwd_a_sig<false>(xa, sg, key0, lim, c_t);
      }
      // sigmoid suffix sum at this chunk's first key, from the warpgroup to the left
      // (warpgroup 0: from warpgroup 3's previous sub-tile)
      float z0 = zs_row;
      if (ok && (wg > 0 || n > 0)) {
        ok = mbar_wait(&zlink[quarter * L::NWG + wg], (wg > 0 ? n : n - 1) & 1, g);
        z0 = xs[wg * 128 + t_row];
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (wg + 1 < L::NWG || n + 1 < N) {
        xs[nwg * 128 + t_row] = z0 - tot;
        mbar_arrive(&zlink[quarter * L::NWG + nwg]);
      }
      float zz = fmaf(-slope2, z0, -lse2);  // the suffix in exponent units (bwd_a_da)
      ok = mbar_wait(dp_full, n & 1, g);
      ok = __all_sync(0xffffffffu, ok);
      float dtot = 0.f;
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t dpr[16];
          tmem_ld16(lane_base + L::TM_DP + 32 * wg + 16 * hh, dpr);
          tmem_ld_wait16(dpr);
          if (hh == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dp_free);
          }
          uint32_t pk[8];
          dtot += masked ? bwd_a_da<true, BF16, STORE>(xa + 16 * hh, sg + 16 * hh, dpr, key0 + 16 * hh, lim, c_a,
                                                       slope2, delta, zz, pk)
                         : bwd_a_da<false, BF16, STORE>(xa + 16 * hh, sg + 16 * hh, dpr, key0 + 16 * hh, lim, c_a,
                                                        slope2, delta, zz, pk);
          if (STORE) {
            uint16_t* dst = pd_row + n * (2 * 128 * 128) + (2 * hh) * 1024;
            st_global_na(dst, make_uint4(pk[0], pk[1], pk[2], pk[3]));
            st_global_na(dst + 1024, make_uint4(pk[4], pk[5], pk[6], pk[7]));
          }
        }
      }
      // dA prefix sum before this chunk's first key, handed along the same way (the
      // first chunk of the row starts from the carry-in, 0 unless a key shard)
      float cc = (p.c_init != nullptr && row_ok && wg == 0 && n == 0) ? p.c_init[ri] : 0.f;
      if (ok && (wg > 0 || n > 0)) {
        ok = mbar_wait(&clink[quarter * L::NWG + wg], (wg > 0 ? n : n - 1) & 1, g);
        cc = xd[wg * 128 + t_row];
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (wg + 1 < L::NWG || n + 1 < N) {
        xd[nwg * 128 + t_row] = cc + dtot;
        mbar_arrive(&clink[quarter * L::NWG + nwg]);
      }
      const int kb32 = key0 / 32;
      if (!STORE && kb32 < p.n_kb32) carry_row[(size_t)kb32 * p.sq_pad] = make_float2(z0, cc);
      uint32_t dso[16];
#pragma unroll
      for (int j2 = 0; j2 < 16; ++j2) {
        const float2 dA = make_float2(__uint_as_float(xa[2 * j2]), __uint_as_float(xa[2 * j2 + 1]));
        float2 c2;
        cc += dA.x;
        c2.x = cc;
        cc += dA.y;
        c2.y = cc;
        const float2 s2 = make_float2(sg[2 * j2], sg[2 * j2 + 1]);
        const float2 sp = __ffma2_rn(make_float2(-s2.x, -s2.y), s2, s2);           // s (1 - s)
        const float2 m = __fmul2_rn(sp, make_float2(-slope, -slope));
        const float2 v = __ffma2_rn(m, c2, dA);                                   // dA - slope s (1 - s) c
        dso[j2] = pack2<BF16>(v.x, v.y);
      }
      if (STORE) {
        uint16_t* dst = pd_row + n * (2 * 128 * 128) + 128 * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          st_global_na(dst + u * 1024, make_uint4(dso[4 * u], dso[4 * u + 1], dso[4 * u + 2], dso[4 * u + 3]));
      }
      // dS buffer n & 1 is free once dQ(n-2) has run
      if (n > 1) ok = mbar_wait(&dq_done[n & 1], ((n - 2) >> 1) & 1, g);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        tmem_st16(lane_base + L::TM_DS + (n & 1) * 64 + 16 * wg, dso);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ds_full[n & 1]);
      }
    }
    // epilogue: dQ = scale * (dS K); warpgroup w writes columns [w D/4, (w+1) D/4)
    if (ok && N > 0) {
      ok = mbar_wait(&dq_done[(N - 1) & 1], ((N - 1) >> 1) & 1, g);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok && N > 0) {
      tc_fence_after();
      constexpr int CW = D / L::NWG;
      uint32_t r[CW];
      if (CW == 32) {
        tmem_ld32(lane_base + L::TM_DQ + wg * CW, r);
        tmem_ld_wait32(r);
      } else {
        tmem_ld16(lane_base + L::TM_DQ + wg * CW, r);
        tmem_ld_wait16(r);
      }
      if (row_ok) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.dq) + ri * D * 2 + wg * CW * 2);
        const float sc = p.sm_scale;
#pragma unroll
        for (int v4 = 0; v4 < CW / 8; ++v4) {
          uint4 pk;
          pk.x = pack2<BF16>(__uint_as_float(r[8 * v4 + 0]) * sc, __uint_as_float(r[8 * v4 + 1]) * sc);
          pk.y = pack2<BF16>(__uint_as_float(r[8 * v4 + 2]) * sc, __uint_as_float(r[8 * v4 + 3]) * sc);
          pk.z = pack2<BF16>(__uint_as_float(r[8 * v4 + 4]) * sc, __uint_as_float(r[8 * v4 + 5]) * sc);
          pk.w = pack2<BF16>(__uint_as_float(r[8 * v4 + 6]) * sc, __uint_as_float(r[8 * v4 + 7]) * sc);
          dst[v4] = pk;
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == L::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TM_COLS);
  }
}

// ---------------------------------------------------------------------------
// 3a. pass B for D = 64: dK, dV
//
// One CTA per 128 keys of a kv head, one softmax warpgroup (a thread per query
// row, the block's 128 keys as four 32-key chunks restarted from pass A's
// carries), accumulators dV = P^T dO and dK = dS^T Q with M = 128 keys.  (D = 128
// uses coalibi_bwd_b128_kernel below.)
// ---------------------------------------------------------------------------
template <int D>
struct BwdBLayout {
  static_assert(D == 64, "pass B for D = 128 is coalibi_bwd_b128_kernel");
  static constexpr int KB = 128;                 // keys per CTA
  static constexpr int NS = 1;                   // S / dS TMEM buffers
  static constexpr int NWG = 1;
  static constexpr int THREADS = 128 * NWG + 64; // + TMA warp + MMA warp
  static constexpr int WARP_TMA = 4 * NWG, WARP_MMA = 4 * NWG + 1;
  static constexpr int QS = 2, PS = 2;           // Q/dO and P/dP shared-memory stages
  static constexpr int QBOX = 128 * 128;         // [128 rows][64 cols] box
  static constexpr int KBOX = KB * 128;          // [KB rows][64 cols] box
  static constexpr int KTILE = KB * D * 2;
  static constexpr int QB = 128 * D * 2;
  static constexpr int PB = 128 * KB * 2;        // one P (or dP) tile: [128 rows][KB keys]
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = KTILE;
  static constexpr int OFF_QDO = 2 * KTILE;      // QS stages of (Q, dO)
  static constexpr int OFF_P = OFF_QDO + QS * 2 * QB;  // PS stages of (P, dP)
  static constexpr int OFF_BAR = OFF_P + PS * 2 * PB;
  static constexpr int NBAR = 1 + 2 * QS + 2 * PS + 2 + 1 + 1 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static constexpr uint32_t TM_S = 0;                 // KB columns
  static constexpr uint32_t TM_DS = KB;               // KB columns
  static constexpr uint32_t TM_DV = 2 * KB;           // D columns (lanes = keys)
  static constexpr uint32_t TM_DK = TM_DV + D;
  static constexpr uint32_t TM_COLS = 512;
  static_assert(TM_DK + D <= 512, "TMEM budget");
};

__device__ __forceinline__ void decode_block(int L, int n_heads, int n_blocks, int& hk, int& blk) {
  // groups of 8 kv heads; within a group the lowest key blocks (most causal work) first
  const int per_group = 8 * n_blocks;
  const int grp = L / per_group;
  const int r = L - grp * per_group;
  const int g0 = grp * 8;
  const int gsz = min(8, n_heads - g0);
  blk = r / gsz;
  hk = g0 + (r - blk * gsz);
}

template <int D, bool BF16>
__global__ void __launch_bounds__(BwdBLayout<D>::THREADS, 1)
    coalibi_bwd_b_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                         const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         const BwdParams p) {
  using L = BwdBLayout<D>;
  constexpr int KB = L::KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sQDO = smem + L::OFF_QDO;
  uint8_t* sP = smem + L::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* qdo_full = kv_full + 1;
  uint64_t* qdo_empty = qdo_full + L::QS;
  uint64_t* pp_full = qdo_empty + L::QS;
  uint64_t* pp_empty = pp_full + L::PS;
  uint64_t* s_full = pp_empty + L::PS;  // 2
  uint64_t* s_free = s_full + 2;
  uint64_t* acc_done = s_free + 1;
  uint64_t* mma_idle = acc_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  int hk, blk;
  decode_block(blockIdx.x, p.B * p.Hkv, p.n_blocks, hk, blk);  // hk = b * Hkv + g
  const int b = hk / p.Hkv;
  const int gkv = hk - b * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int key0 = blk * KB;
  const int m_start = p.causal ? key0 / 128 : 0;
  const int nM = max(0, p.n_qtiles - m_start);
  const int NIT = G * nM;
  CtaGuard g{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < L::QS; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    for (int i = 0; i < L::PS; ++i) {
      mbar_init(&pp_full[i], 128 * L::NWG);
      mbar_init(&pp_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(s_free, 128);
    mbar_init(acc_done, 1);
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == L::WARP_MMA) {
    tmem_alloc(tmem_slot, L::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // before any global-memory access
  grid_dep_launch();

  if (warp == L::WARP_TMA) {
    if (lane == 0 && NIT > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(kv_full, 2 * L::KTILE);
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) {
        tma_load_3d(sK + bx * L::KBOX, &tmK, kv_full, bx * 64, key0, hk);
        tma_load_3d(sV + bx * L::KBOX, &tmV, kv_full, bx * 64, key0, hk);
      }
      int nq = 0;
      for (int it = 0; it < NIT; ++it) {
        const int hh = gkv * G + it / nM;
        const int m = m_start + it % nM;
        const int bhq = b * p.Hq + hh;
        const int st = it % L::QS;
        if (!mbar_wait(&qdo_empty[st], ((it / L::QS) & 1) ^ 1, g)) break;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * L::QB);
        uint8_t* sq = sQDO + st * 2 * L::QB;
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx) {
          tma_load_3d(sq + bx * L::QBOX, &tmQ, &qdo_full[st], bx * 64, m * 128, bhq);
          tma_load_3d(sq + L::QB + bx * L::QBOX, &tmDO, &qdo_full[st], bx * 64, m * 128, bhq);
        }
        ++nq;
      }
      mbar_drain(kv_full, 0, g.timeout_ns);
      for (int s = 0; s < L::QS; ++s) {
        const int uses = (nq > s) ? (nq - 1 - s) / L::QS + 1 : 0;
        if (uses > 0) mbar_drain(&qdo_full[s], (uses - 1) & 1, g.timeout_ns);
      }
    }
  } else if (warp == L::WARP_MMA) {
    if (lane == 0 && NIT > 0) {
      constexpr uint32_t idS = make_idesc_f16(BF16, 128, KB, false, false);
      // dV[key][d] = P^T[key][row] dO[row][d]  (A = P^T MN-major, B = dO MN-major), M = KB, N = D
      constexpr uint32_t idAcc = make_idesc_f16(BF16, KB, D, true, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      const uint32_t qdo_addr = smem_u32(sQDO), p_addr = smem_u32(sP);
      auto issue_SdS = [&](int it) {
        const int st = it % L::QS;
        tc_fence_after();
        const uint32_t qa = qdo_addr + st * 2 * L::QB, da = qa + L::QB;
        const int sb = it % L::NS;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qo = (kk >> 2) * L::QBOX + (kk & 3) * 32;
          const uint32_t ko = (kk >> 2) * L::KBOX + (kk & 3) * 32;
          umma_ss(tmem + L::TM_S + sb * KB, make_sdesc_sw128(qa + qo, 16, 1024),
                  make_sdesc_sw128(k_addr + ko, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qo = (kk >> 2) * L::QBOX + (kk & 3) * 32;
          const uint32_t ko = (kk >> 2) * L::KBOX + (kk & 3) * 32;
          umma_ss(tmem + L::TM_DS + sb * KB, make_sdesc_sw128(da + qo, 16, 1024),
                  make_sdesc_sw128(v_addr + ko, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
      };
      // Non-blocking issue loop: dV/dK(it) go out as soon as P/dP(it) are
      // published -- never queued behind the load of a later query tile -- which
      // frees that tile's Q/dO stage for the next load as early as possible;
      // S/dS(j) go out once Q/dO(j) landed and their TMEM buffer is free.
      bool ok = mbar_wait(kv_full, 0, g);
      int next_s = 0, next_d = 0, sfree_seen = 0;
      int idle = 0;
      uint64_t t_idle = 0;
      while (ok && next_d < NIT) {
        bool progressed = false;
        if (next_d < next_s && mbar_test(&pp_full[next_d % L::PS], (next_d / L::PS) & 1)) {
          const int it = next_d;
          tc_fence_after();
          const int ps = it % L::PS;
          const int st = it % L::QS;
          const uint32_t qa = qdo_addr + st * 2 * L::QB, da = qa + L::QB;
          const uint32_t pa = p_addr + ps * 2 * L::PB, dpa = pa + L::PB;
          const uint32_t acc = (it > 0) ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < 128 / 16; ++kk) {  // K = 128 query rows, 16 per MMA
            const uint32_t ko = kk * 16 * 128;        // 16 rows of 128 bytes
            // A: P^T / dP^T (MN = keys, two 64-key blocks 128*128 bytes apart), B: dO / Q (MN = d)
            umma_ss(tmem + L::TM_DV, make_sdesc_sw128(pa + ko, 128 * 128, 1024),
                    make_sdesc_sw128(da + ko, L::QBOX, 1024), idAcc, (acc || kk > 0) ? 1u : 0u);
            umma_ss(tmem + L::TM_DK, make_sdesc_sw128(dpa + ko, 128 * 128, 1024),
                    make_sdesc_sw128(qa + ko, L::QBOX, 1024), idAcc, (acc || kk > 0) ? 1u : 0u);
          }
          umma_commit(&pp_empty[ps]);
          umma_commit(&qdo_empty[st]);
          ++next_d;
          progressed = true;
        }
        if (next_s < NIT) {
          // the single TMEM buffer of S/dS(next_s) is free once s_free says the
          // softmax read S/dS(next_s - 1)
          if (sfree_seen < next_s && mbar_test(s_free, sfree_seen & 1)) ++sfree_seen;
          const bool buf_free = sfree_seen >= next_s;
          if (buf_free && mbar_test(&qdo_full[next_s % L::QS], (next_s / L::QS) & 1)) {
            issue_SdS(next_s);
            ++next_s;
            progressed = true;
          }
        }
        if (progressed) {
          idle = 0;
          t_idle = 0;
        } else {
          if (++idle == 64) {
            idle = 0;
            const uint64_t now = global_timer_ns();
            if (t_idle == 0) t_idle = now;
            if (g.aborted()) ok = false;
            else if (now - t_idle > g.timeout_ns) {
              g.raise(kStatusTimeout);
              ok = false;
            }
          }
        }
      }
      if (ok) umma_commit(acc_done);
      umma_commit(mma_idle);
      mbar_drain(mma_idle, 0, g.timeout_ns);
    }
  } else {
    const int wg = warp >> 2;
    const int t_row = threadIdx.x & 127;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float c_t = 0.5f * p.sm_scale;
    const float c_a = p.sm_scale * kLog2e;
    // keys of the block this thread covers: [key0 + wkey0, key0 + wkey0 + WKB)
    constexpr int WKB = KB / L::NWG;
    const int wkey0 = wg * WKB;
    const int kb32 = (key0 + wkey0) / 32;
    bool ok = true;
    // Per-row inputs of an iteration (lse, delta, and pass A's carries at this key
    // block) are loaded one iteration ahead so their latency overlaps the current
    // iteration's work instead of stalling its start.
    struct RowIn {
      float lse2, delta, zs, cacc;
    };
    auto load_row = [&](int it_) -> RowIn {
      RowIn r{0.f, 0.f, 0.f, 0.f};
      if (it_ >= NIT) return r;
      const int hh_ = gkv * G + it_ / nM;
      const int m_ = m_start + it_ % nM;
      const int bhq_ = b * p.Hq + hh_;
      const int row_ = m_ * 128 + t_row;
      if (row_ < p.Sq) r.lse2 = p.lse[(size_t)bhq_ * p.Sq + row_] * kLog2e;
      r.delta = p.delta[(size_t)bhq_ * p.sq_pad + row_];
      const float2 cin = p.carry[((size_t)bhq_ * p.n_kb32 + kb32) * p.sq_pad + row_];
      r.zs = cin.x;
      r.cacc = cin.y;
      return r;
    };
    RowIn nxt = load_row(0);
    for (int it = 0; it < NIT; ++it) {
      const int hh = gkv * G + it / nM;
      const int m = m_start + it % nM;
      const int row = m * 128 + t_row;
      const bool row_ok = row < p.Sq;
      const float slope = load_slope(p.slopes, p.slopes_dtype, hh);
      const float slope2 = slope * kLog2e;
      const RowIn cur = nxt;
      nxt = load_row(it + 1);
      const float lse2 = cur.lse2;
      const float delta = cur.delta;
      float zs = cur.zs, cacc = cur.cacc;
      const int lim = row_ok ? (p.causal ? min(row + 1, p.Skv) : p.Skv) : 0;
      const int mkey0 = key0 + wkey0;
      const bool masked =
          (m * 128 + 128 > p.Sq) || (mkey0 + WKB > p.Skv) || (p.causal && mkey0 + WKB - 1 > m * 128);

      const int sb = it % L::NS;
      ok = mbar_wait(&s_full[sb], (it / L::NS) & 1, g);
      const int ps = it % L::PS;
      if (ok) ok = mbar_wait(&pp_empty[ps], ((it / L::PS) & 1) ^ 1, g);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint8_t* prow = sP + ps * 2 * L::PB;
      uint8_t* dprow = prow + L::PB;
      const uint32_t rsw = t_row & 7;
      const uint32_t rbase = (t_row >> 3) * 1024 + rsw * 128;
#pragma unroll 1
      for (int c = 0; c < WKB / 32; ++c) {
        const int kc = wkey0 / 32 + c;  // 32-key chunk index within the block
        uint32_t sreg[32], dsreg[32];
        tmem_ld32(lane_base + L::TM_S + sb * KB + kc * 32, sreg);
        tmem_ld32(lane_base + L::TM_DS + sb * KB + kc * 32, dsreg);
        tmem_ld_wait32(sreg);
        tmem_ld_fence32(dsreg);
        if (L::NS == 1 && c == WKB / 32 - 1) {
          tc_fence_before();
          mbar_arrive(s_free);
        }
        uint32_t po[16], dpo[16];
        if (masked)
          bwd_chunk<true, BF16, true>(sreg, dsreg, key0 + kc * 32, lim, c_t, c_a, slope, slope2, lse2, delta,
                                      zs, cacc, dpo, po);
        else
          bwd_chunk<false, BF16, true>(sreg, dsreg, key0 + kc * 32, lim, c_t, c_a, slope, slope2, lse2, delta,
                                       zs, cacc, dpo, po);
        // 32 keys = four 16-byte chunks; 64-key swizzle rows, 128x128-byte blocks
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = kc * 4 + u;          // 8-key chunk index within the KB keys
          const uint32_t blk64 = chunk >> 3;    // which 64-key block
          const uint32_t cc = chunk & 7;
          const uint32_t off = blk64 * (128 * 128) + rbase + ((cc ^ rsw) << 4);
          *reinterpret_cast<uint4*>(prow + off) = make_uint4(po[4 * u], po[4 * u + 1], po[4 * u + 2], po[4 * u + 3]);
          *reinterpret_cast<uint4*>(dprow + off) =
              make_uint4(dpo[4 * u], dpo[4 * u + 1], dpo[4 * u + 2], dpo[4 * u + 3]);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&pp_full[ps]);
    }
    // epilogue: lane t = key, columns = d
    const int bkv = hk;
    if (NIT > 0) {
      if (ok) {
        ok = mbar_wait(acc_done, 0, g);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        tc_fence_after();
        const int key = key0 + t_row;
        uint8_t* dvrow = static_cast<uint8_t*>(p.dv) + ((size_t)bkv * p.Skv + key) * D * 2;
        uint8_t* dkrow = static_cast<uint8_t*>(p.dk) + ((size_t)bkv * p.Skv + key) * D * 2;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rv[32], rk[32];
          tmem_ld32(lane_base + L::TM_DV + c * 32, rv);
          tmem_ld32(lane_base + L::TM_DK + c * 32, rk);
          tmem_ld_wait32(rv);
          tmem_ld_fence32(rk);
          if (key < p.Skv) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 a, bb;
              a.x = pack2<BF16>(__uint_as_float(rv[8 * v4 + 0]), __uint_as_float(rv[8 * v4 + 1]));
              a.y = pack2<BF16>(__uint_as_float(rv[8 * v4 + 2]), __uint_as_float(rv[8 * v4 + 3]));
              a.z = pack2<BF16>(__uint_as_float(rv[8 * v4 + 4]), __uint_as_float(rv[8 * v4 + 5]));
              a.w = pack2<BF16>(__uint_as_float(rv[8 * v4 + 6]), __uint_as_float(rv[8 * v4 + 7]));
              const float s = p.sm_scale;
              bb.x = pack2<BF16>(__uint_as_float(rk[8 * v4 + 0]) * s, __uint_as_float(rk[8 * v4 + 1]) * s);
              bb.y = pack2<BF16>(__uint_as_float(rk[8 * v4 + 2]) * s, __uint_as_float(rk[8 * v4 + 3]) * s);
              bb.z = pack2<BF16>(__uint_as_float(rk[8 * v4 + 4]) * s, __uint_as_float(rk[8 * v4 + 5]) * s);
              bb.w = pack2<BF16>(__uint_as_float(rk[8 * v4 + 6]) * s, __uint_as_float(rk[8 * v4 + 7]) * s);
              reinterpret_cast<uint4*>(dvrow + c * 64)[v4] = a;
              reinterpret_cast<uint4*>(dkrow + c * 64)[v4] = bb;
            }
          }
        }
      }
    } else {
      // no query row sees these keys: their gradients are zero
      const int key = key0 + t_row;
      if (key < p.Skv) {
        uint4* dvrow = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.dv) + ((size_t)bkv * p.Skv + key) * D * 2);
        uint4* dkrow = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.dk) + ((size_t)bkv * p.Skv + key) * D * 2);
        for (int v4 = 0; v4 < D / 8; ++v4) {
          dvrow[v4] = make_uint4(0, 0, 0, 0);
          dkrow[v4] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == L::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TM_COLS);
  }
}

// ---------------------------------------------------------------------------
// 3b. pass B for D = 128: 128-key blocks, four softmax warpgroups
//
// One CTA per 128 keys of a kv head, so S = Q K^T and dP = dO V^T run at
// N = 128 and every query tile loaded from L2 serves 128 keys.  Warpgroup w
// takes keys [32w, 32w+32) of every query tile; pass A's carries every 32 keys
// make the four chunks independent (no exchange).  The per-key maths run in two
// phases so that P reaches its MMA before dP is even needed: phase A (S only)
// forms the sigmoids and P and writes P; dV^T += dO^T P then runs and frees dO
// for the next tile's load while phase B (needs dP) forms dS, which goes to its
// own buffer for dK^T += Q^T dS.  Shared memory: K, V (64 KB), a two-deep Q ring
// (64 KB), one dO tile (32 KB), P and dS tiles (32 KB each) = 224 KB.  Each
// thread copies its S and dP columns to registers and releases them, so S/dP of
// the next tile run during this one's softmax.  TMEM: S [0,128), dP [128,256),
// dV^T [256,384), dK^T [384,512) (lanes = d, columns = keys).
// ---------------------------------------------------------------------------
struct BwdB128Layout {
  static constexpr int D = 128, KB = 128, NWG = 4;
  static constexpr int QS = 2;                    // Q stages (dO has one)
  static constexpr int BOX = 128 * 128;           // one [128 rows][64 cols] TMA box
  static constexpr int KTILE = KB * D * 2;        // 32 KB
  static constexpr int QB = 128 * D * 2;          // 32 KB
  static constexpr int PBLK = 128 * 64 * 2;       // [128 query rows][64 keys], 16 KB
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = KTILE;
  static constexpr int OFF_Q = 2 * KTILE;         // QS stages
  static constexpr int OFF_DO = OFF_Q + QS * QB;
  static constexpr int OFF_P = OFF_DO + QB;       // P of one query tile (two 64-key blocks)
  static constexpr int OFF_DS = OFF_P + 2 * PBLK; // dS of one query tile
  static constexpr int OFF_BAR = OFF_DS + 2 * PBLK;
  static constexpr int NBAR = 1 + 2 * QS + 2 + 12;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static constexpr int THREADS = 128 * NWG + 128;  // + producer warpgroup (TMA, MMA, two idle warps)
  static constexpr int WARP_TMA = 4 * NWG, WARP_MMA = 4 * NWG + 1;
  static constexpr int REGS_SOFTMAX = 104, REGS_PRODUCER = 64;
  static_assert(4 * REGS_SOFTMAX + REGS_PRODUCER <= 5 * 96, "register split exceeds the launch allocation");
  static constexpr uint32_t TM_S = 0, TM_DP = 128, TM_DV = 256, TM_DK = 384, TM_COLS = 512;
  static_assert(ALLOC <= 232448, "shared memory budget");
};

// Phase A of a 32-key chunk (S only): sigmoids kept in sg, P kept in sreg (over
// the scores) and packed into po; zs is the sigmoid suffix from the chunk's first
// key on (inclusive) and is advanced past the chunk.
template <bool MASK, bool BF16>
__device__ __forceinline__ void bwd_b_phase_a(uint32_t* sreg, float* sg, uint32_t* po, int key0, int lim,
                                              float c_t, float c_a, float slope2, float lse2, float& zs) {
#pragma unroll
  for (int j2 = 0; j2 < 16; ++j2) {
    const int j = 2 * j2;
    const float2 x = make_float2(__uint_as_float(sreg[j]), __uint_as_float(sreg[j + 1]));
    const float2 u = __fmul2_rn(x, make_float2(c_t, c_t));
    float2 s = __ffma2_rn(make_float2(0.5f, 0.5f), make_float2(tanh_approx(u.x), tanh_approx(u.y)),
                          make_float2(0.5f, 0.5f));
    if (MASK && key0 + j >= lim) s.x = 0.f;
    if (MASK && key0 + j + 1 >= lim) s.y = 0.f;
    float2 z;  // sigmoid suffix from each key on (inclusive)
    z.x = zs;
    z.y = zs - s.x;
    zs = z.y - s.y;
    const float2 e = __ffma2_rn(make_float2(-slope2, -slope2), z,
                                __ffma2_rn(x, make_float2(c_a, c_a), make_float2(-lse2, -lse2)));
    // A quarter of the exponentials on the FMA pipe relieves the MUFU unit,
    // which also carries the tanh of every key.
    float2 P = ((j2 & 3) == 3) ? exp2_poly2(e) : make_float2(ex2_approx(e.x), ex2_approx(e.y));
    if (MASK && key0 + j >= lim) P.x = 0.f;
    if (MASK && key0 + j + 1 >= lim) P.y = 0.f;
    sg[j] = s.x;
    sg[j + 1] = s.y;
    sreg[j] = __float_as_uint(P.x);
    sreg[j + 1] = __float_as_uint(P.y);
    po[j2] = pack2<BF16>(P.x, P.y);
  }
}

// Phase B on 16 keys (needs dP): dA = P (dP - delta), c = running dA prefix,
// dS = dA - slope s (1 - s) c, packed into dso.
template <bool BF16>
__device__ __forceinline__ void bwd_b_phase_b(const uint32_t* preg, const float* sg, const uint32_t* dpr,
                                              float slope, float delta, float& cacc, uint32_t* dso) {
#pragma unroll
  for (int j2 = 0; j2 < 8; ++j2) {
    const int j = 2 * j2;
    const float2 P = make_float2(__uint_as_float(preg[j]), __uint_as_float(preg[j + 1]));
    const float2 dA = __fmul2_rn(
        P, __fadd2_rn(make_float2(__uint_as_float(dpr[j]), __uint_as_float(dpr[j + 1])), make_float2(-delta, -delta)));
    float2 c;  // dA prefix up to each key (inclusive)
    c.x = cacc + dA.x;
    c.y = c.x + dA.y;
    cacc = c.y;
    const float2 s2 = make_float2(sg[j], sg[j + 1]);
    const float2 sp = __ffma2_rn(make_float2(-s2.x, -s2.y), s2, s2);  // s (1 - s)
    const float2 dp = __ffma2_rn(__fmul2_rn(sp, make_float2(-slope, -slope)), c, dA);
    dso[j2] = pack2<BF16>(dp.x, dp.y);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(BwdB128Layout::THREADS, 1)
    coalibi_bwd_b128_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                            const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                            const BwdParams p) {
  using L = BwdB128Layout;
  constexpr int D = L::D, KB = L::KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sDO = smem + L::OFF_DO;
  uint8_t* sP = smem + L::OFF_P;
  uint8_t* sDS = smem + L::OFF_DS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* q_full = kv_full + 1;       // [QS]
  uint64_t* q_empty = q_full + L::QS;   // [QS] dK^T of the tile read Q
  uint64_t* do_full = q_empty + L::QS;
  uint64_t* do_empty = do_full + 1;     // dV^T of the tile read dO
  uint64_t* s_full = do_empty + 1;      // S of the tile in TMEM
  uint64_t* s_free = s_full + 1;        // every softmax warp copied S out
  uint64_t* dp_full = s_free + 1;
  uint64_t* dp_free = dp_full + 1;
  uint64_t* p_full = dp_free + 1;       // P of the tile written
  uint64_t* p_empty = p_full + 1;       // dV^T read it
  uint64_t* ds_full = p_empty + 1;
  uint64_t* ds_empty = ds_full + 1;     // dK^T read it
  uint64_t* acc_done = ds_empty + 1;
  uint64_t* mma_idle = acc_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  int hk, blk;
  decode_block(blockIdx.x, p.B * p.Hkv, p.n_blocks, hk, blk);  // hk = b * Hkv + g
  const int b = hk / p.Hkv;
  const int gkv = hk - b * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int key0 = blk * KB;
  const int m_start = p.causal ? key0 / 128 : 0;
  const int nM = max(0, p.n_qtiles - m_start);
  const int NIT = G * nM;
  CtaGuard g{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < L::QS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 4 * L::NWG);
    mbar_init(dp_full, 1);
    mbar_init(dp_free, 4 * L::NWG);
    mbar_init(p_full, 4 * L::NWG);
    mbar_init(p_empty, 1);
    mbar_init(ds_full, 4 * L::NWG);
    mbar_init(ds_empty, 1);
    mbar_init(acc_done, 1);
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == L::WARP_MMA) {
    tmem_alloc(tmem_slot, L::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // before any global-memory access
  grid_dep_launch();

  if (warp >= L::WARP_TMA) {
    regs_decrease<L::REGS_PRODUCER>();
  if (warp == L::WARP_TMA) {
    if (lane == 0 && NIT > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(kv_full, 2 * L::KTILE);
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) {
        tma_load_3d(sK + bx * L::BOX, &tmK, kv_full, bx * 64, key0, hk);
        tma_load_3d(sV + bx * L::BOX, &tmV, kv_full, bx * 64, key0, hk);
      }
      int nq = 0, ndo = 0;
      bool ok = true;
      auto bhq_of = [&](int it) { return b * p.Hq + gkv * G + it / nM; };
      auto m_of = [&](int it) { return m_start + it % nM; };
      auto load_q = [&](int it) -> bool {
        const int st = it % L::QS;
        if (!mbar_wait(&q_empty[st], ((it / L::QS) & 1) ^ 1, g)) return false;
        mbar_arrive_expect_tx(&q_full[st], L::QB);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sQ + st * L::QB + bx * L::BOX, &tmQ, &q_full[st], bx * 64, m_of(it) * 128, bhq_of(it));
        ++nq;
        return true;
      };
      // Q runs a tile ahead of dO: dO(it) waits for dV^T(it - 1), Q(it + 1) for dK^T(it - 1)
      ok = load_q(0);
      for (int it = 0; ok && it < NIT; ++it) {
        if (!(ok = mbar_wait(do_empty, (it & 1) ^ 1, g))) break;
        mbar_arrive_expect_tx(do_full, L::QB);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sDO + bx * L::BOX, &tmDO, do_full, bx * 64, m_of(it) * 128, bhq_of(it));
        ++ndo;
        if (it + 1 < NIT) ok = load_q(it + 1);
      }
      mbar_drain(kv_full, 0, g.timeout_ns);
      for (int s = 0; s < L::QS; ++s) {
        const int uses = (nq > s) ? (nq - 1 - s) / L::QS + 1 : 0;
        if (uses > 0) mbar_drain(&q_full[s], (uses - 1) & 1, g.timeout_ns);
      }
      if (ndo > 0) mbar_drain(do_full, (ndo - 1) & 1, g.timeout_ns);
    }
  } else if (warp == L::WARP_MMA) {
    if (lane == 0 && NIT > 0) {
      constexpr uint32_t idS = make_idesc_f16(BF16, 128, KB, false, false);
      // dV^T[d][key] = dO^T[d][row] P[row][key], dK^T = Q^T dS: A MN-major (d), B MN-major (keys)
      constexpr uint32_t idAcc = make_idesc_f16(BF16, D, KB, true, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sDO);
      const uint32_t p_addr = smem_u32(sP), ds_addr = smem_u32(sDS);
      bool ok = mbar_wait(kv_full, 0, g);
      if (ok) tc_fence_after();
      auto acc_mma = [&](uint32_t acc_t, uint32_t a_base, uint32_t b_base, bool first) {
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {  // K = 128 query rows, 16 per MMA
          const uint32_t ko = kk * 16 * 128;
          umma_ss(acc_t, make_sdesc_sw128(a_base + ko, L::BOX, 1024), make_sdesc_sw128(b_base + ko, L::PBLK, 1024),
                  idAcc, (!first || kk > 0) ? 1u : 0u);
        }
      };
      // Issue in the order the softmax produces work, each step a (suspending)
      // wait: S(it+1) as soon as S(it) was copied out, dV(it) on P(it), dK(it) on
      // dS(it), dP(it+1) once dP(it) was copied out and dO(it+1) landed.
      auto issue_S = [&](int it) {
        tc_fence_after();
        const uint32_t qa = q_addr + (it % L::QS) * L::QB;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * L::BOX + (kk & 3) * 32;
          umma_ss(tmem + L::TM_S, make_sdesc_sw128(qa + o, 16, 1024), make_sdesc_sw128(k_addr + o, 16, 1024), idS,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
      };
      auto issue_dP = [&]() {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * L::BOX + (kk & 3) * 32;
          umma_ss(tmem + L::TM_DP, make_sdesc_sw128(do_addr + o, 16, 1024), make_sdesc_sw128(v_addr + o, 16, 1024),
                  idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(dp_full);
      };
      if (ok) ok = mbar_wait(&q_full[0], 0, g);
      if (ok) issue_S(0);
      if (ok) ok = mbar_wait(do_full, 0, g);
      if (ok) issue_dP();
      for (int it = 0; ok && it < NIT; ++it) {
        if (it + 1 < NIT) {
          if (!(ok = mbar_wait(s_free, it & 1, g))) break;
          if (!(ok = mbar_wait(&q_full[(it + 1) % L::QS], ((it + 1) / L::QS) & 1, g))) break;
          issue_S(it + 1);
        }
        if (!(ok = mbar_wait(p_full, it & 1, g))) break;
        tc_fence_after();
        acc_mma(tmem + L::TM_DV, do_addr, p_addr, it == 0);
        umma_commit(p_empty);
        umma_commit(do_empty);
        if (!(ok = mbar_wait(ds_full, it & 1, g))) break;
        tc_fence_after();
        acc_mma(tmem + L::TM_DK, q_addr + (it % L::QS) * L::QB, ds_addr, it == 0);
        umma_commit(ds_empty);
        umma_commit(&q_empty[it % L::QS]);
        if (it + 1 == NIT) umma_commit(acc_done);
        if (it + 1 < NIT) {
          if (!(ok = mbar_wait(dp_free, it & 1, g))) break;
          if (!(ok = mbar_wait(do_full, (it + 1) & 1, g))) break;
          issue_dP();
        }
      }
      umma_commit(mma_idle);
      mbar_drain(mma_idle, 0, g.timeout_ns);
    }
  }
  } else {
    regs_increase<L::REGS_SOFTMAX>();
    const int wg = warp >> 2;
    const int quarter = warp & 3;
    const int t_row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float c_t = 0.5f * p.sm_scale;
    const float c_a = p.sm_scale * kLog2e;
    const int ckey0 = key0 + 32 * wg;  // this warpgroup's 32 keys
    const int kb32 = ckey0 / 32;
    bool ok = true;
    struct RowIn {
      float lse2, delta, zs, cacc;
    };
    // per-row inputs of an iteration, loaded one iteration ahead (pinned loads: the
    // compiler would otherwise sink them next to their use and expose the latency)
    auto load_row = [&](int it_, int hh_, int m_) -> RowIn {
      RowIn r{0.f, 0.f, 0.f, 0.f};
      if (it_ >= NIT) return r;
      const int bhq_ = b * p.Hq + hh_;
      const int row_ = m_ * 128 + t_row;
      if (row_ < p.Sq) r.lse2 = ldg_pinned(p.lse + (size_t)bhq_ * p.Sq + row_);
      r.delta = ldg_pinned(p.delta + (size_t)bhq_ * p.sq_pad + row_);
      if (kb32 < p.n_kb32) {
        const float2 cin = ldg_pinned(p.carry + ((size_t)bhq_ * p.n_kb32 + kb32) * p.sq_pad + row_);
        r.zs = cin.x;
        r.cacc = cin.y;
      }
      return r;
    };
    int slope_hh = -1;
    float slope = 0.f;
    RowIn nxt = load_row(0, gkv * G, m_start);
    int hh = gkv * G, m = m_start;          // head and query tile of iteration it
    int hh_n = hh + (nM == 1 ? 1 : 0), m_n = (nM == 1) ? m_start : m_start + 1;  // of it + 1
    // this thread's row in the 128B-swizzled P/dS tiles: keys of block (wg >> 1), 16-byte chunks (wg & 1) * 4 + u
    const uint32_t rsw = t_row & 7;
    const uint32_t pb_row = (uint32_t)(wg >> 1) * L::PBLK + (t_row >> 3) * 1024 + rsw * 128;
    for (int it = 0; it < NIT; ++it) {
      const int row = m * 128 + t_row;
      const bool row_ok = row < p.Sq;
      if (hh != slope_hh) {
        slope = load_slope(p.slopes, p.slopes_dtype, hh);
        slope_hh = hh;
      }
      const float slope2 = slope * kLog2e;
      const RowIn cur = nxt;
      nxt = load_row(it + 1, hh_n, m_n);
      float zs = cur.zs, cacc = cur.cacc;
      const int lim = row_ok ? (p.causal ? min(row + 1, p.Skv) : p.Skv) : 0;
      const bool masked =
          (m * 128 + 128 > p.Sq) || (ckey0 + 32 > p.Skv) || (p.causal && ckey0 + 31 > m * 128);
      // ---- phase A: S -> sigmoids and P
      ok = mbar_wait(s_full, it & 1, g);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sreg[32];
      float sg[32];
      tmem_ld32(lane_base + L::TM_S + 32 * wg, sreg);
      tmem_ld_wait32(sreg);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      {
        uint32_t po[16];
        if (masked)
          bwd_b_phase_a<true, BF16>(sreg, sg, po, ckey0, lim, c_t, c_a, slope2, cur.lse2 * kLog2e, zs);
        else
          bwd_b_phase_a<false, BF16>(sreg, sg, po, ckey0, lim, c_t, c_a, slope2, cur.lse2 * kLog2e, zs);
        // P of this tile once dV^T of the previous one read the P tile
        if (it > 0) ok = mbar_wait(p_empty, (it - 1) & 1, g);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t off = pb_row + ((((uint32_t)(wg & 1) * 4 + u) ^ rsw) << 4);
          *reinterpret_cast<uint4*>(sP + off) = make_uint4(po[4 * u], po[4 * u + 1], po[4 * u + 2], po[4 * u + 3]);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // ---- phase B: dP -> dS
      ok = mbar_wait(dp_full, it & 1, g);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t dso[16];
#pragma unroll
      for (int hh2 = 0; hh2 < 2; ++hh2) {
        uint32_t dpr[16];
        tmem_ld16(lane_base + L::TM_DP + 32 * wg + 16 * hh2, dpr);
        tmem_ld_wait16(dpr);
        if (hh2 == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dp_free);
        }
        bwd_b_phase_b<BF16>(sreg + 16 * hh2, sg + 16 * hh2, dpr, slope, cur.delta, cacc, dso + 8 * hh2);
      }
      // dS of this tile once dK^T of the previous one read the dS tile
      if (it > 0) ok = mbar_wait(ds_empty, (it - 1) & 1, g);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t off = pb_row + ((((uint32_t)(wg & 1) * 4 + u) ^ rsw) << 4);
        *reinterpret_cast<uint4*>(sDS + off) = make_uint4(dso[4 * u], dso[4 * u + 1], dso[4 * u + 2], dso[4 * u + 3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
      hh = hh_n;
      m = m_n;
      if (++m_n == p.n_qtiles) {
        m_n = m_start;
        ++hh_n;
      }
    }
    // epilogue: lanes = d, columns = keys; warpgroup w writes its 32 keys
    const int bkv = hk;
    if (NIT > 0) {
      if (ok) {
        ok = mbar_wait(acc_done, 0, g);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        tc_fence_after();
        const int d = t_row;
        uint32_t rv[32], rk[32];
        tmem_ld32(lane_base + L::TM_DV + 32 * wg, rv);
        tmem_ld32(lane_base + L::TM_DK + 32 * wg, rk);
        tmem_ld_wait32(rv);
        tmem_ld_fence32(rk);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int key = ckey0 + j;
          if (key < p.Skv) {
            const size_t o = ((size_t)bkv * p.Skv + key) * D + d;
            const uint32_t pv = pack2<BF16>(__uint_as_float(rv[j]), 0.f);
            const uint32_t pk = pack2<BF16>(__uint_as_float(rk[j]) * p.sm_scale, 0.f);
            static_cast<uint16_t*>(p.dv)[o] = (uint16_t)(pv & 0xffffu);
            static_cast<uint16_t*>(p.dk)[o] = (uint16_t)(pk & 0xffffu);
          }
        }
      }
    } else {
      // no query row sees these keys: their gradients are zero
      const int d = t_row;
      for (int j = 0; j < 32; ++j) {
        const int key = ckey0 + j;
        if (key < p.Skv) {
          const size_t o = ((size_t)bkv * p.Skv + key) * D + d;
          static_cast<uint16_t*>(p.dv)[o] = 0;
          static_cast<uint16_t*>(p.dk)[o] = 0;
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == L::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host-side helpers (called from coalibi.cu)
// ---------------------------------------------------------------------------
int make_tmap(CUtensorMap* map, const void* base, int D, int rows, int heads, int box_rows, bool bf16);

// ---------------------------------------------------------------------------
// 3c. pass B of the stored path: dK, dV as a streaming GEMM
//
// One CTA per 128 keys of a kv head.  For every query head of the GQA group and
// every query tile that sees the block, TMA brings in the (query tile, key
// block) tiles of P and dS that pass A wrote (one 32 KB bulk copy each: pass A
// wrote them in the core-matrix order of a no-swizzle MN-major operand), with dO
// and Q of the query tile (TMA, 128-byte swizzle), and one thread issues
//   dV[key][d] += P^T[key][row] dO[row][d],   dK[key][d] += dS^T[key][row] Q[row][d]
// (M = 128 keys, N = D, K = 128 rows; both operands MN-major).  No per-score maths is left: the kernel
// streams 64 KB of P / dS per query tile from HBM, and Q / dO tiles, which every
// key block of the head re-reads, mostly from L2.  A ring of NSLOT slots holds
// alternately (P, dO) and (dS, Q).  TMEM: dV [0, D), dK [D, 2D) (lanes = keys).
// ---------------------------------------------------------------------------
template <int D>
struct BwdKVLayout {
  static constexpr int NSLOT = (D == 128) ? 3 : 4;
  static constexpr int BOX = 128 * 128;        // [128 rows][64 cols] 16-bit box, 128-byte swizzle
  static constexpr int PT = 128 * 128 * 2;     // a P or dS tile: two 64-key boxes
  static constexpr int QT = 128 * D * 2;       // a Q or dO tile: D / 64 boxes
  static constexpr int SLOT = PT + QT;
  static constexpr int OFF_BAR = NSLOT * SLOT;
  static constexpr int NBAR = 2 * NSLOT + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static constexpr int THREADS = 192;          // warps 0-3 epilogue, 4 TMA, 5 MMA
  static constexpr int WARP_TMA = 4, WARP_MMA = 5;
  static constexpr uint32_t TM_DV = 0, TM_DK = D, TM_COLS = (2 * D <= 128) ? 128 : 256;
  static_assert(ALLOC <= 232448, "shared memory budget");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(BwdKVLayout<D>::THREADS, 1)
    coalibi_bwd_kv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                          const BwdParams p) {
  using L = BwdKVLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* slot_full = bars;
  uint64_t* slot_empty = slot_full + L::NSLOT;
  uint64_t* acc_done = slot_empty + L::NSLOT;
  uint64_t* mma_idle = acc_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  int hk, blk;
  decode_block(blockIdx.x, p.B * p.Hkv, p.n_kvtiles, hk, blk);  // hk = b * Hkv + g
  const int b = hk / p.Hkv;
  const int gkv = hk - b * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int m_start = p.causal ? blk : 0;  // first query tile that sees key tile blk
  const int nM = max(0, p.n_qtiles - m_start);
  const int NSTEP = 2 * G * nM;            // half-steps: (P, dO) then (dS, Q) per query tile
  CtaGuard g{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::NSLOT; ++i) {
      mbar_init(&slot_full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == L::WARP_MMA) {
    tmem_alloc(tmem_slot, L::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // before any global-memory access
  grid_dep_launch();

  if (warp == L::WARP_TMA) {
    if (lane == 0 && NSTEP > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      int issued = 0;
      for (int i = 0; i < NSTEP; ++i) {
        const int it = i >> 1;
        const bool second = (i & 1) != 0;  // (dS, Q) half
        const int hh = gkv * G + it / nM;
        const int m = m_start + it % nM;
        const int bhq = b * p.Hq + hh;
        const size_t tile = (size_t)bhq * p.tiles_per_head + tile_row_start(m, p.n_kvtiles, p.causal != 0) + blk;
        const int sl = i % L::NSLOT;
        if (!mbar_wait(&slot_empty[sl], ((i / L::NSLOT) & 1) ^ 1, g)) break;
        mbar_arrive_expect_tx(&slot_full[sl], L::SLOT);
        uint8_t* dst = smem + sl * L::SLOT;
        bulk_load(dst, p.pstore + (2 * tile + (second ? 1 : 0)) * (128 * 128), L::PT, &slot_full[sl]);
        const void* tq = second ? static_cast<const void*>(&tmQ) : static_cast<const void*>(&tmDO);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx) tma_load_3d(dst + L::PT + bx * L::BOX, tq, &slot_full[sl], bx * 64, m * 128, bhq);
        ++issued;
      }
      // every issued copy must land before the CTA exits
      for (int s2 = 0; s2 < L::NSLOT; ++s2) {
        const int uses = (issued > s2) ? (issued - 1 - s2) / L::NSLOT + 1 : 0;
        if (uses > 0) mbar_drain(&slot_full[s2], (uses - 1) & 1, g.timeout_ns);
      }
    }
  } else if (warp == L::WARP_MMA) {
    if (lane == 0 && NSTEP > 0) {
      // M = 128 keys, N = D, K = 16 rows per MMA.  A = P^T / dS^T, MN-major without
      // swizzle: core matrices of 8 rows x 8 keys, 128 bytes apart along the rows (K)
      // and 128 x 16 = 2048 bytes apart along the keys (MN).  B = dO / Q, MN-major
      // 128-byte swizzle (D / 64 boxes BOX bytes apart).
      constexpr uint32_t idAcc = make_idesc_f16(BF16, 128, D, true, true);
      const uint32_t base = smem_u32(smem);
      bool ok = true;
      for (int i = 0; i < NSTEP && ok; ++i) {
        const int sl = i % L::NSLOT;
        if (!(ok = mbar_wait(&slot_full[sl], (i / L::NSLOT) & 1, g))) break;
        tc_fence_after();
        const uint32_t a = base + sl * L::SLOT;
        const uint32_t bq = a + L::PT;
        const uint32_t dst = tmem + ((i & 1) ? L::TM_DK : L::TM_DV);
        const uint32_t acc = (i >= 2) ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          umma_ss(dst, make_sdesc_noswz(a + kk * 256, 128, 2048), make_sdesc_sw128(bq + kk * 16 * 128, L::BOX, 1024),
                  idAcc, (acc || kk > 0) ? 1u : 0u);
        }
        umma_commit(&slot_empty[sl]);
      }
      if (ok) umma_commit(acc_done);
      umma_commit(mma_idle);
      mbar_drain(mma_idle, 0, g.timeout_ns);
    }
  } else {
    // epilogue: thread t = key key0 + t of the block, columns = d
    const int quarter = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const int key = blk * 128 + (int)threadIdx.x;
    uint8_t* dvrow = static_cast<uint8_t*>(p.dv) + ((size_t)hk * p.Skv + key) * D * 2;
    uint8_t* dkrow = static_cast<uint8_t*>(p.dk) + ((size_t)hk * p.Skv + key) * D * 2;
    if (NSTEP > 0) {
      bool ok = mbar_wait(acc_done, 0, g);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float sc = p.sm_scale;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rv[32], rk[32];
          tmem_ld32(lane_base + L::TM_DV + c * 32, rv);
          tmem_ld32(lane_base + L::TM_DK + c * 32, rk);
          tmem_ld_wait32(rv);
          tmem_ld_fence32(rk);
          if (key < p.Skv) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 a, bb;
              a.x = pack2<BF16>(__uint_as_float(rv[8 * v4 + 0]), __uint_as_float(rv[8 * v4 + 1]));
              a.y = pack2<BF16>(__uint_as_float(rv[8 * v4 + 2]), __uint_as_float(rv[8 * v4 + 3]));
              a.z = pack2<BF16>(__uint_as_float(rv[8 * v4 + 4]), __uint_as_float(rv[8 * v4 + 5]));
              a.w = pack2<BF16>(__uint_as_float(rv[8 * v4 + 6]), __uint_as_float(rv[8 * v4 + 7]));
              bb.x = pack2<BF16>(__uint_as_float(rk[8 * v4 + 0]) * sc, __uint_as_float(rk[8 * v4 + 1]) * sc);
              bb.y = pack2<BF16>(__uint_as_float(rk[8 * v4 + 2]) * sc, __uint_as_float(rk[8 * v4 + 3]) * sc);
              bb.z = pack2<BF16>(__uint_as_float(rk[8 * v4 + 4]) * sc, __uint_as_float(rk[8 * v4 + 5]) * sc);
              bb.w = pack2<BF16>(__uint_as_float(rk[8 * v4 + 6]) * sc, __uint_as_float(rk[8 * v4 + 7]) * sc);
              reinterpret_cast<uint4*>(dvrow + c * 64)[v4] = a;
              reinterpret_cast<uint4*>(dkrow + c * 64)[v4] = bb;
            }
          }
        }
      }
    } else if (key < p.Skv) {
      // no query row sees these keys: their gradients are zero
      for (int v4 = 0; v4 < D / 8; ++v4) {
        reinterpret_cast<uint4*>(dvrow)[v4] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(dkrow)[v4] = make_uint4(0, 0, 0, 0);
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == L::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TM_COLS);
  }
}

template <typename K>
inline bool bwd_set_smem_one(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
}

inline bool bwd_set_smem_attributes() {
  bool ok = true;
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<128, false, false>, BwdALayout<128>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<128, true, false>, BwdALayout<128>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<64, false, false>, BwdALayout<64>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<64, true, false>, BwdALayout<64>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<128, false, true>, BwdALayout<128>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<128, true, true>, BwdALayout<128>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<64, false, true>, BwdALayout<64>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_a_kernel<64, true, true>, BwdALayout<64>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_kv_kernel<128, false>, BwdKVLayout<128>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_kv_kernel<128, true>, BwdKVLayout<128>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_kv_kernel<64, false>, BwdKVLayout<64>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_kv_kernel<64, true>, BwdKVLayout<64>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_b128_kernel<false>, BwdB128Layout::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_b128_kernel<true>, BwdB128Layout::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_b_kernel<64, false>, BwdBLayout<64>::ALLOC);
  ok &= bwd_set_smem_one(coalibi_bwd_b_kernel<64, true>, BwdBLayout<64>::ALLOC);
  return ok;
}

template <int D, bool BF16>
inline int bwd_launch_t(const CoalibiBwdArgs& a, const BwdWorkspace& ws, unsigned long long tmo,
                        cudaStream_t stream, int phases, const float* c_init) {
  BwdParams p{};
  p.c_init = c_init;
  p.o = a.o;
  p.dout = a.dout;
  p.lse = a.lse;
  p.rowsig = a.rowsig;
  p.slopes = a.slopes;
  p.dq = a.dq;
  p.dk = a.dk;
  p.dv = a.dv;
  uint8_t* wsb = static_cast<uint8_t*>(a.workspace);
  p.delta = reinterpret_cast<float*>(wsb + ws.delta_off);
  p.carry = ws.stored ? nullptr : reinterpret_cast<float2*>(wsb + ws.carry_off);
  p.pstore = ws.stored ? reinterpret_cast<uint16_t*>(wsb + ws.p_off) : nullptr;
  p.tiles_per_head = ws.tiles_per_head;
  p.B = a.B;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.Sq = a.Sq;
  p.Skv = a.Skv;
  p.slopes_dtype = a.slopes_dtype;
  p.causal = a.causal ? 1 : 0;
  p.sm_scale = a.sm_scale;
  p.status = a.status;
  p.timeout_ns = tmo;
  p.n_qtiles = (a.Sq + 127) / 128;
  p.n_kvtiles = (a.Skv + 127) / 128;
  p.n_kb32 = (a.Skv + 31) / 32;
  int kb_b;  // keys per pass-B CTA
  if constexpr (D == 128) kb_b = BwdB128Layout::KB;
  else kb_b = BwdBLayout<D>::KB;
  p.n_blocks = (a.Skv + kb_b - 1) / kb_b;
  p.sq_pad = p.n_qtiles * 128;

  CUtensorMap tq, tdo, tk, tv, tkb, tvb;
  int rc;
  if ((rc = make_tmap(&tq, a.q, D, a.Sq, a.B * a.Hq, 128, BF16))) return rc;
  if ((rc = make_tmap(&tdo, a.dout, D, a.Sq, a.B * a.Hq, 128, BF16))) return rc;
  if ((rc = make_tmap(&tk, a.k, D, a.Skv, a.B * a.Hkv, 128, BF16))) return rc;
  if ((rc = make_tmap(&tv, a.v, D, a.Skv, a.B * a.Hkv, 128, BF16))) return rc;
  if (!ws.stored) {
    if ((rc = make_tmap(&tkb, a.k, D, a.Skv, a.B * a.Hkv, kb_b, BF16))) return rc;
    if ((rc = make_tmap(&tvb, a.v, D, a.Skv, a.B * a.Hkv, kb_b, BF16))) return rc;
  }

  const long long rows = (long long)a.B * a.Hq * p.sq_pad;
  cudaError_t e = cudaSuccess;
  auto keep = [&e](cudaError_t r) {
    if (e == cudaSuccess) e = r;
  };
  if (phases & 1)
    keep(launch_pdl(coalibi_bwd_delta_kernel<D, BF16>, dim3((unsigned)((rows + 8 * (256 / D) - 1) / (8 * (256 / D)))),
                    dim3(256), 0, stream, p));
  if ((phases & 2) && ws.stored)
    keep(launch_pdl(coalibi_bwd_a_kernel<D, BF16, true>, dim3(a.B * a.Hq * p.n_qtiles), dim3(BwdALayout<D>::THREADS),
                    BwdALayout<D>::ALLOC, stream, tq, tdo, tk, tv, p));
  if ((phases & 2) && !ws.stored)
    keep(launch_pdl(coalibi_bwd_a_kernel<D, BF16, false>, dim3(a.B * a.Hq * p.n_qtiles), dim3(BwdALayout<D>::THREADS),
                    BwdALayout<D>::ALLOC, stream, tq, tdo, tk, tv, p));
  if ((phases & 4) && ws.stored) {
    keep(launch_pdl(coalibi_bwd_kv_kernel<D, BF16>, dim3(a.B * a.Hkv * p.n_kvtiles), dim3(BwdKVLayout<D>::THREADS),
                    BwdKVLayout<D>::ALLOC, stream, tq, tdo, p));
  } else if (phases & 4) {
    if constexpr (D == 128)
      keep(launch_pdl(coalibi_bwd_b128_kernel<BF16>, dim3(a.B * a.Hkv * p.n_blocks), dim3(BwdB128Layout::THREADS),
                      BwdB128Layout::ALLOC, stream, tq, tdo, tkb, tvb, p));
    else
      keep(launch_pdl(coalibi_bwd_b_kernel<D, BF16>, dim3(a.B * a.Hkv * p.n_blocks), dim3(BwdBLayout<D>::THREADS),
                      BwdBLayout<D>::ALLOC, stream, tq, tdo, tkb, tvb, p));
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? COALIBI_OK : COALIBI_ERR_LAUNCH;
}

inline int bwd_launch(const CoalibiBwdArgs& a, const BwdWorkspace& ws, unsigned long long tmo,
                      cudaStream_t stream, int phases, const float* c_init = nullptr) {
  const bool bf16 = a.dtype == COALIBI_BF16;
  if (a.D == 128)
    return bf16 ? bwd_launch_t<128, true>(a, ws, tmo, stream, phases, c_init)
                : bwd_launch_t<128, false>(a, ws, tmo, stream, phases, c_init);
  return bf16 ? bwd_launch_t<64, true>(a, ws, tmo, stream, phases, c_init)
              : bwd_launch_t<64, false>(a, ws, tmo, stream, phases, c_init);
}

}  // namespace coalibi
