// Co-ALiBi attention forward for sm_100a.
//
// One CTA owns a 128-row query tile of one (batch, head) and sweeps the key
// tiles from RIGHT to LEFT, so the inclusive suffix sum z_ij = sum_{t>=j} s_it
// of the sigmoids is carried online from tile to tile (the reference kernel
// co_alibi_attn/co_alibi_fwd_kernel.py:66-113 uses the same sweep direction).
//
// Roles (640 threads):
//   warps 0-15 softmax: warpgroup w takes keys [32w, 32w+32) of every key tile
//              for the 32 rows of its lane quarter; a tcgen05 32x32b TMEM load
//              hands each thread its 32 scores, so the reverse suffix scan is
//              sequential in-register work; the four chunks of a row exchange
//              (sigmoid total, max) once per tile through shared memory.
//   warp  16   TMA producer: Q once, then K and V tiles into separate rings.
//   warp  17   TMEM allocator + single-thread tcgen05.mma issuer.
//
// TMEM (512 columns x 128 lanes, fp32): two S buffers [0,128) and [128,256),
// P (16-bit pairs) aliased over the first 64 columns of its S buffer, O at 256.
// The MMA warp keeps S two key tiles ahead of PV.  Softmax works in the log2
// domain with a lazily updated reference max (O is rescaled in TMEM only when
// the row max grows by more than 2^8), which is exact because O and l share the
// same stale reference.
#pragma once

#include <cuda.h>
#include "sm100.cuh"

namespace coalibi {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct FwdParams {
  void* o;
  float* lse;
  float* rowsig;
  const void* slopes;
  int B, Hq, Hkv, Sq, Skv;
  int slopes_dtype;
  int causal;
  float sm_scale;
  int* status;
  unsigned long long timeout_ns;
  int n_qtiles;
  int n_kvtiles;
};

__device__ __forceinline__ float load_slope(const void* slopes, int dtype, int h) {
  if (dtype == 2) return static_cast<const float*>(slopes)[h];
  if (dtype == 1) return __bfloat162float(static_cast<const __nv_bfloat16*>(slopes)[h]);
  return __half2float(static_cast<const __half*>(slopes)[h]);
}

// Map a linear CTA index to (bh, q_tile): heads are taken in groups of 8 (so the
// K/V of concurrently running CTAs stay L2 resident) and, within a group, the
// longest causal rows (highest q tile) go first.
__device__ __forceinline__ void decode_tile(int L, int BH, int nQ, int& bh, int& m) {
  const int per_group = 8 * nQ;
  const int grp = L / per_group;
  const int r = L - grp * per_group;
  const int g0 = grp * 8;
  const int gsz = min(8, BH - g0);
  const int mq = r / gsz;
  bh = g0 + (r - mq * gsz);
  m = nQ - 1 - mq;
}

// One 128-row query tile per CTA; each row's 128 keys of a tile are split over
// four softmax warpgroups (warpgroup w: keys [32w, 32w+32)), so four softmax
// warps share each SM sub-partition.  S is double-buffered in TMEM: the MMA
// warp computes S of the next key tile while the softmax works on this one.
template <int D>
struct FwdLayout {
  static constexpr int BM = 128, BN = 128, NWG = 4;
  static constexpr int KS = (D == 128) ? 3 : 4;
  static constexpr int VS = (D == 128) ? 2 : 3;
  static constexpr int BOX = 128 * 128;  // one [128 rows][64 cols] 16-bit box, SW128
  static constexpr int TILE = BN * D * 2;
  static constexpr int QB = BM * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + QB;
  static constexpr int OFF_V = OFF_K + KS * TILE;
  static constexpr int OFF_X = OFF_V + VS * TILE;  // float2 [3][NWG][128]: chunk exchange x2 (tile parity), row sums
  static constexpr int OFF_BAR = OFF_X + 3 * NWG * 128 * 8;
  static constexpr int NBAR = 2 + 2 * KS + 2 * VS + 2 + 2 + 1 + 1 + 1 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  // warps 0-15: softmax (warpgroup = warp / 4, lane quarter = warp % 4);
  // warp 16: TMA producer; warp 17: TMEM allocator + MMA issuer; warps 18-19 idle.
  // Launched at 96 registers/thread (5 warps per SM sub-partition); the softmax
  // warpgroups then take 104 and the producer warpgroup keeps 64: 4*104 + 64 = 5*96.
  static constexpr int THREADS = 640;
  static constexpr int WARP_TMA = 16, WARP_MMA = 17;
  static constexpr int REGS_SOFTMAX = 104, REGS_PRODUCER = 64;
  static_assert(4 * REGS_SOFTMAX + REGS_PRODUCER <= 5 * 96, "register split exceeds the launch allocation");
  // TMEM: S buffers [0,128) and [128,256), P (16-bit pairs) aliased over the first
  // 64 columns of its S buffer once read; O [256, 256+D)
  static constexpr uint32_t TM_SBUF = 128, TM_O = 256, TM_COLS = 512;
  static_assert(ALLOC <= 232448, "shared memory budget");
};

// Sigmoids, suffix sums and penalised log2-domain logits of one 32-key chunk (raw
// q.k dot products in sreg[0..31], keys key0..key0+31), right to left, as four
// 8-key sub-chunks whose suffix sums each start at 0: four short dependent add
// chains, two in flight at a time, instead of one of 32.  Writes
// a'_j = c_a x_j - slope2 * (sigmoid suffix of key j within its sub-chunk) back into
// sreg[].  The sub-chunks right of sub-chunk k add their sigmoid totals to every
// suffix in it; the caller folds that into the sub-chunk's exponent shift,
// soff[k] = slope2 * (sigmoid total of sub-chunks k+1..3), so no per-key work is
// added.  Returns (chunk sigmoid total, max over the chunk of a' - soff).
template <bool MASK>
__device__ __forceinline__ float2 fwd_scan_chunk(uint32_t* sreg, int key0, int lim, float c_t, float c_a,
                                                 float slope2, float* soff) {
  float tot[4], mxk[4];
#pragma unroll
  for (int c = 1; c >= 0; --c) {  // 16-key groups (sub-chunks 2c+1 and 2c), right to left
    float sg[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = 16 * c + 2 * q;
      const float2 u = __fmul2_rn(make_float2(__uint_as_float(sreg[j]), __uint_as_float(sreg[j + 1])),
                                  make_float2(c_t, c_t));
      const float2 s = __ffma2_rn(make_float2(0.5f, 0.5f), make_float2(tanh_approx(u.x), tanh_approx(u.y)),
                                  make_float2(0.5f, 0.5f));
      sg[2 * q] = (MASK && key0 + j >= lim) ? 0.f : s.x;
      sg[2 * q + 1] = (MASK && key0 + j + 1 >= lim) ? 0.f : s.y;
    }
    float run[2] = {0.f, 0.f}, m[2] = {-INFINITY, -INFINITY};  // [0]: sub-chunk 2c, [1]: 2c + 1
#pragma unroll
    for (int q = 3; q >= 0; --q) {
#pragma unroll
      for (int h = 1; h >= 0; --h) {
        const int qq = q + 4 * h;  // pair within the 16-key group
        const int j = 16 * c + 2 * qq;
        run[h] += sg[2 * qq + 1];
        const float r1 = run[h];
        run[h] += sg[2 * qq];
        const float r0 = run[h];
        const float2 xa = __fmul2_rn(make_float2(__uint_as_float(sreg[j]), __uint_as_float(sreg[j + 1])),
                                     make_float2(c_a, c_a));
        float2 a = __ffma2_rn(make_float2(-slope2, -slope2), make_float2(r0, r1), xa);
        if (MASK && key0 + j >= lim) a.x = -INFINITY;
        if (MASK && key0 + j + 1 >= lim) a.y = -INFINITY;
        m[h] = max3(m[h], a.x, a.y);
        sreg[j] = __float_as_uint(a.x);
        sreg[j + 1] = __float_as_uint(a.y);
      }
    }
    tot[2 * c] = run[0];
    tot[2 * c + 1] = run[1];
    mxk[2 * c] = m[0];
    mxk[2 * c + 1] = m[1];
  }
  const float o2 = tot[3], o1 = o2 + tot[2], o0 = o1 + tot[1];
  soff[3] = 0.f;
  soff[2] = slope2 * o2;
  soff[1] = slope2 * o1;
  soff[0] = slope2 * o0;
  const float mx = fmaxf(fmaxf(mxk[3], mxk[2] - soff[2]), fmaxf(mxk[1] - soff[1], mxk[0] - soff[0]));
  return make_float2(o0 + tot[0], mx);
}

// A CTA's work list: in round r it takes item r * G + c (c = blockIdx.x, G =
// gridDim.x) of the (head, query tile) order of decode_tile, or item
// r * G + G - 1 - c in odd rounds.  That order is longest-first within each group
// of heads, so the alternating ("snake") rounds even out the causal work per CTA.
// Each item sweeps its key tiles right to left; every role walks the same
// flattened (item, key tile) sequence.
__device__ __forceinline__ int fwd_work_item(int r) {
  return r * (int)gridDim.x + ((r & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
}

struct FwdItem {
  int bh, qt, zkv, h, last, N;
};

__device__ __forceinline__ FwdItem fwd_item(const FwdParams& p, int L) {
  FwdItem it;
  decode_tile(L, p.B * p.Hq, p.n_qtiles, it.bh, it.qt);
  const int b = it.bh / p.Hq;
  it.h = it.bh - b * p.Hq;
  it.zkv = b * p.Hkv + it.h / (p.Hq / p.Hkv);
  // last key tile this query tile sees; the sweep visits key tiles last, last-1, ..., 0
  it.last = p.causal ? min(p.n_kvtiles - 1, it.qt) : p.n_kvtiles - 1;
  it.N = it.last + 1;
  return it;
}

struct FwdCursor {  // position in the flattened (item, key tile) sequence
  int n, k;          // key-tile step within the item, round (= items so far)
  FwdItem it;
  bool valid;
  __device__ __forceinline__ void start(const FwdParams& p, int n_items) {
    n = 0;
    k = 0;
    const int L = fwd_work_item(0);
    valid = L < n_items;
    if (valid) it = fwd_item(p, L);
  }
  __device__ __forceinline__ void next(const FwdParams& p, int n_items) {
    if (++n == it.N) {
      n = 0;
      ++k;
      const int L = fwd_work_item(k);
      valid = L < n_items;
      if (valid) it = fwd_item(p, L);
    }
  }
};

template <int D, bool BF16>
__global__ void __launch_bounds__(640, 1)
    coalibi_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using L = FwdLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  float2* xch = reinterpret_cast<float2*>(smem + L::OFF_X);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;      // every S of the item completed: the next Q may load
  uint64_t* k_full = q_empty + 1;
  uint64_t* k_empty = k_full + L::KS;
  uint64_t* v_full = k_empty + L::KS;
  uint64_t* v_empty = v_full + L::VS;
  uint64_t* s_full = v_empty + L::VS;  // [2] per S buffer
  uint64_t* p_full = s_full + 2;       // [2] per S buffer
  uint64_t* pv_done = p_full + 2;      // completes once per PV
  uint64_t* o_full = pv_done + 1;      // every PV of the item completed
  uint64_t* o_free = o_full + 1;       // the softmax has read O of the item
  uint64_t* mma_idle = o_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  const int n_items = p.B * p.Hq * p.n_qtiles;
  CtaGuard g{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < L::KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < L::VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4 * L::NWG);  // lane 0 of every softmax warp
    }
    mbar_init(pv_done, 1);
    mbar_init(o_full, 1);
    mbar_init(o_free, 4 * L::NWG);
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

  if (warp >= 16) {
    regs_decrease<L::REGS_PRODUCER>();
  if (warp == L::WARP_TMA) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int nk = 0, nv = 0, nq = 0;
      bool ok = true;
      FwdCursor kc, vc;  // K runs two key tiles ahead of V (S runs two ahead of PV)
      kc.start(p, n_items);
      vc.start(p, n_items);
      auto load_k = [&]() -> bool {
        if (kc.n == 0) {
          // Q of the item: the previous item's S MMAs must all have completed
          if (!mbar_wait(q_empty, (kc.k & 1) ^ 1, g)) return false;
          mbar_arrive_expect_tx(q_full, L::QB);
#pragma unroll
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_3d(sQ + bx * L::BOX, &tmQ, q_full, bx * 64, kc.it.qt * L::BM, kc.it.bh);
          ++nq;
        }
        const int ks = nk % L::KS;
        if (!mbar_wait(&k_empty[ks], ((nk / L::KS) & 1) ^ 1, g)) return false;
        mbar_arrive_expect_tx(&k_full[ks], L::TILE);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sK + ks * L::TILE + bx * L::BOX, &tmK, &k_full[ks], bx * 64, (kc.it.last - kc.n) * L::BN,
                      kc.it.zkv);
        ++nk;
        kc.next(p, n_items);
        return true;
      };
      for (int i = 0; ok && i < 2 && kc.valid; ++i) ok = load_k();
      while (ok && vc.valid) {
        const int vs = nv % L::VS;
        if (!(ok = mbar_wait(&v_empty[vs], ((nv / L::VS) & 1) ^ 1, g))) break;
        mbar_arrive_expect_tx(&v_full[vs], L::TILE);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sV + vs * L::TILE + bx * L::BOX, &tmV, &v_full[vs], bx * 64, (vc.it.last - vc.n) * L::BN,
                      vc.it.zkv);
        ++nv;
        vc.next(p, n_items);
        if (kc.valid) ok = load_k();
      }
      // Drain: every issued copy must have landed before the CTA may exit.
      if (nq > 0) mbar_drain(q_full, (nq - 1) & 1, g.timeout_ns);
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
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_f16(BF16, 128, L::BN, false, false);
      constexpr uint32_t idPV = make_idesc_f16(BF16, 128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t v_addr = smem_u32(sV);
      // Issue order over the flattened key tiles t: S(0), S(1), PV(0), S(2), PV(1),
      // S(3), ...  S(t+2) reuses the TMEM buffer P(t) is aliased in; tcgen05.mma ops
      // issued by one thread run in issue order, so PV(t) has read P(t) before
      // S(t+2) writes there (the same aliasing CUTLASS's sm100 attention mainloop
      // relies on).
      FwdCursor sc, pc;
      sc.start(p, n_items);
      pc.start(p, n_items);
      int ts = 0, tp = 0;  // flattened indices of the next S and the next PV
      auto issue_S = [&]() -> bool {
        if (sc.n == 0) {
          if (!mbar_wait(q_full, sc.k & 1, g)) return false;
        }
        const int ks = ts % L::KS;
        if (!mbar_wait(&k_full[ks], (ts / L::KS) & 1, g)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (ts & 1) * L::TM_SBUF;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::BOX + (kk & 3) * 32;
          umma_ss(d, make_sdesc_sw128(q_addr + off, 16, 1024), make_sdesc_sw128(k_addr + ks * L::TILE + off, 16, 1024),
                  idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[ts & 1]);
        umma_commit(&k_empty[ks]);                     // K(t) only feeds S(t)
        if (sc.n + 1 == sc.it.N) umma_commit(q_empty);  // last S of the item
        ++ts;
        sc.next(p, n_items);
        return true;
      };
      bool ok = true;
      for (int i = 0; ok && i < 2 && sc.valid; ++i) ok = issue_S();
      while (ok && pc.valid) {
        if (pc.n == 0 && pc.k > 0) {
          // O still holds the previous item until its softmax read it out
          if (!(ok = mbar_wait(o_free, (pc.k - 1) & 1, g))) break;
        }
        if (!(ok = mbar_wait(&p_full[tp & 1], (tp >> 1) & 1, g))) break;
        const int vs = tp % L::VS;
        if (!(ok = mbar_wait(&v_full[vs], (tp / L::VS) & 1, g))) break;
        tc_fence_after();
        const uint32_t pa = tmem + (tp & 1) * L::TM_SBUF;
#pragma unroll
        for (int kk = 0; kk < L::BN / 16; ++kk) {
          const uint64_t vdesc = make_sdesc_sw128(v_addr + vs * L::TILE + kk * 16 * 128, L::BOX, 1024);
          umma_ts(tmem + L::TM_O, pa + kk * 8, vdesc, idPV, (pc.n > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[vs]);
        if (pc.n + 1 == pc.it.N) umma_commit(o_full);  // last PV of the item
        ++tp;
        pc.next(p, n_items);
        if (sc.valid) ok = issue_S();
      }
      // every MMA issued above must have finished before TMEM is released
      umma_commit(mma_idle);
      mbar_drain(mma_idle, 0, g.timeout_ns);
    }
  }
  } else {
    regs_increase<L::REGS_SOFTMAX>();
    // ------------------------------------------------------------ softmax: 4 x 32 keys per row
    const int wg = warp >> 2;
    const int quarter = warp & 3;
    const int t = quarter * 32 + lane;  // row within the tile
    const int xbar = 1 + quarter;      // named barrier of the four warps sharing these rows
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    constexpr int OC = D / L::NWG;      // O columns this warpgroup rescales and writes
    const float c_t = 0.5f * p.sm_scale;  // sigmoid(p) = 1/2 + tanh(p / 2) / 2
    const float c_a = p.sm_scale * kLog2e;
    float2* xl = xch + 2 * (L::NWG * 128);  // row-sum exchange at the end of an item
    bool ok = true;
    bool left = false;  // left at a named barrier: all four warps of the quarter together
    int tg = 0;  // flattened key-tile index
    for (int k = 0; fwd_work_item(k) < n_items; ++k) {
      const FwdItem it = fwd_item(p, fwd_work_item(k));
      const int row = it.qt * L::BM + t;
      const float slope = load_slope(p.slopes, p.slopes_dtype, it.h);
      const float slope2 = slope * kLog2e;
      const int lim = p.causal ? min(row + 1, p.Skv) : p.Skv;
      float m_ref = -INFINITY, l = 0.f, carry = 0.f;
      for (int n = 0; n < it.N; ++n, ++tg) {
        const int key0 = (it.last - n) * L::BN + 32 * wg;  // this warpgroup's 32 keys of the tile
        if (ok) ok = mbar_wait(&s_full[tg & 1], (tg >> 1) & 1, g);
        ok = __all_sync(0xffffffffu, ok);
        uint32_t sreg[32];
        float soff[4];  // per-sub-chunk exponent shifts from fwd_scan_chunk
        float2 loc = make_float2(0.f, -INFINITY);
        if (ok) {
          tc_fence_after();
          tmem_ld32(lane_base + (tg & 1) * L::TM_SBUF + 32 * wg, sreg);
          tmem_ld_wait32(sreg);
          const bool masked = (key0 + 32 > p.Skv) || (p.causal && key0 + 31 > it.qt * L::BM);
          loc = masked ? fwd_scan_chunk<true>(sreg, key0, lim, c_t, c_a, slope2, soff)
                       : fwd_scan_chunk<false>(sreg, key0, lim, c_t, c_a, slope2, soff);
        }
        // exchange (chunk sigmoid total, chunk max of a') among the row's four warpgroups;
        // the barrier also orders every S read of this buffer before the P writes into it
        float2* xb = xch + (tg & 1) * (L::NWG * 128);
        xb[wg * 128 + t] = loc;
        tc_fence_before();
        ok = named_bar_and(xbar, 128, ok);
        if (!ok) {
          left = true;
          break;
        }
        tc_fence_after();
        float2 tw[L::NWG];
#pragma unroll
        for (int w = 0; w < L::NWG; ++w) tw[w] = xb[w * 128 + t];
        // offset of chunk w = carry + sigmoid totals of the chunks right of it
        float off = carry, my_off = 0.f, tmax = -INFINITY;
#pragma unroll
        for (int w = L::NWG - 1; w >= 0; --w) {
          if (w == wg) my_off = off;
          tmax = fmaxf(tmax, tw[w].y - slope2 * off);
          off += tw[w].x;
        }
        carry = off;
        float alpha = 1.f;
        bool resc = false;
        if (m_ref == -INFINITY) {
          m_ref = tmax;
        } else if (tmax > m_ref + 8.f) {
          alpha = ex2_approx(m_ref - tmax);
          m_ref = tmax;
          resc = true;
        }
        const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
        if (__any_sync(0xffffffffu, resc)) {
          // O must hold every PV of the item before this tile's: PV(tg-1) may still run
          ok = mbar_wait(pv_done, (tg - 1) & 1, g);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            tc_fence_after();
            uint32_t oreg[OC];
            if (OC == 32) {
              tmem_ld32(lane_base + L::TM_O + wg * OC, oreg);
              tmem_ld_wait32(oreg);
            } else {
              tmem_ld16(lane_base + L::TM_O + wg * OC, oreg);
              tmem_ld_wait16(oreg);
            }
#pragma unroll
            for (int j = 0; j < OC; ++j) oreg[j] = __float_as_uint(__uint_as_float(oreg[j]) * alpha);
            if (OC == 32) tmem_st32(lane_base + L::TM_O + wg * OC, oreg);
            else tmem_st16(lane_base + L::TM_O + wg * OC, oreg);
          }
        }
        if (ok) {
          // e = 2^(a' - slope2 * my_offset - m)
          const float shift = m_use + slope2 * my_off;
          float2 ls = make_float2(0.f, 0.f);
          uint32_t preg[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float sh = shift + soff[j >> 2];  // keys 2j, 2j+1 lie in sub-chunk j / 4
            const float2 x = __fadd2_rn(make_float2(__uint_as_float(sreg[2 * j]), __uint_as_float(sreg[2 * j + 1])),
                                        make_float2(-sh, -sh));
            // a quarter of the exponentials as a polynomial on the FMA pipe (measured best:
            // all on MUFU and half on the FMA pipe are both slower)
            const float2 e = ((j & 3) == 3) ? exp2_poly2(x) : make_float2(ex2_approx(x.x), ex2_approx(x.y));
            ls = __fadd2_rn(ls, e);
            preg[j] = pack2<BF16>(e.x, e.y);
          }
          // P aliased over the first 64 columns of this S buffer (every S read is done)
          tmem_st16(lane_base + (tg & 1) * L::TM_SBUF + 16 * wg, preg);
          l = fmaf(l, alpha, ls.x + ls.y);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[tg & 1]);
        }
      }
      if (left) break;
      // combine the four chunks' row sums (every warp of the quarter that finished
      // the item takes this barrier, whatever its ok), then wait for the item's PVs
      xl[wg * 128 + t] = make_float2(l, 0.f);
      ok = named_bar_and(xbar, 128, ok);
      if (!ok) {
        left = true;
        break;
      }
      float l_row = 0.f;
#pragma unroll
      for (int w = 0; w < L::NWG; ++w) l_row += xl[w * 128 + t].x;
      ok = mbar_wait(o_full, k & 1, g);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float inv = 1.0f / (l_row + 1e-9f);
        uint32_t oreg[OC];
        if (OC == 32) {
          tmem_ld32(lane_base + L::TM_O + wg * OC, oreg);
          tmem_ld_wait32(oreg);
        } else {
          tmem_ld16(lane_base + L::TM_O + wg * OC, oreg);
          tmem_ld_wait16(oreg);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_free);
        if (row < p.Sq) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.o) + ((size_t)it.bh * p.Sq + row) * D * 2 +
                                                wg * OC * 2);
#pragma unroll
          for (int v4 = 0; v4 < OC / 8; ++v4) {
            uint4 pk;
            pk.x = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 0]) * inv, __uint_as_float(oreg[8 * v4 + 1]) * inv);
            pk.y = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 2]) * inv, __uint_as_float(oreg[8 * v4 + 3]) * inv);
            pk.z = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 4]) * inv, __uint_as_float(oreg[8 * v4 + 5]) * inv);
            pk.w = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 6]) * inv, __uint_as_float(oreg[8 * v4 + 7]) * inv);
            dst[v4] = pk;
          }
          if (wg == 0) {
            const size_t ri = (size_t)it.bh * p.Sq + row;
            p.lse[ri] = m_ref * kLn2 + logf(l_row + 1e-9f);
            p.rowsig[ri] = carry;
          }
        }
      }
      // the next item's row-sum exchange reuses xl: no warp may write it before all
      // four have read it; the next item's first tile exchange (a named barrier)
      // comes before that write, so it separates them
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

}  // namespace coalibi
