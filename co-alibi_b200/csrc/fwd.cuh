// Co-ALiBi attention forward for sm_100a.
//
// One CTA owns a 128-row query tile of one (batch, head) and sweeps the key
// tiles from RIGHT to LEFT, so the inclusive suffix sum z_ij = sum_{t>=j} s_it
// of the sigmoids is carried online from tile to tile (the reference kernel
// co_alibi_attn/co_alibi_fwd_kernel.py:66-113 uses the same sweep direction).
//
// Roles (192 threads):
//   warps 0-3  softmax: thread t owns query row t of the tile.  A tcgen05
//              32x32b TMEM load hands it the whole score row, so the reverse
//              suffix scan, the row max and the row sum are sequential
//              in-register work with no shuffles.
//   warp  4    TMA producer: Q once, then K and V tiles into separate rings.
//   warp  5    TMEM allocator + single-thread tcgen05.mma issuer.
//
// TMEM (512 columns x 128 lanes, fp32):
//   [0,128) S buffer 0 | [128,256) S buffer 1 | [256,256+D) O accumulator |
//   two 64-column P buffers (fp16/bf16 pairs) used as the TMEM A operand of O += P V.
//
// Per KV tile n (processing order), the MMA warp issues S_n = Q K_n^T into S
// buffer n%2 as soon as K_n lands, and O += P_n V_n once the softmax warps
// publish P_n.  Softmax works in the log2 domain with a lazily updated
// reference max (O is rescaled in TMEM only when the row max grows by more
// than 2^8), which is exact because O and l share the same stale reference.
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

// Two 128-row query tiles ("slots") per CTA; each slot's rows are split over
// two warpgroups -- one thread per (row, 64-key half) -- so four softmax warps
// share each SM sub-partition and hide each other's latencies.
template <int D>
struct FwdLayout {
  static constexpr int BM = 128, BN = 128;
  static constexpr int KS = (D == 128) ? 2 : 4;
  static constexpr int VS = (D == 128) ? 2 : 3;
  static constexpr int BOX = 128 * 128;  // one [128 rows][64 cols] 16-bit box, SW128
  static constexpr int TILE = BN * D * 2;
  static constexpr int QB = BM * D * 2;
  static constexpr int OFF_Q = 0;  // two query tiles
  static constexpr int OFF_K = OFF_Q + 2 * QB;
  static constexpr int OFF_V = OFF_K + KS * TILE;
  static constexpr int OFF_X = OFF_V + VS * TILE;  // half-row exchange: [2 parity][2 slot][2 half][128] float2
  static constexpr int OFF_BAR = OFF_X + 2 * 2 * 2 * 128 * 8;
  static constexpr int NBAR = 1 + 2 * KS + 2 * VS + 2 + 2 + 2 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  // warps 0-15: softmax (slot = warp / 8, half = (warp / 4) % 2, lane quarter = warp % 4);
  // warp 16: TMA producer; warp 17: TMEM allocator + MMA issuer; warps 18-19 idle.
  // Launched at 96 registers/thread (5 warps per SM sub-partition); the softmax
  // warpgroups then take 104 and the producer warpgroup keeps 64: 4*104 + 64 = 5*96.
  static constexpr int THREADS = 640;
  static constexpr int WARP_TMA = 16, WARP_MMA = 17;
  static constexpr int REGS_SOFTMAX = 104, REGS_PRODUCER = 64;
  static_assert(4 * REGS_SOFTMAX + REGS_PRODUCER <= 5 * 96, "register split exceeds the launch allocation");
  // TMEM per slot s at column 256*s: S [0,128) with P aliased in [0,64); O [128,128+D)
  static constexpr uint32_t TM_SLOT = 256;
  static constexpr uint32_t TM_O = 128;
  static constexpr uint32_t TM_COLS = 512;
  static_assert(ALLOC <= 232448, "shared memory budget");
};

// Sigmoids, local suffix sums and penalised log2-domain logits of one 64-key
// half row (raw q.k dot products in sreg[0..63], keys key0h..key0h+63), right to
// left, starting the suffix sum at 0.  Writes a' = c_a x - slope2 * local_suffix
// back into sreg[]; returns the half's sigmoid total and the max of a'.
template <bool MASK>
__device__ __forceinline__ float2 fwd_scan_half(uint32_t* sreg, int key0h, int lim, float c_sig, float c_a,
                                                float slope2) {
  const float2 csig2 = make_float2(c_sig, c_sig);
  float run = 0.f, mx = -INFINITY;
#pragma unroll
  for (int c = 3; c >= 0; --c) {  // 16-key groups, right to left
    float sg[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = 16 * c + 2 * q;
      const float2 xn = __fmul2_rn(make_float2(__uint_as_float(sreg[j]), __uint_as_float(sreg[j + 1])), csig2);
      sg[2 * q] = sigmoid_from_neg_log2(xn.x);
      sg[2 * q + 1] = sigmoid_from_neg_log2(xn.y);
      if (MASK && key0h + j >= lim) sg[2 * q] = 0.f;
      if (MASK && key0h + j + 1 >= lim) sg[2 * q + 1] = 0.f;
    }
#pragma unroll
    for (int q = 7; q >= 0; --q) {
      const int j = 16 * c + 2 * q;
      run += sg[2 * q + 1];
      const float r1 = run;
      run += sg[2 * q];
      const float r0 = run;
      float a0 = fmaf(-slope2, r0, __uint_as_float(sreg[j]) * c_a);
      float a1 = fmaf(-slope2, r1, __uint_as_float(sreg[j + 1]) * c_a);
      if (MASK && key0h + j >= lim) a0 = -INFINITY;
      if (MASK && key0h + j + 1 >= lim) a1 = -INFINITY;
      mx = max3(mx, a0, a1);
      sreg[j] = __float_as_uint(a0);
      sreg[j + 1] = __float_as_uint(a1);
    }
  }
  return make_float2(run, mx);
}

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
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + L::KS;
  uint64_t* v_full = k_empty + L::KS;
  uint64_t* v_empty = v_full + L::VS;
  uint64_t* s_full = v_empty + L::VS;  // [2] per slot
  uint64_t* p_full = s_full + 2;       // [2]
  uint64_t* pv_done = p_full + 2;      // [2]
  uint64_t* mma_idle = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  const int BH = p.B * p.Hq;
  const int n_pairs = (p.n_qtiles + 1) / 2;
  int bh, pair;
  decode_tile(blockIdx.x, BH, n_pairs, bh, pair);
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int zkv = b * p.Hkv + h / (p.Hq / p.Hkv);
  const bool has1 = (2 * pair + 1) < p.n_qtiles;
  // last key tile visited by each slot (causal: tiles starting at or before the slot's last row)
  const int last0 = p.causal ? min(p.n_kvtiles - 1, 2 * pair) : p.n_kvtiles - 1;
  const int last1 = has1 ? (p.causal ? min(p.n_kvtiles - 1, 2 * pair + 1) : p.n_kvtiles - 1) : -1;
  const int last = max(last0, last1);
  const int N = last + 1;  // tile n of the sweep is key tile last - n
  // slot s is active on sweep step n iff its query tile sees key tile last - n
  auto active = [&](int s, int n) -> bool { return (last - n) <= (s == 0 ? last0 : last1); };

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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&pv_done[i], 1);
    }
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

  if (warp >= 16) {
    regs_decrease<L::REGS_PRODUCER>();
  if (warp == L::WARP_TMA) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, (has1 ? 2 : 1) * L::QB);
      for (int s = 0; s < (has1 ? 2 : 1); ++s)
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sQ + s * L::QB + bx * L::BOX, &tmQ, q_full, bx * 64, (2 * pair + s) * L::BM, bh);
      int nk = 0, nv = 0;
      for (int n = 0; n < N; ++n) {
        const int key0 = (last - n) * L::BN;
        const int ks = n % L::KS;
        if (!mbar_wait(&k_empty[ks], ((n / L::KS) & 1) ^ 1, g)) break;
        mbar_arrive_expect_tx(&k_full[ks], L::TILE);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sK + ks * L::TILE + bx * L::BOX, &tmK, &k_full[ks], bx * 64, key0, zkv);
        ++nk;
        const int vs = n % L::VS;
        if (!mbar_wait(&v_empty[vs], ((n / L::VS) & 1) ^ 1, g)) break;
        mbar_arrive_expect_tx(&v_full[vs], L::TILE);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_3d(sV + vs * L::TILE + bx * L::BOX, &tmV, &v_full[vs], bx * 64, key0, zkv);
        ++nv;
      }
      // Drain: every issued copy must have landed before the CTA may exit.
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
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_f16(BF16, 128, L::BN, false, false);
      constexpr uint32_t idPV = make_idesc_f16(BF16, 128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t v_addr = smem_u32(sV);
      // Slots are served in strict alternation: PV_0(n), S_0(n+1), PV_1(n), S_1(n+1), ...
      // This keeps the two softmax warpgroups half a tile apart (ping-pong): while
      // one waits for its MMAs the other has the exponential unit to itself.
      int k_waited = -1, v_waited = -1;
      int pv_cnt[2] = {0, 0};  // PVs issued per slot
      auto wait_k = [&](int n) -> bool {
        for (; k_waited < n; ++k_waited)
          if (!mbar_wait(&k_full[(k_waited + 1) % L::KS], ((k_waited + 1) / L::KS) & 1, g)) return false;
        return true;
      };
      auto wait_v = [&](int n) -> bool {
        for (; v_waited < n; ++v_waited)
          if (!mbar_wait(&v_full[(v_waited + 1) % L::VS], ((v_waited + 1) / L::VS) & 1, g)) return false;
        return true;
      };
      auto issue_S = [&](int s, int n) -> bool {
        if (!wait_k(n)) return false;
        tc_fence_after();
        const int ks = n % L::KS;
        const uint32_t d = tmem + s * L::TM_SLOT;
        const uint32_t qa = q_addr + s * L::QB;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::BOX + (kk & 3) * 32;
          umma_ss(d, make_sdesc_sw128(qa + off, 16, 1024), make_sdesc_sw128(k_addr + ks * L::TILE + off, 16, 1024),
                  idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        // slot 0 always issues before slot 1 for a given n: release K(n) after the last reader
        if (s == 1 || !active(1, n)) umma_commit(&k_empty[ks]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, g);
      for (int s = 0; ok && s < 2; ++s)
        if (active(s, 0)) ok = issue_S(s, 0);
      for (int n = 0; ok && n < N; ++n) {
        for (int s = 0; ok && s < 2; ++s) {
          const bool act = active(s, n);
          if (act) {
            // P_s(n) published by the slot's softmax warps
            if (!(ok = mbar_wait(&p_full[s], pv_cnt[s] & 1, g))) break;
            if (!(ok = wait_v(n))) break;
            tc_fence_after();
            const int vs = n % L::VS;
            const uint32_t pa = tmem + s * L::TM_SLOT;
#pragma unroll
            for (int kk = 0; kk < L::BN / 16; ++kk) {
              const uint64_t vdesc = make_sdesc_sw128(v_addr + vs * L::TILE + kk * 16 * 128, L::BOX, 1024);
              umma_ts(tmem + s * L::TM_SLOT + L::TM_O, pa + kk * 8, vdesc, idPV,
                      (pv_cnt[s] > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&pv_done[s]);
            ++pv_cnt[s];
            if (s == 1 || !active(1, n)) umma_commit(&v_empty[vs]);
          }
          if (n + 1 < N && active(s, n + 1)) {
            // S_s(n+1) overwrites the TMEM columns P_s(n) is read from.  No wait is
            // needed: tcgen05.mma ops issued by one thread execute in issue order, so
            // PV_s(n) has read P_s(n) before S_s(n+1) writes there (the same aliasing
            // CUTLASS's sm100 attention mainloop relies on).  The commit that
            // publishes S_s(n+1) also covers PV_s(n), so the softmax may rescale O.
            ok = issue_S(s, n + 1);
          }
        }
      }
      // every MMA issued above must have finished before TMEM is released
      umma_commit(mma_idle);
      mbar_drain(mma_idle, 0, g.timeout_ns);
    }
  }
  } else {
    regs_increase<L::REGS_SOFTMAX>();
    // ------------------------------------------------------------ softmax: 2 slots x 2 half rows
    const int slot = warp >> 3;
    const int hf = (warp >> 2) & 1;   // 0: keys [64,128) of the tile (swept first), 1: keys [0,64)
    const int quarter = warp & 3;
    const int t = quarter * 32 + lane;  // row within the slot's tile
    const int pair_bar = 1 + slot * 4 + quarter;  // named barrier of the two warps sharing these rows
    const int qt = 2 * pair + slot;
    const int row = qt * L::BM + t;
    const uint32_t lane_base = tmem + slot * L::TM_SLOT + ((uint32_t)(quarter * 32) << 16);
    const int scol = hf ? 0 : 64;           // my S columns (fp32)
    const int pcol = hf ? 0 : 32;           // my packed P columns
    const int ocol = hf ? 0 : D / 2;        // my O columns
    const float slope = load_slope(p.slopes, p.slopes_dtype, h);
    const float c_sig = -p.sm_scale * kLog2e;
    const float c_a = p.sm_scale * kLog2e;
    const float slope2 = slope * kLog2e;
    const int lim = p.causal ? min(row + 1, p.Skv) : p.Skv;
    float m_ref = -INFINITY, l = 0.f, carry = 0.f;
    bool ok = true;
    int it = 0;
    if (slot == 0 || has1) {
      for (int n = 0; n < N; ++n) {
        if (!active(slot, n)) continue;
        const int key0 = (last - n) * L::BN;
        ok = mbar_wait(&s_full[slot], it & 1, g);
        ok = named_bar_and(pair_bar, 64, ok);  // both halves leave together on an abort
        if (!ok) break;
        tc_fence_after();
        uint32_t sreg[64];
        tmem_ld32(lane_base + scol + 32, sreg + 32);
        tmem_ld32(lane_base + scol, sreg);
        tmem_ld_wait32(sreg + 32);
        tmem_ld_fence32(sreg);
        const bool masked = (key0 + L::BN > p.Skv) || (p.causal && key0 + L::BN - 1 > qt * L::BM);
        const int key0h = key0 + scol;
        const float2 loc = masked ? fwd_scan_half<true>(sreg, key0h, lim, c_sig, c_a, slope2)
                                  : fwd_scan_half<false>(sreg, key0h, lim, c_sig, c_a, slope2);
        // exchange (half sigmoid total, half max of a') with the partner thread of this row
        float2* xb = xch + (it & 1) * 512 + slot * 256;
        xb[hf * 128 + t] = loc;
        named_bar_sync(pair_bar, 64);
        const float2 other = xb[(1 - hf) * 128 + t];
        const float2 right = hf ? other : loc;
        const float2 left = hf ? loc : other;
        const float off_r = carry, off_l = carry + right.x;
        const float tmax = fmaxf(right.y - slope2 * off_r, left.y - slope2 * off_l);
        carry = (carry + right.x) + left.x;
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
        // O is free of this slot's previous PV: the commit that published S_s(it) covers it.
        if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t oreg[32];
            tmem_ld32(lane_base + L::TM_O + ocol + c * 32, oreg);
            tmem_ld_wait32(oreg);
#pragma unroll
            for (int j = 0; j < 32; ++j) oreg[j] = __float_as_uint(__uint_as_float(oreg[j]) * alpha);
            tmem_st32(lane_base + L::TM_O + ocol + c * 32, oreg);
          }
        }
        // e = 2^(a' - slope2 * my_offset - m)
        const float shift = m_use + slope2 * (hf ? off_l : off_r);
        float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t preg[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            // half of the exponentials on the MUFU unit, half as a polynomial on the FMA pipe
            float e0, e1;
            if (j & 1) {
              const float2 e = exp2_poly2(__fadd2_rn(
                  make_float2(__uint_as_float(sreg[32 * c + 2 * j]), __uint_as_float(sreg[32 * c + 2 * j + 1])),
                  make_float2(-shift, -shift)));
              e0 = e.x;
              e1 = e.y;
            } else {
              e0 = ex2_approx(__uint_as_float(sreg[32 * c + 2 * j]) - shift);
              e1 = ex2_approx(__uint_as_float(sreg[32 * c + 2 * j + 1]) - shift);
            }
            ls0 += e0;
            ls1 += e1;
            preg[j] = pack2<BF16>(e0, e1);
          }
          tmem_st16(lane_base + pcol + c * 16, preg);  // P aliased over the S columns already read
        }
        l = fmaf(l, alpha, ls0 + ls1);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[slot]);
        ++it;
      }
      if (ok && it > 0) {
        // combine the two halves' row sums, then wait for the last PV
        float2* xb = xch + (it & 1) * 512 + slot * 256;
        xb[hf * 128 + t] = make_float2(l, 0.f);
        named_bar_sync(pair_bar, 64);
        const float l_other = xb[(1 - hf) * 128 + t].x;
        const float l_row = hf ? (l_other + l) : (l + l_other);  // right + left in both threads
        ok = mbar_wait(&pv_done[slot], (it - 1) & 1, g);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
          const float inv = 1.0f / (l_row + 1e-9f);
          uint8_t* orow = static_cast<uint8_t*>(p.o) + ((size_t)bh * p.Sq + row) * D * 2 + ocol * 2;
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t oreg[32];
            tmem_ld32(lane_base + L::TM_O + ocol + c * 32, oreg);
            tmem_ld_wait32(oreg);
            if (row < p.Sq) {
              uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
              for (int v4 = 0; v4 < 4; ++v4) {
                uint4 pk;
                pk.x = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 0]) * inv, __uint_as_float(oreg[8 * v4 + 1]) * inv);
                pk.y = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 2]) * inv, __uint_as_float(oreg[8 * v4 + 3]) * inv);
                pk.z = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 4]) * inv, __uint_as_float(oreg[8 * v4 + 5]) * inv);
                pk.w = pack2<BF16>(__uint_as_float(oreg[8 * v4 + 6]) * inv, __uint_as_float(oreg[8 * v4 + 7]) * inv);
                dst[v4] = pk;
              }
            }
          }
          if (row < p.Sq && hf == 0) {
            const size_t ri = (size_t)bh * p.Sq + row;
            p.lse[ri] = m_ref * kLn2 + logf(l_row + 1e-9f);
            p.rowsig[ri] = carry;
          }
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

}  // namespace coalibi
