// Co-ALiBi forward for few query rows against a long key/value sequence
// ("decode": Sq <= 16, typically 1), on sm_100a.
//
// The forward kernel's 128-row query tiles would be almost empty here and the
// work is a scan over K and V, so the path is HBM-bound and split over the keys:
//
//   partial kernel: one CTA per (batch, kv head, chunk of keys, group of up to 16
//     query rows -- the G query heads of the kv head times the Sq rows); each of
//     its four warps takes a quarter of the chunk and walks it right to left in
//     16- or 32-key steps: S = Q K^T and O += P V on the tensor cores (warp-level MMA,
//     the 16 query rows padded), sigmoids, the inclusive sigmoid suffix sum
//     restarted at 0 at the warp's right end, logits a' = c_a p - slope2 * z_local
//     and an online softmax.  It writes the warp's sigmoid total T, max m, sum l
//     and unnormalised O.
//   combine kernel: one CTA per query row.  The keys right of chunk c add
//     R_c = sum_{c' > c} T_c' to every z of chunk c, i.e. shift its logits by
//     -slope2 * R_c: m'_c = m_c - slope2 * R_c, then the usual log-sum-exp merge
//     gives o, lse and rowsig = sum_c T_c -- the same quantities as the forward
//     kernel (co_alibi_attn/co_alibi_fwd_kernel.py:29-127 semantics).
#pragma once

#include <cuda.h>
#include "sm100.cuh"
#include "fwd.cuh"

namespace coalibi {

constexpr int kDecodeMaxSq = 16;   // COALIBI_DECODE_MAX_SQ
constexpr int kDecodeRows = 16;    // query rows per partial CTA (the MMA's M)
constexpr int kDecodeBlock = 128;  // CTA chunks are multiples of this many keys (four warps x 32)

struct DecodeParams {
  const void* q;
  const void* k;
  const void* v;
  const void* slopes;
  void* o;
  float* lse;
  float* rowsig;
  float* ws;  // partials: stats [rows][n_chunks][4] (T, m, l, -), then O [rows][n_chunks][D]
  int B, Hq, Hkv, Sq, Skv;
  int slopes_dtype;
  int causal;
  float sm_scale;
  int n_chunks, chunk_keys, n_rgroups;
};

struct DecodePlan {
  int cta_chunks;  // key chunks per (b, kv head, row group), one CTA each
  int chunk_keys;  // keys per CTA chunk, a multiple of 128 (four warps x 32)
  int n_rgroups;
  int records;     // partial records per query row: four per CTA chunk (one per warp)
  size_t bytes;
};

// Chunking of the keys: about 512 CTAs over (b, kv head, row group, chunk), chunks
// a multiple of 128 keys, no empty CTA chunk.
template <int D>
inline DecodePlan decode_plan(int B, int Hq, int Hkv, int Sq, int Skv) {
  DecodePlan pl;
  const int G = Hq / Hkv;
  pl.n_rgroups = (G * Sq + kDecodeRows - 1) / kDecodeRows;
  const long long units = (long long)B * Hkv * pl.n_rgroups;
  const int blocks = (Skv + kDecodeBlock - 1) / kDecodeBlock;
  int n = (int)((512 + units - 1) / units);
  n = n < 1 ? 1 : (n > blocks ? blocks : n);
  pl.chunk_keys = ((blocks + n - 1) / n) * kDecodeBlock;
  pl.cta_chunks = (Skv + pl.chunk_keys - 1) / pl.chunk_keys;
  pl.records = 4 * pl.cta_chunks;
  const size_t rows = (size_t)B * Hq * Sq;
  pl.bytes = rows * pl.records * (4 + D) * sizeof(float);
  return pl;
}

// Asynchronous 16-byte global -> shared copy; src_ok false fills zeros (nothing is read).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, bool src_ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
               "r"(src_ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's most recent cp.async groups are still pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_pending() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Partial kernel.  Every warp of the CTA is its own chunk of the keys (a quarter
// of the CTA's range, its own right-to-left suffix, merged by the combine kernel
// like any other chunk), so no step inside a block needs the other warps.  Per 16- or
// 32-key step a warp stages K and V (cp.async, double-buffered,
// padded rows), computes S = Q K^T with mma.m16n8k16 (Q: the 16 padded query
// rows as A fragments held in registers), runs the sigmoid suffix scan on the C
// fragments (quad shuffles within an 8-key tile, tile totals in registers),
// exponentiates, and accumulates O += P V with P's C fragments reused as A
// fragments and V read with ldmatrix.trans.
// ---------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <int D, int STEP_ = 32>
struct DecodeMmaSmem {
  static constexpr int STEP = STEP_;         // keys per warp step (16 or 32)
  static constexpr int NT = STEP / 8;        // 8-key n-tiles of S per step
  static constexpr int ROW = D * 2 + 16;     // padded rows: the 8 rows of an ldmatrix hit distinct banks
  static constexpr int TILE = STEP * ROW;    // one K or V step tile
#ifndef COALIBI_DECODE_STAGES
#define COALIBI_DECODE_STAGES 3
#endif
  static constexpr int NBUF = COALIBI_DECODE_STAGES;  // per-warp ring of K/V steps: NBUF - 1 steps in flight
  static constexpr int PER_WARP = 2 * NBUF * TILE;    // K and V, NBUF buffers each
  static constexpr int BYTES = 4 * PER_WARP;
};

template <int D, bool BF16, int STEP = 32>
__global__ void __launch_bounds__(128) coalibi_decode_mma_kernel(const DecodeParams p) {
  using S = DecodeMmaSmem<D, STEP>;
  constexpr int NT = S::NT;
  constexpr int KK = D / 16;  // k-steps of QK^T, d-tile pairs of PV
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, tig = lane & 3;
  const int bg = blockIdx.x, cc = blockIdx.y;
  const int b = bg / p.Hkv, g = bg - b * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int r0 = blockIdx.z * 16;
  const int R = min(16, G * p.Sq - r0);
  const int sub = p.chunk_keys / 4;
  const int lo = cc * p.chunk_keys + warp * sub;
  const int hi = min(p.Skv, lo + sub);
  const float c_t = 0.5f * p.sm_scale;  // sigmoid(p) = 1/2 + tanh(p / 2) / 2
  const float c_a = p.sm_scale * kLog2e;
  uint8_t* wbase = smem + warp * S::PER_WARP;

  // rows gq and gq + 8 of the 16 (padded) query rows
  int lim[2];
  float slope2[2];
  bool rok[2];
  size_t rowidx[2];
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int u = gq + 8 * x;
    rok[x] = u < R;
    const int rr = r0 + (rok[x] ? u : 0);
    const int h = g * G + rr / p.Sq, i = rr % p.Sq;
    lim[x] = rok[x] ? (p.causal ? min(i + 1, p.Skv) : p.Skv) : 0;
    slope2[x] = load_slope(p.slopes, p.slopes_dtype, h) * kLog2e;
    rowidx[x] = ((size_t)b * p.Hq + h) * p.Sq + i;
  }
  // Q as A fragments: a0 (row gq, cols 2tig..), a1 (row gq+8), a2 / a3 (cols + 8)
  uint32_t qa[KK][4];
  const uint16_t* qg = static_cast<const uint16_t*>(p.q);
#pragma unroll
  for (int kk = 0; kk < KK; ++kk) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const size_t off = rowidx[x] * D + 16 * kk + 8 * hf + 2 * tig;
        qa[kk][2 * hf + x] = rok[x] ? *reinterpret_cast<const uint32_t*>(qg + off) : 0u;
      }
    }
  }
  float o[2 * KK][4];
#pragma unroll
  for (int dn = 0; dn < 2 * KK; ++dn) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.f, 0.f}, carry[2] = {0.f, 0.f};

  const int nsteps = hi > lo ? (hi - lo + S::STEP - 1) / S::STEP : 0;
  auto stage = [&](int st) {
    const int kb = lo + st * S::STEP;
    uint8_t* kt = wbase + (st % S::NBUF) * 2 * S::TILE;
    uint8_t* vt = kt + S::TILE;
#pragma unroll
    for (int it = 0; it < S::STEP * (D / 8) / 32; ++it) {
      const int idx = it * 32 + lane;
      const int key = idx / (D / 8), pc = idx - key * (D / 8);
      const bool ok = kb + key < hi;
      const size_t off = ok ? ((size_t)bg * p.Skv + kb + key) * D + pc * 8 : 0;
      cp_async16(kt + key * S::ROW + pc * 16, static_cast<const uint16_t*>(p.k) + off, ok);
      cp_async16(vt + key * S::ROW + pc * 16, static_cast<const uint16_t*>(p.v) + off, ok);
    }
  };
  // one cp.async group per step (empty past the last one), NBUF - 1 steps ahead of the one computed
#pragma unroll
  for (int a = 1; a < S::NBUF; ++a) {
    if (nsteps - a >= 0) stage(nsteps - a);
    cp_async_commit();
  }
  const int mat = lane >> 3, row8 = lane & 7;
  for (int st = nsteps - 1; st >= 0; --st) {
    if (st - (S::NBUF - 1) >= 0) stage(st - (S::NBUF - 1));
    cp_async_commit();
    cp_async_wait_pending<S::NBUF - 1>();  // the group of step st has landed
    __syncwarp();
    const int kb = lo + st * S::STEP;
    const uint32_t kt = smem_u32(wbase + (st % S::NBUF) * 2 * S::TILE);
    const uint32_t vt = kt + S::TILE;
    // ---- S = Q K^T: n-tile nt holds keys 8nt .. 8nt+7 of the step
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KK; ++kk) {
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        const int key = 16 * np + (mat >> 1) * 8 + row8;
        ldsm_x4(kt + key * S::ROW + (16 * kk + (mat & 1) * 8) * 2, b0, b1, b2, b3);
        mma16816<BF16>(sc[2 * np], qa[kk], b0, b1);
        mma16816<BF16>(sc[2 * np + 1], qa[kk], b2, b3);
      }
    }
    // ---- sigmoids, suffix sums (this warp's keys right of each key), logits, online max
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      float sg[NT][2], excl[NT], tt[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kb + 8 * nt + 2 * tig + e;
          const bool vis = key < lim[x] && key < hi;
          sg[nt][e] = vis ? fmaf(0.5f, tanh_approx(c_t * sc[nt][2 * x + e]), 0.5f) : 0.f;
        }
        const float pp = sg[nt][0] + sg[nt][1];
        float inc = pp;  // inclusive suffix over the quad (keys grow with tig)
        float y = __shfl_down_sync(0xffffffffu, inc, 1);
        if (tig < 3) inc += y;
        y = __shfl_down_sync(0xffffffffu, inc, 2);
        if (tig < 2) inc += y;
        tt[nt] = __shfl_sync(0xffffffffu, inc, lane & ~3);  // the tile's total
        excl[nt] = inc - pp;
      }
      float right = carry[x], mx = -INFINITY;
#pragma unroll
      for (int nt = NT - 1; nt >= 0; --nt) {
        const float z1 = sg[nt][1] + excl[nt] + right;
        const float z0 = z1 + sg[nt][0];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kb + 8 * nt + 2 * tig + e;
          const bool vis = key < lim[x] && key < hi;
          const float a = vis ? fmaf(c_a, sc[nt][2 * x + e], -slope2[x] * (e ? z1 : z0)) : -INFINITY;
          sc[nt][2 * x + e] = a;
          mx = fmaxf(mx, a);
        }
        right += tt[nt];
      }
      carry[x] = right;
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[x], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float fac = (m_run[x] == -INFINITY) ? 0.f : ex2_approx(m_run[x] - m_use);
      m_run[x] = m_new;
      l_part[x] *= fac;
#pragma unroll
      for (int dn = 0; dn < 2 * KK; ++dn) {
        o[dn][2 * x] *= fac;
        o[dn][2 * x + 1] *= fac;
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float a = sc[nt][2 * x + e];
          const float pe = (a == -INFINITY) ? 0.f : ex2_approx(a - m_use);
          sc[nt][2 * x + e] = pe;
          l_part[x] += pe;
        }
      }
    }
    // ---- O += P V: P's C fragments of n-tiles 2kk2, 2kk2+1 form the A fragment of k-step kk2
#pragma unroll
    for (int kk2 = 0; kk2 < NT / 2; ++kk2) {
      uint32_t pa[4];
      pa[0] = pack2<BF16>(sc[2 * kk2][0], sc[2 * kk2][1]);
      pa[1] = pack2<BF16>(sc[2 * kk2][2], sc[2 * kk2][3]);
      pa[2] = pack2<BF16>(sc[2 * kk2 + 1][0], sc[2 * kk2 + 1][1]);
      pa[3] = pack2<BF16>(sc[2 * kk2 + 1][2], sc[2 * kk2 + 1][3]);
#pragma unroll
      for (int dp = 0; dp < KK; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int key = 16 * kk2 + (mat & 1) * 8 + row8;
        ldsm_x4_t(vt + key * S::ROW + (16 * dp + (mat >> 1) * 8) * 2, b0, b1, b2, b3);
        mma16816<BF16>(o[2 * dp], pa, b0, b1);
        mma16816<BF16>(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncwarp();  // this buffer is refilled by the prefetch two steps later
  }
  // ---- this warp's record: sigmoid total, max, sum and unnormalised O per row
  const size_t rows = (size_t)p.B * p.Hq * p.Sq;
  float* stats = p.ws;
  float* obuf = p.ws + rows * p.n_chunks * 4;
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    float l = l_part[x];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (rok[x]) {
      const size_t rec = rowidx[x] * p.n_chunks + cc * 4 + warp;
#pragma unroll
      for (int dn = 0; dn < 2 * KK; ++dn)
        *reinterpret_cast<float2*>(obuf + rec * D + 8 * dn + 2 * tig) = make_float2(o[dn][2 * x], o[dn][2 * x + 1]);
      if (tig == 0) *reinterpret_cast<float4*>(stats + rec * 4) = make_float4(carry[x], m_run[x], l, 0.f);
    }
  }
  cp_async_wait_all();
}

// One CTA (D threads) per query row: merge the chunks right to left.
template <int D, bool BF16>
__global__ void __launch_bounds__(D) coalibi_decode_combine_kernel(const DecodeParams p) {
  const size_t row = blockIdx.x;
  const int d = threadIdx.x;
  const int h = (int)((row / p.Sq) % p.Hq);
  const float slope2 = load_slope(p.slopes, p.slopes_dtype, h) * kLog2e;
  const size_t rows = (size_t)p.B * p.Hq * p.Sq;
  const float4* stats = reinterpret_cast<const float4*>(p.ws) + row * p.n_chunks;
  const float* obuf = p.ws + rows * p.n_chunks * 4 + row * p.n_chunks * D;
  // chunk c's logits shift by -slope2 * (sigmoid totals of the chunks right of it)
  float right = 0.f, M = -INFINITY;
  for (int c = p.n_chunks - 1; c >= 0; --c) {
    const float4 s = stats[c];
    if (s.y != -INFINITY) M = fmaxf(M, s.y - slope2 * right);
    right += s.x;
  }
  const float m_use = (M == -INFINITY) ? 0.f : M;
  float L = 0.f, O = 0.f;
  right = 0.f;
  for (int c = p.n_chunks - 1; c >= 0; --c) {
    const float4 s = stats[c];
    if (s.y != -INFINITY) {
      const float w = ex2_approx(s.y - slope2 * right - m_use);
      L = fmaf(s.z, w, L);
      O = fmaf(obuf[(size_t)c * D + d], w, O);
    }
    right += s.x;
  }
  const float inv = 1.0f / (L + 1e-9f);
  uint16_t* o = static_cast<uint16_t*>(p.o) + row * D;
  if (BF16) {
    o[d] = __bfloat16_as_ushort(__float2bfloat16_rn(O * inv));
  } else {
    o[d] = __half_as_ushort(__float2half_rn(O * inv));
  }
  if (d == 0) {
    p.lse[row] = m_use * kLn2 + logf(L + 1e-9f);
    p.rowsig[row] = right;
  }
}

}  // namespace coalibi
