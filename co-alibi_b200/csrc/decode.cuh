// Co-ALiBi forward for few query rows against a long key/value sequence
// ("decode": Sq <= 16, typically 1), on sm_100a CUDA cores.
//
// The forward kernel's 128-row query tiles would be almost empty here and the
// work is a scan over K and V, so the path is HBM-bound and split over the keys:
//
//   partial kernel: one CTA per (batch, kv head, chunk of keys, group of up to 16
//     query rows -- the G query heads of the kv head times the Sq rows).  It walks
//     its chunk right to left in 128-key blocks staged in shared memory: scores
//     (one thread per key, all rows), sigmoids, the inclusive sigmoid suffix sum
//     restarted at 0 at the chunk's right end (warp shuffles plus a running carry
//     across blocks), logits a' = c_a p - slope2 * z_local, an online softmax and
//     O = sum 2^(a' - m) v (one thread per output dimension).  It writes the
//     chunk's sigmoid total T, max m, sum l and unnormalised O.
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
constexpr int kDecodeRows = 16;    // query rows per partial CTA
constexpr int kDecodeBlock = 128;  // keys per shared-memory block (= threads per CTA)

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
  int n_chunks, chunk_keys, n_rgroups;
  size_t bytes;
};

// Chunking of the keys: about 1024 partial CTAs over (b, kv head, row group, chunk),
// chunks a multiple of 128 keys, no empty chunk.
template <int D>
inline DecodePlan decode_plan(int B, int Hq, int Hkv, int Sq, int Skv) {
  DecodePlan pl;
  const int G = Hq / Hkv;
  pl.n_rgroups = (G * Sq + kDecodeRows - 1) / kDecodeRows;
  const long long units = (long long)B * Hkv * pl.n_rgroups;
  const int blocks = (Skv + kDecodeBlock - 1) / kDecodeBlock;
  int n = (int)((1024 + units - 1) / units);
  n = n < 1 ? 1 : (n > blocks ? blocks : n);
  pl.chunk_keys = ((blocks + n - 1) / n) * kDecodeBlock;
  pl.n_chunks = (Skv + pl.chunk_keys - 1) / pl.chunk_keys;
  const size_t rows = (size_t)B * Hq * Sq;
  pl.bytes = rows * pl.n_chunks * (4 + D) * sizeof(float);
  return pl;
}

// Asynchronous 16-byte global -> shared copy; src_ok false fills zeros (nothing is read).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, bool src_ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
               "r"(src_ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all_but_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int D>
struct DecodeSmem {
  static constexpr int KROW = D * 2 + 16;  // padded K rows: thread-per-key 16-byte reads hit distinct banks
  static constexpr int KBUF = kDecodeBlock * KROW;
  static constexpr int VBUF = kDecodeBlock * D * 2;
  static constexpr int OFF_K = 0;                                          // [2] K blocks
  static constexpr int OFF_V = OFF_K + 2 * KBUF;                           // [2] V blocks
  static constexpr int OFF_Q = OFF_V + 2 * VBUF;                           // float [16][D]
  static constexpr int OFF_E = OFF_Q + kDecodeRows * D * 4;                // float [128 keys][16 rows]
  static constexpr int OFF_W = OFF_E + kDecodeBlock * kDecodeRows * 4;     // float [4 warps][16] sigmoid totals
  static constexpr int OFF_X = OFF_W + 4 * kDecodeRows * 4;                // float [4 warps][16] block maxima
  static constexpr int OFF_L = OFF_X + 4 * kDecodeRows * 4;                // float [4 warps][16] block row sums
  static constexpr int OFF_R = OFF_L + 4 * kDecodeRows * 4;                // row state: m, carry, slope2, lim, l
  static constexpr int BYTES = OFF_R + 5 * kDecodeRows * 4;
  // PV: a thread owns two adjacent dimensions and one group of the block's keys
  static constexpr int NGRP = kDecodeBlock / (D / 2);                    // key groups (2 for D=128, 4 for D=64)
  static constexpr int KPG = kDecodeBlock / NGRP;                        // keys per group
  static_assert((NGRP - 1) * kDecodeRows * D * 4 <= 2 * KBUF, "the group fold reuses the K buffers");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kDecodeBlock) coalibi_decode_partial_kernel(const DecodeParams p) {
  using S = DecodeSmem<D>;
  extern __shared__ __align__(16) uint8_t smem[];
  float* qs = reinterpret_cast<float*>(smem + S::OFF_Q);
  float* es = reinterpret_cast<float*>(smem + S::OFF_E);
  float* wsum = reinterpret_cast<float*>(smem + S::OFF_W);
  float* wmax = reinterpret_cast<float*>(smem + S::OFF_X);
  float* wl = reinterpret_cast<float*>(smem + S::OFF_L);
  float* m_s = reinterpret_cast<float*>(smem + S::OFF_R);
  float* carry_s = m_s + kDecodeRows;
  float* slope_s = carry_s + kDecodeRows;
  int* lim_s = reinterpret_cast<int*>(slope_s + kDecodeRows);
  float* l_s = reinterpret_cast<float*>(lim_s + kDecodeRows);

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int bg = blockIdx.x;  // b * Hkv + g
  const int c = blockIdx.y;   // key chunk (at most 1024 of them)
  const int b = bg / p.Hkv, g = bg - b * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int r0 = blockIdx.z * kDecodeRows;
  const int R = min(kDecodeRows, G * p.Sq - r0);
  const int key_lo = c * p.chunk_keys;
  const int key_hi = min(p.Skv, key_lo + p.chunk_keys);
  const float c_t = 0.5f * p.sm_scale;  // sigmoid(p) = 1/2 + tanh(p / 2) / 2
  const float c_a = p.sm_scale * kLog2e;

  // local row u -> query head g*G + (r0+u)/Sq, query position (r0+u)%Sq
  if (t < kDecodeRows) {
    m_s[t] = -INFINITY;
    carry_s[t] = 0.f;
    l_s[t] = 0.f;
    slope_s[t] = 0.f;
    lim_s[t] = 0;
    if (t < R) {
      const int rr = r0 + t;
      const int h = g * G + rr / p.Sq, i = rr % p.Sq;
      slope_s[t] = load_slope(p.slopes, p.slopes_dtype, h) * kLog2e;
      lim_s[t] = p.causal ? min(i + 1, p.Skv) : p.Skv;
    }
  }
  for (int idx = t; idx < kDecodeRows * D; idx += kDecodeBlock) {
    const int u = idx / D, d = idx - u * D;
    float x = 0.f;
    if (u < R) {
      const int rr = r0 + u;
      const int h = g * G + rr / p.Sq, i = rr % p.Sq;
      const uint16_t raw = static_cast<const uint16_t*>(p.q)[(((size_t)b * p.Hq + h) * p.Sq + i) * D + d];
      x = BF16 ? __bfloat162float(__ushort_as_bfloat16(raw)) : __half2float(__ushort_as_half(raw));
    }
    qs[idx] = x;
  }

  // PV ownership: dimensions 2 * (t % (D/2)) and +1, keys of group t / (D/2)
  const int dpair = t % (D / 2);
  const int kgrp = t / (D / 2);
  float2 oacc[kDecodeRows];
#pragma unroll
  for (int u = 0; u < kDecodeRows; ++u) oacc[u] = make_float2(0.f, 0.f);

  constexpr int PIECES = D / 8;  // 16-byte pieces per row
  const int nblk = (key_hi - key_lo + kDecodeBlock - 1) / kDecodeBlock;
  // K (padded rows) and V of the 128 keys of block blk into buffer blk & 1, zeros past
  // the chunk end; the copies run while the previous block is being processed
  auto stage = [&](int blk) {
    const int kb = key_lo + blk * kDecodeBlock;
    uint8_t* kd = smem + S::OFF_K + (blk & 1) * S::KBUF;
    uint8_t* vd = smem + S::OFF_V + (blk & 1) * S::VBUF;
#pragma unroll
    for (int it = 0; it < PIECES; ++it) {
      const int idx = it * kDecodeBlock + t;
      const int j = idx / PIECES, pc = idx - j * PIECES;
      const bool ok = kb + j < key_hi;
      const size_t off = ok ? ((size_t)bg * p.Skv + kb + j) * D + pc * 8 : 0;
      cp_async16(kd + j * S::KROW + pc * 16, static_cast<const uint16_t*>(p.k) + off, ok);
      cp_async16(vd + (j * D + pc * 8) * 2, static_cast<const uint16_t*>(p.v) + off, ok);
    }
  };
  stage(nblk - 1);
  cp_async_commit();
  for (int blk = nblk - 1; blk >= 0; --blk) {
    const int kb = key_lo + blk * kDecodeBlock;
    const uint8_t* ks = smem + S::OFF_K + (blk & 1) * S::KBUF;
    const uint16_t* vs = reinterpret_cast<const uint16_t*>(smem + S::OFF_V + (blk & 1) * S::VBUF);
    if (blk > 0) stage(blk - 1);
    cp_async_commit();           // (an empty group on the last block keeps the count uniform)
    cp_async_wait_all_but_one();  // this block's copies have landed
    __syncthreads();              // ... for every thread; the row setup is visible too
    // ---- scores q_u . k_key: thread t = key kb + t, all rows
    const int key = kb + t;
    float sc[kDecodeRows];
#pragma unroll
    for (int u = 0; u < kDecodeRows; ++u) sc[u] = 0.f;
#pragma unroll 2
    for (int pc = 0; pc < PIECES; ++pc) {
      const uint4 kr = *reinterpret_cast<const uint4*>(ks + t * S::KROW + pc * 16);
      const float2 k01 = unpack2<BF16>(kr.x), k23 = unpack2<BF16>(kr.y);
      const float2 k45 = unpack2<BF16>(kr.z), k67 = unpack2<BF16>(kr.w);
#pragma unroll
      for (int u = 0; u < kDecodeRows; ++u) {
        if (u < R) {
          const float4 qa = *reinterpret_cast<const float4*>(qs + u * D + pc * 8);
          const float4 qb = *reinterpret_cast<const float4*>(qs + u * D + pc * 8 + 4);
          float2 acc = __fmul2_rn(make_float2(qa.x, qa.y), k01);
          acc = __ffma2_rn(make_float2(qa.z, qa.w), k23, acc);
          acc = __ffma2_rn(make_float2(qb.x, qb.y), k45, acc);
          acc = __ffma2_rn(make_float2(qb.z, qb.w), k67, acc);
          sc[u] += acc.x + acc.y;
        }
      }
    }
    // ---- sigmoids and the inclusive suffix sum within each warp (keys grow with the lane)
    float sf[kDecodeRows];
#pragma unroll
    for (int u = 0; u < kDecodeRows; ++u) {
      sf[u] = 0.f;
      if (u < R) {
        const bool vis = key < lim_s[u] && key < key_hi;
        float x = vis ? fmaf(0.5f, tanh_approx(c_t * sc[u]), 0.5f) : 0.f;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, x, off);
          if (lane + off < 32) x += y;
        }
        if (lane == 0) wsum[warp * kDecodeRows + u] = x;
        sf[u] = x;
      }
    }
    __syncthreads();
    // ---- logits a' = c_a p - slope2 z, z = suffix within the chunk; block maxima
#pragma unroll
    for (int u = 0; u < kDecodeRows; ++u) {
      if (u < R) {
        const bool vis = key < lim_s[u] && key < key_hi;
        float right = carry_s[u];
        for (int w = warp + 1; w < kDecodeBlock / 32; ++w) right += wsum[w * kDecodeRows + u];
        const float a = vis ? fmaf(c_a, sc[u], -slope_s[u] * (sf[u] + right)) : -INFINITY;
        sc[u] = a;
        float mx = a;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        if (lane == 0) wmax[warp * kDecodeRows + u] = mx;
      }
    }
    __syncthreads();
    // ---- exponentials against the running max; per-row rescale factor of O and l
    float fac[kDecodeRows];
#pragma unroll
    for (int u = 0; u < kDecodeRows; ++u) {
      fac[u] = 1.f;
      if (u < R) {
        float bm = wmax[u];
#pragma unroll
        for (int w = 1; w < kDecodeBlock / 32; ++w) bm = fmaxf(bm, wmax[w * kDecodeRows + u]);
        const float m_old = m_s[u];
        const float m_new = fmaxf(m_old, bm);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float e = (sc[u] == -INFINITY) ? 0.f : ex2_approx(sc[u] - m_use);
        es[t * kDecodeRows + u] = e;
        fac[u] = (m_old == -INFINITY) ? 0.f : ex2_approx(m_old - m_use);
        float ls = e;  // the block's row sum
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
        if (lane == 0) wl[warp * kDecodeRows + u] = ls;
      }
    }
    __syncthreads();  // every thread has read m_s and written es
    if (t < R) {
      float bm = wmax[t], tot = 0.f, ls = 0.f;
      for (int w = 0; w < kDecodeBlock / 32; ++w) {
        bm = fmaxf(bm, wmax[w * kDecodeRows + t]);
        tot += wsum[w * kDecodeRows + t];
        ls += wl[w * kDecodeRows + t];
      }
      const float m_old = m_s[t];
      const float m_use = (fmaxf(m_old, bm) == -INFINITY) ? 0.f : fmaxf(m_old, bm);
      l_s[t] = fmaf(l_s[t], (m_old == -INFINITY) ? 0.f : ex2_approx(m_old - m_use), ls);
      m_s[t] = fmaxf(m_old, bm);
      carry_s[t] += tot;
    }
    // ---- O += sum_j e_j v_j over this thread's key group, two dimensions
#pragma unroll
    for (int u = 0; u < kDecodeRows; ++u) oacc[u] = __fmul2_rn(oacc[u], make_float2(fac[u], fac[u]));
    const int j0 = kgrp * S::KPG;
#pragma unroll 4
    for (int jj = 0; jj < S::KPG; ++jj) {
      const int j = j0 + jj;
      const float2 vv = unpack2<BF16>(*reinterpret_cast<const uint32_t*>(vs + j * D + 2 * dpair));
#pragma unroll
      for (int u4 = 0; u4 < kDecodeRows / 4; ++u4) {
        if (u4 * 4 < R) {
          const float4 e = *reinterpret_cast<const float4*>(es + j * kDecodeRows + u4 * 4);
          oacc[u4 * 4 + 0] = __ffma2_rn(make_float2(e.x, e.x), vv, oacc[u4 * 4 + 0]);
          oacc[u4 * 4 + 1] = __ffma2_rn(make_float2(e.y, e.y), vv, oacc[u4 * 4 + 1]);
          oacc[u4 * 4 + 2] = __ffma2_rn(make_float2(e.z, e.z), vv, oacc[u4 * 4 + 2]);
          oacc[u4 * 4 + 3] = __ffma2_rn(make_float2(e.w, e.w), vv, oacc[u4 * 4 + 3]);
        }
      }
    }
    __syncthreads();  // every thread is done with this block's buffers before they are refilled
  }
  // fold the key groups into group 0 (the K buffers are free now)
  float* hx = reinterpret_cast<float*>(smem + S::OFF_K);
  if (kgrp > 0) {
#pragma unroll
    for (int u = 0; u < kDecodeRows; ++u)
      if (u < R) *reinterpret_cast<float2*>(hx + ((kgrp - 1) * kDecodeRows + u) * D + 2 * dpair) = oacc[u];
  }
  __syncthreads();
  if (kgrp == 0) {
    for (int gi = 1; gi < S::NGRP; ++gi) {
#pragma unroll
      for (int u = 0; u < kDecodeRows; ++u)
        if (u < R) {
          const float2 x = *reinterpret_cast<const float2*>(hx + ((gi - 1) * kDecodeRows + u) * D + 2 * dpair);
          oacc[u] = __fadd2_rn(oacc[u], x);
        }
    }
    const size_t rows = (size_t)p.B * p.Hq * p.Sq;
    float* stats = p.ws;
    float* obuf = p.ws + rows * p.n_chunks * 4;
#pragma unroll
    for (int u = 0; u < kDecodeRows; ++u) {
      if (u < R) {
        const int rr = r0 + u;
        const int h = g * G + rr / p.Sq, i = rr % p.Sq;
        const size_t row = ((size_t)b * p.Hq + h) * p.Sq + i;
        const size_t rec = row * p.n_chunks + c;
        *reinterpret_cast<float2*>(obuf + rec * D + 2 * dpair) = oacc[u];
        if (dpair == 0) *reinterpret_cast<float4*>(stats + rec * 4) = make_float4(carry_s[u], m_s[u], l_s[u], 0.f);
      }
    }
  }
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
