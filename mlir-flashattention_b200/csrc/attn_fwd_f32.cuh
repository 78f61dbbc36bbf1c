// attn_fwd_f32.cuh — fp32 attention forward on the CUDA cores (sm_100a).
//
// The reference op is f32 end to end (include/Attention/AttentionOps.td:36-41)
// and its users compare against it at 1e-4 relative tolerance, which TF32
// tensor-core inputs (10-bit mantissa) cannot meet.  This kernel keeps every
// product and sum in fp32 and follows the same online-softmax recurrence as
// lib/Attention/TilingPass.cpp:279-374 (running max, alpha rescale, running
// sum, final divide), with the general i1 mask operand supported
// (TilingPass.cpp:254-277: masked -> -inf).
//
// Layout: CTA = 4 warps = 4 query rows of one (batch, head) slice; keys are
// processed in chunks of 32 staged in shared memory (K with a padded row so
// lane-per-key dot products are bank-conflict free, V unpadded for
// lane-per-column accumulation).  Exponentials use expf.
#pragma once

#include <cstdint>

namespace attn_f32 {

struct F32Params {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  float* lse;
  const uint8_t* mask;
  int64_t q_sb, q_sh, q_sn;
  int64_t k_sb, k_sh, k_sn;
  int64_t v_sb, v_sh, v_sn;
  int64_t o_sb, o_sh, o_sn;
  int64_t m_sb, m_sh, m_sn;  // bytes
  int Hq, group, Nq, Nk, D;
  int mask_kind;  // 0 none, 1 causal, 2 dense
  float scale;
  int vec4;       // 1: K/V rows are 16-byte aligned with D % 4 == 0 (float4 staging)
};

constexpr int kRows = 4;
constexpr int kChunk = 32;

template <int DMAX>
__global__ void __launch_bounds__(kRows * 32)
    attn_fwd_f32_kernel(const F32Params p) {
  extern __shared__ float sm[];
  float* sK = sm;                                // [32][DMAX+1]
  float* sV = sK + kChunk * (DMAX + 1);          // [32][DMAX]
  float* sQ = sV + kChunk * DMAX;                // [4][DMAX]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh - (bh / p.Hq) * p.Hq, hk = h / p.group;
  const int row = blockIdx.x * kRows + warp;
  const bool live = row < p.Nq;
  const int D = p.D;

  const float* Q = p.q + b * p.q_sb + h * p.q_sh;
  const float* K = p.k + b * p.k_sb + hk * p.k_sh;
  const float* V = p.v + b * p.v_sb + hk * p.v_sh;
  for (int d = lane; d < D; d += 32) sQ[warp * DMAX + d] = live ? Q[row * p.q_sn + d] : 0.f;

  constexpr int NO = DMAX / 32;
  float o[NO];
#pragma unroll
  for (int i = 0; i < NO; ++i) o[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  // Dense masks: a row masked over all of keys [0, 128) (the reference's
  // first KV tile) is NaN in the reference, whose loop evaluates
  // exp(-inf - -inf) there (TilingPass.cpp:291-305).
  bool seen_first_tile = p.mask_kind != 2;

  int kend = p.Nk;
  if (p.mask_kind == 1) {
    // Keys beyond the last row of this CTA are masked for every row in it.
    const int last = min(blockIdx.x * kRows + kRows - 1, p.Nq - 1);
    kend = min(p.Nk, last + 1);
  }
  for (int k0 = 0; k0 < kend; k0 += kChunk) {
    __syncthreads();
    if (p.vec4) {
      // 16-byte loads, all of a thread's loads issued before any store.
      const int D4 = D >> 2;
      constexpr int kPer = (kChunk * DMAX / 4 + kRows * 32 - 1) / (kRows * 32);
      float4 kv[kPer], vv[kPer];
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = threadIdx.x + u * kRows * 32;
        const int kr = idx / D4, d4 = idx - (idx / D4) * D4;
        const int key = k0 + kr;
        const bool in = idx < kChunk * D4 && key < p.Nk;
        kv[u] = in ? __ldg(reinterpret_cast<const float4*>(K + key * p.k_sn) + d4)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
        vv[u] = in ? __ldg(reinterpret_cast<const float4*>(V + key * p.v_sn) + d4)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = threadIdx.x + u * kRows * 32;
        if (idx >= kChunk * D4) break;
        const int kr = idx / D4, d = (idx - (idx / D4) * D4) * 4;
        float* k_dst = sK + kr * (DMAX + 1) + d;  // padded rows: scalar stores
        k_dst[0] = kv[u].x; k_dst[1] = kv[u].y; k_dst[2] = kv[u].z; k_dst[3] = kv[u].w;
        *reinterpret_cast<float4*>(sV + kr * DMAX + d) = vv[u];
      }
    } else {
      for (int idx = threadIdx.x; idx < kChunk * D; idx += blockDim.x) {
        const int kr = idx / D, d = idx - (idx / D) * D;
        const int key = k0 + kr;
        const bool in = key < p.Nk;
        sK[kr * (DMAX + 1) + d] = in ? K[key * p.k_sn + d] : 0.f;
        sV[kr * DMAX + d] = in ? V[key * p.v_sn + d] : 0.f;
      }
    }
    __syncthreads();
    const int key = k0 + lane;
    float s = 0.f;
    for (int d = 0; d < D; ++d) s = fmaf(sQ[warp * DMAX + d], sK[lane * (DMAX + 1) + d], s);
    s *= p.scale;
    bool masked = key >= p.Nk;
    if (p.mask_kind == 1) masked = masked || key > row;
    if (p.mask_kind == 2 && live && key < p.Nk)
      masked = masked || p.mask[b * p.m_sb + h * p.m_sh + row * p.m_sn + key] != 0;
    if (masked) s = -INFINITY;
    if (k0 < 128) seen_first_tile |= __any_sync(0xffffffffu, !masked);
    float mx = s;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m, mx);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = expf(m - m_use);
    const float pr = expf(s - m_use);
    float ps = pr;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    l = l * alpha + ps;
#pragma unroll
    for (int i = 0; i < NO; ++i) o[i] *= alpha;
    for (int kr = 0; kr < kChunk; ++kr) {
      const float pk = __shfl_sync(0xffffffffu, pr, kr);
#pragma unroll
      for (int i = 0; i < NO; ++i) {
        const int d = lane + 32 * i;
        if (d < D) o[i] = fmaf(pk, sV[kr * DMAX + d], o[i]);
      }
    }
    m = m_new;
  }
  if (live) {
    const float nan = __int_as_float(0x7fc00000);
    float* O = p.o + b * p.o_sb + h * p.o_sh + row * p.o_sn;
#pragma unroll
    for (int i = 0; i < NO; ++i) {
      const int d = lane + 32 * i;
      if (d < D) O[d] = seen_first_tile ? o[i] / l : nan;
    }
    if (p.lse && lane == 0)
      p.lse[static_cast<int64_t>(bh) * p.Nq + row] = seen_first_tile ? m + logf(l) : nan;
  }
}

template <int DMAX>
constexpr size_t f32_smem_bytes() {
  return sizeof(float) * (kChunk * (DMAX + 1) + kChunk * DMAX + kRows * DMAX);
}

// Register-tiled variant for head_dim 64 / 128 with 16-byte aligned rows.
// CTA = 128 threads on a 64-row Q tile; key blocks of 64.  Thread (ty, tx),
// ty = tid / 16, tx = tid % 16, owns S rows 8·ty.. +8 and keys 4·tx.. +4 of
// each block (32 scores in registers) and O rows 8·ty.. +8, columns
// (D/16)·tx.. of the output.  Q and K sit transposed in shared memory, so a
// score step is two broadcast float4 loads of Q, one float4 of K and 32 FMAs;
// P goes through shared memory row-major for the P·V step (8 broadcast loads
// of P, D/64 float4 loads of V and 8·D/16 FMAs per key).  Same recurrence,
// masks and NaN rules as attn_fwd_f32_kernel; the first KV tile of the
// reference (keys [0, 128)) spans two key blocks here.
constexpr int kTBM = 64, kTBN = 64, kTThreads = 128;

template <int D>
constexpr size_t f32_tiled_smem_bytes() {
  return sizeof(float) * (D * kTBM + D * kTBN + kTBN * D + kTBM * (kTBN + 1));
}

template <int D>
__global__ void __launch_bounds__(kTThreads)
    attn_fwd_f32_tiled(const F32Params p) {
  constexpr int TN = D / 16;  // output columns per thread
  extern __shared__ float4 smem4[];
  float* sQt = reinterpret_cast<float*>(smem4);  // [D][64]
  float* sKt = sQt + D * kTBM;                    // [D][64]
  float* sV = sKt + D * kTBN;                     // [64][D]
  float* sP = sV + kTBN * D;                      // [64][64 + 1]
  // Row pitch 65: the two row groups a warp reads in the P·V loop (8 rows
  // apart) fall in different banks.
  constexpr int PLD = kTBN + 1;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh - (bh / p.Hq) * p.Hq, hk = h / p.group;
  const int q0 = blockIdx.x * kTBM;
  const float* Q = p.q + b * p.q_sb + h * p.q_sh;
  const float* K = p.k + b * p.k_sb + hk * p.k_sh;
  const float* V = p.v + b * p.v_sb + hk * p.v_sh;
  constexpr int D4 = D / 4;
  // Q tile, transposed: consecutive threads take consecutive rows.
  for (int i = tid; i < kTBM * D4; i += kTThreads) {
    const int r = i % kTBM, d4 = i / kTBM;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < p.Nq) v = __ldg(reinterpret_cast<const float4*>(Q + (q0 + r) * p.q_sn) + d4);
    sQt[(4 * d4 + 0) * kTBM + r] = v.x;
    sQt[(4 * d4 + 1) * kTBM + r] = v.y;
    sQt[(4 * d4 + 2) * kTBM + r] = v.z;
    sQt[(4 * d4 + 3) * kTBM + r] = v.w;
  }
  float o[8][TN];
  float m[8], l[8];
  bool seen[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    seen[i] = p.mask_kind != 2;
#pragma unroll
    for (int c = 0; c < TN; ++c) o[i][c] = 0.f;
  }
  int kend = p.Nk;
  if (p.mask_kind == 1) kend = min(p.Nk, min(q0 + kTBM, p.Nq));  // keys past the last row
  for (int k0 = 0; k0 < kend; k0 += kTBN) {
    __syncthreads();  // the previous block's K, V and P reads are done
    for (int i = tid; i < kTBN * D4; i += kTThreads) {  // K transposed
      const int kr = i % kTBN, d4 = i / kTBN;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + kr < p.Nk) v = __ldg(reinterpret_cast<const float4*>(K + (k0 + kr) * p.k_sn) + d4);
      sKt[(4 * d4 + 0) * kTBN + kr] = v.x;
      sKt[(4 * d4 + 1) * kTBN + kr] = v.y;
      sKt[(4 * d4 + 2) * kTBN + kr] = v.z;
      sKt[(4 * d4 + 3) * kTBN + kr] = v.w;
    }
    for (int i = tid; i < kTBN * D4; i += kTThreads) {  // V row-major
      const int kr = i / D4, d4 = i % D4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + kr < p.Nk) v = __ldg(reinterpret_cast<const float4*>(V + (k0 + kr) * p.v_sn) + d4);
      *reinterpret_cast<float4*>(sV + kr * D + 4 * d4) = v;
    }
    __syncthreads();
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; ++d) {
      const float4 a0 = *reinterpret_cast<const float4*>(sQt + d * kTBM + ty * 8);
      const float4 a1 = *reinterpret_cast<const float4*>(sQt + d * kTBM + ty * 8 + 4);
      const float4 kb = *reinterpret_cast<const float4*>(sKt + d * kTBN + tx * 4);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float kk[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[i][j] = fmaf(a[i], kk[j], sc[i][j]);
    }
    // scale, mask, online softmax per row (16 threads share a row)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = q0 + ty * 8 + i;
      const uint8_t* mrow = nullptr;
      if (p.mask_kind == 2 && row < p.Nq) mrow = p.mask + b * p.m_sb + h * p.m_sh + row * p.m_sn;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = k0 + tx * 4 + j;
        bool masked = key >= p.Nk;
        if (p.mask_kind == 1) masked = masked || key > row;
        if (mrow && key < p.Nk) masked = masked || mrow[key] != 0;
        if (key < 128 && !masked) seen[i] = true;
        const float v = sc[i][j] * p.scale;
        sc[i][j] = masked ? -INFINITY : v;
        mx = fmaxf(mx, sc[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m[i], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = expf(m[i] - m_use);
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[i][j] = expf(sc[i][j] - m_use);
        ps += sc[i][j];
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[i] = l[i] * alpha + ps;
#pragma unroll
      for (int c = 0; c < TN; ++c) o[i][c] *= alpha;
      m[i] = m_new;
#pragma unroll
      for (int j = 0; j < 4; ++j) sP[(ty * 8 + i) * PLD + tx * 4 + j] = sc[i][j];
    }
    __syncthreads();
#pragma unroll 2
    for (int kr = 0; kr < kTBN; ++kr) {
      float pv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pv[i] = sP[(ty * 8 + i) * PLD + kr];
      float vv[TN];
#pragma unroll
      for (int c4 = 0; c4 < TN / 4; ++c4) {
        const float4 v = *reinterpret_cast<const float4*>(sV + kr * D + tx * TN + 4 * c4);
        vv[4 * c4] = v.x; vv[4 * c4 + 1] = v.y; vv[4 * c4 + 2] = v.z; vv[4 * c4 + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < TN; ++c) o[i][c] = fmaf(pv[i], vv[c], o[i][c]);
    }
  }
  const float nan = __int_as_float(0x7fc00000);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // The 16 threads of a row hold the same statistics; OR `seen` over them
    // (lanes 0-15 hold one row of the warp, lanes 16-31 the other).
    unsigned grp = __ballot_sync(0xffffffffu, seen[i]);
    grp = (ty & 1) ? (grp >> 16) : (grp & 0xffffu);
    const bool row_seen = grp != 0u;
    const int row = q0 + ty * 8 + i;
    if (row >= p.Nq) continue;
    float* O = p.o + b * p.o_sb + h * p.o_sh + row * p.o_sn + tx * TN;
#pragma unroll
    for (int c4 = 0; c4 < TN / 4; ++c4) {
      float4 r;
      r.x = row_seen ? o[i][4 * c4] / l[i] : nan;
      r.y = row_seen ? o[i][4 * c4 + 1] / l[i] : nan;
      r.z = row_seen ? o[i][4 * c4 + 2] / l[i] : nan;
      r.w = row_seen ? o[i][4 * c4 + 3] / l[i] : nan;
      *reinterpret_cast<float4*>(O + 4 * c4) = r;
    }
    if (p.lse && tx == 0)
      p.lse[static_cast<int64_t>(bh) * p.Nq + row] = row_seen ? m[i] + logf(l[i]) : nan;
  }
}

}  // namespace attn_f32
