// attn_fwd_sm100.cuh — fused attention forward for B200 (sm_100a).
//
// Computes, for every (batch, q-head) slice, the `attention.fused` op of the
// reference (include/Attention/AttentionOps.td:20-54):
//     O = softmax(Q·Kᵀ·scale, masked -> -inf) · V
// with the online-softmax recurrence its TilingPass emits
// (lib/Attention/TilingPass.cpp:279-374: running max m, running sum l, O
// rescaled by alpha = exp(m_old - m_new)), restated for the tensor cores:
//
//   CTA = two Q tiles of 128 rows (256 query rows) of one slice.
//   warp 8      TMA producer: Q tiles once, then K_j / V_j tiles (128 keys)
//               through an NS-stage shared-memory ring (mbarrier full/empty).
//   warp 9      MMA issuer (one thread): S_t = Q_t·K_jᵀ into TMEM (SS form),
//               O_t += P_t·V_j with P_t read from TMEM (TS form).
//   warps 0-3   softmax for Q tile 0, warps 4-7 for Q tile 1: one thread per
//               query row reads its S row from TMEM, applies the mask, updates
//               (m, l) in registers, writes P (bf16 / e4m3) back into the S
//               columns and rescales its O row in TMEM when m moved.
//   The two Q tiles ping-pong: while one softmax group works, the tensor
//   cores run the other tile's GEMMs.
//
// TMEM (512 columns): S0/P0 [0,128) S1/P1 [128,256) O0 [256,256+D)
// O1 [256+D, 256+2D).  Exponentials are base 2 with the scale folded in:
// p = 2^(s·scale·log2e − m).  The running max only moves when it grows by
// more than 2^8 (values of p stay <= 256, exact in bf16/e4m3 range), which
// skips most O rescales; the final O/l and LSE are unaffected by the choice.
//
// Causal (the mask mask[i][j] = j > i): KV tiles wholly above the diagonal
// are never loaded or multiplied (the FULL / MASKED / BOUNDARY tile split of
// the reference design, Design.md:412-419); only diagonal and ragged-edge
// tiles apply a per-element mask.
//
// Hang safety: every mbarrier wait is bounded (wall-clock limit); on expiry
// the CTA records ATTN_ERR_TIMEOUT in the status word, all roles leave their
// loops, in-flight TMA and MMA work is drained (again bounded) and TMEM is
// freed before the CTA exits.
#pragma once

#include "sm100_ptx.cuh"

namespace attn_sm100 {

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait

struct FwdParams {
  void* o;
  int64_t o_sb, o_sh, o_sn;  // element strides of O
  float* lse;                // [B, Hq, Nq] or null
  int32_t* status;
  int Hq, group, Nq, Nk;
  int num_pairs;             // ceil(Nq / 256)
  float scale_log2;          // scale * log2(e) (* q/k descales for e4m3)
  float o_scale;             // v descale for e4m3, else 1
  int out_f32;               // 1: O is fp32, 0: O is bf16
};

template <int D, bool FP8>
struct FwdCfg {
  static constexpr int kEB = FP8 ? 1 : 2;               // bytes per input element
  static constexpr int kBoxCols = 128 / kEB;            // elements per 128-byte row
  static constexpr int kNBox = (D * kEB) / 128;         // 128-byte column boxes per tile
  static constexpr int kBoxBytes = 128 * 128;           // 128 rows x 128 bytes
  static constexpr int kTileBytes = kNBox * kBoxBytes;  // one 128-row tile
  static constexpr int kStages = (FP8 || D == 64) ? 8 : 4;
  static constexpr int kKStepsS = (D * kEB) / 32;       // 32 bytes of K per MMA
  static constexpr int kKeysPerStep = 32 / kEB;         // keys per P·V MMA
  static constexpr int kKStepsPV = 128 / kKeysPerStep;
  static constexpr uint32_t kFmt = FP8 ? 0u : 1u;       // e4m3 : bf16
  static constexpr int kKind = FP8 ? 1 : 0;
  static constexpr int kPCols = 128 * kEB / 4;          // TMEM columns holding P
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 1;
  static constexpr size_t kSmemBytes =
      1024 /*align slack*/ + 2 * kTileBytes + kStages * kTileBytes + kNumBars * 8 + 16;
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(kNBox >= 1, "tile must span at least one 128-byte box");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

constexpr int kThreads = 320;

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// Warp-uniform bounded wait: every lane waits, the warp agrees on the result.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* status) {
  bool ok = mbar_wait_bounded(bar, parity, abort, status, kWaitLimitNs);
  return __all_sync(0xffffffffu, ok);
}

// Drain wait: ignores the abort flag (waits for this CTA's own copies / MMAs
// in flight), still bounded in time.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* status) {
  int never = 0;
  mbar_wait_bounded(bar, parity, &never, status, kWaitLimitNs);
}

template <int D, bool CAUSAL, bool FP8>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using C = FwdCfg<D, FP8>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + 2 * C::kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + C::kStages * C::kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + C::kStages;
  uint64_t* s_full = kv_empty + C::kStages;
  uint64_t* p_ready = s_full + 2;
  uint64_t* pv_done = p_ready + 2;
  uint64_t* drain = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x;  // flat (batch, q-head)
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int hk = h / p.group;
  // Causal: heaviest Q tiles first (longest-processing-time order).
  const int pair = CAUSAL ? (p.num_pairs - 1 - static_cast<int>(blockIdx.y))
                          : static_cast<int>(blockIdx.y);
  const int q0 = pair * 256;
  const int nkv_all = cdiv(p.Nk, 128);
  int n_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = q0 + 128 * t;
    if (qs >= p.Nq) {
      n_t[t] = 0;
    } else if (CAUSAL) {
      const int last_row = min(qs + 127, p.Nq - 1);
      n_t[t] = min(nkv_all, last_row / 128 + 1);
    } else {
      n_t[t] = nkv_all;
    }
  }
  const int nmax = max(n_t[0], n_t[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 128);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, 2 * C::kTileBytes);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < C::kNBox; ++c)
          tma_load_4d(sQ + t * C::kTileBytes + c * C::kBoxBytes, &tmQ, q_full, c * C::kBoxCols,
                      q0 + 128 * t, h, b);
      int it = 0;
      bool ok = true;
      for (int j = 0; j < nmax && ok; ++j) {
#pragma unroll
        for (int kv = 0; kv < 2; ++kv) {
          const int s = it % C::kStages;
          const uint32_t u = static_cast<uint32_t>(it / C::kStages);
          if (!mbar_wait_bounded(&kv_empty[s], (u & 1u) ^ 1u, abort_flag, p.status,
                                 kWaitLimitNs)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[s], C::kTileBytes);
#pragma unroll
          for (int c = 0; c < C::kNBox; ++c)
            tma_load_4d(sKV + s * C::kTileBytes + c * C::kBoxBytes, kv ? &tmV : &tmK,
                        &kv_full[s], c * C::kBoxCols, j * 128, hk, b);
          ++it;
        }
      }
      // Wait for every copy this thread started before the CTA may exit.
      drain_wait(q_full, 0, p.status);
      for (int s = 0; s < C::kStages; ++s) {
        if (it > s) {
          const int armed = (it - 1 - s) / C::kStages + 1;
          drain_wait(&kv_full[s], static_cast<uint32_t>((armed - 1) & 1), p.status);
        }
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc(128, 128, C::kFmt, false);
      constexpr uint32_t idO = make_idesc(128, D, C::kFmt, true);
      const uint32_t sQa = smem_u32(sQ);
      const uint32_t sKVa = smem_u32(sKV);
      auto issue_S = [&](int t, int stage) {
#pragma unroll
        for (int kk = 0; kk < C::kKStepsS; ++kk) {
          const uint32_t kb = kk * 32;
          const uint32_t off = (kb / 128) * C::kBoxBytes + (kb % 128);
          const uint64_t a = make_sdesc(sQa + t * C::kTileBytes + off, 16, 1024);
          const uint64_t bd = make_sdesc(sKVa + stage * C::kTileBytes + off, 16, 1024);
          mma_ss<C::kKind>(tmem + t * 128, a, bd, idS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_PV = [&](int t, int stage, bool acc) {
#pragma unroll
        for (int kk = 0; kk < C::kKStepsPV; ++kk) {
          const uint64_t bd = make_sdesc(
              sKVa + stage * C::kTileBytes + kk * C::kKeysPerStep * 128, C::kBoxBytes, 1024);
          mma_ts<C::kKind>(tmem + 256 + t * D, tmem + t * 128 + kk * 8, bd, idO,
                           (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, p.status, kWaitLimitNs) &&
                mbar_wait_bounded(&kv_full[0], 0, abort_flag, p.status, kWaitLimitNs);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (n_t[t] > 0) {
            issue_S(t, 0);
            mma_commit(&s_full[t]);
          }
        mma_commit(&kv_empty[0]);  // K_0 is free once both S GEMMs finish
      }
      // Per KV step j, for each Q tile t in turn: O_t += P_t(j)·V_j, then
      // S_t(j+1) = Q_t·K_{j+1}ᵀ as soon as that P·V GEMM has finished reading
      // P_t(j) (P lives in the S_t columns).  Tile t's next softmax can then
      // start while the tensor cores run the other tile's GEMMs, so the two
      // softmax warpgroups alternate with the tensor pipe.
      for (int j = 0; j < nmax && ok; ++j) {
        const int vs = (2 * j + 1) % C::kStages;
        const uint32_t vu = static_cast<uint32_t>((2 * j + 1) / C::kStages);
        const int nks = (2 * j + 2) % C::kStages;
        const uint32_t nku = static_cast<uint32_t>((2 * j + 2) / C::kStages);
        bool k_next = false;
        if (!mbar_wait_bounded(&kv_full[vs], vu & 1u, abort_flag, p.status, kWaitLimitNs)) {
          ok = false;
          break;
        }
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= n_t[t]) continue;
          if (!mbar_wait_bounded(&p_ready[t], static_cast<uint32_t>(j & 1), abort_flag, p.status,
                                 kWaitLimitNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_PV(t, vs, j > 0);
          mma_commit(&pv_done[t]);
          if (j + 1 < n_t[t]) {
            if (!k_next) {
              if (!mbar_wait_bounded(&kv_full[nks], nku & 1u, abort_flag, p.status,
                                     kWaitLimitNs)) {
                ok = false;
                break;
              }
              k_next = true;
            }
            if (!mbar_wait_bounded(&pv_done[t], static_cast<uint32_t>(j & 1), abort_flag,
                                   p.status, kWaitLimitNs)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_S(t, nks);
            mma_commit(&s_full[t]);
          }
        }
        if (!ok) break;
        mma_commit(&kv_empty[vs]);  // V_j is free once the P·V GEMMs finish
        if (j + 1 < nmax) {
          if (!k_next &&
              !mbar_wait_bounded(&kv_full[nks], nku & 1u, abort_flag, p.status, kWaitLimitNs)) {
            ok = false;
            break;
          }
          mma_commit(&kv_empty[nks]);  // K_{j+1} is free once its S GEMMs finish
        }
      }
      // Drain every MMA this thread issued before TMEM is released.
      mma_commit(drain);
      drain_wait(drain, 0, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;  // Q tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + 256 + t * D;
    const int qs = q0 + 128 * t;
    const int row = qs + r;
    const int n = n_t[t];
    const float sl2 = p.scale_log2;
    const bool pos = sl2 >= 0.f;
    const float mask_val = pos ? -INFINITY : INFINITY;
    float m = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(&s_full[t], static_cast<uint32_t>(j & 1), abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(tS + 0, r0);
        tmem_ld32(tS + 32, r1);
        tmem_ld32(tS + 64, r2);
        tmem_ld32(tS + 96, r3);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(r0[i]);
          s[32 + i] = __uint_as_float(r1[i]);
          s[64 + i] = __uint_as_float(r2[i]);
          s[96 + i] = __uint_as_float(r3[i]);
        }
      }
      const int kbase = j * 128;
      const bool edge = (kbase + 128 > p.Nk) || (CAUSAL && kbase + 127 > qs);
      if (edge) {
        const int lim = CAUSAL ? min(row + 1, p.Nk) : p.Nk;  // keys < lim are visible
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (kbase + c >= lim) s[c] = mask_val;
      }
      float red;
      if (pos) {
        float a0 = fmaxf(s[0], s[1]), a1 = fmaxf(s[2], s[3]);
#pragma unroll
        for (int c = 4; c < 128; c += 4) {
          a0 = fmaxf(a0, fmaxf(s[c], s[c + 1]));
          a1 = fmaxf(a1, fmaxf(s[c + 2], s[c + 3]));
        }
        red = fmaxf(a0, a1);
      } else {
        float a0 = fminf(s[0], s[1]), a1 = fminf(s[2], s[3]);
#pragma unroll
        for (int c = 4; c < 128; c += 4) {
          a0 = fminf(a0, fminf(s[c], s[c + 1]));
          a1 = fminf(a1, fminf(s[c + 2], s[c + 3]));
        }
        red = fminf(a0, a1);
      }
      const float m_cand = red * sl2;
      float alpha = 1.f;
      if (m_cand > m + 8.f) {  // m = -inf: any finite candidate moves it
        alpha = ex2(m - m_cand);
        m = m_cand;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      float sum0 = 0.f, sum1 = 0.f;
      if constexpr (!FP8) {
        uint32_t pk[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p0 = ex2(fmaf(s[2 * c], sl2, neg_m));
          const float p1 = ex2(fmaf(s[2 * c + 1], sl2, neg_m));
          sum0 += p0;
          sum1 += p1;
          pk[c] = pack_bf16(p0, p1);
        }
        tmem_st32(tS + 0, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
        tmem_st32(tS + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
      } else {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p0 = ex2(fmaf(s[4 * c], sl2, neg_m));
          const float p1 = ex2(fmaf(s[4 * c + 1], sl2, neg_m));
          const float p2 = ex2(fmaf(s[4 * c + 2], sl2, neg_m));
          const float p3 = ex2(fmaf(s[4 * c + 3], sl2, neg_m));
          sum0 += p0 + p2;
          sum1 += p1 + p3;
          pk[c] = pack_e4m3x4(p0, p1, p2, p3);
        }
        tmem_st32(tS + 0, pk);
      }
      l = l * alpha + (sum0 + sum1);
      const bool need = (j > 0) && (alpha != 1.f);
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_ready[t]);
    }
    // ---------------------------------------------------------- epilogue
    if (ok && n > 0 && warp_wait(&pv_done[t], static_cast<uint32_t>((n - 1) & 1), abort_flag,
                                 p.status)) {
      tc_fence_after();
      const float inv_l = p.o_scale / l;
      const int64_t obase = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh +
                            static_cast<int64_t>(row) * p.o_sn;
      const bool live = row < p.Nq;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
        if (live) {
          if (p.out_f32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.o) + obase + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l,
                                   __uint_as_float(o[4 * i + 1]) * inv_l,
                                   __uint_as_float(o[4 * i + 2]) * inv_l,
                                   __uint_as_float(o[4 * i + 3]) * inv_l);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.o) + obase + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 v;
              v.x = pack_bf16(__uint_as_float(o[8 * i + 0]) * inv_l,
                              __uint_as_float(o[8 * i + 1]) * inv_l);
              v.y = pack_bf16(__uint_as_float(o[8 * i + 2]) * inv_l,
                              __uint_as_float(o[8 * i + 3]) * inv_l);
              v.z = pack_bf16(__uint_as_float(o[8 * i + 4]) * inv_l,
                              __uint_as_float(o[8 * i + 5]) * inv_l);
              v.w = pack_bf16(__uint_as_float(o[8 * i + 6]) * inv_l,
                              __uint_as_float(o[8 * i + 7]) * inv_l);
              dst[i] = v;
            }
          }
        }
      }
      if (live && p.lse)
        p.lse[static_cast<int64_t>(bh) * p.Nq + row] = (m + __log2f(l)) * 0.69314718055994531f;
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn_sm100
