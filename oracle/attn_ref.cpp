// attn_ref.cpp — TEST INFRASTRUCTURE ONLY (the oracle).  Nothing in the product
// links this file; only tests/, __graft_entry__.smoke() and bench.py's CPU legs
// load it, as the checker and as the timed CPU baseline.
//
// A CPU restatement of the reference's lowering of `attention.fused`
// (luisroayerdi/MLIR-FlashAttention, lib/Attention/TilingPass.cpp:155-392),
// written loop for loop so that every output element sees the same sequence of
// IEEE-754 single-precision operations the lowered MLIR performs:
//   * Q-tile outer loop, KV-tile inner loop, tile T (TilingPass.cpp:188,208;
//     default T = 128, AttentionPasses.td:45-50);
//   * O_acc = 0, m_acc = -inf, l_acc = 0 per Q tile (TilingPass.cpp:193-202);
//   * S = Q·Kᵀ as `acc = acc + q*k` over d in order from 0.0
//     (TilingPass.cpp:219-241), then S = S*scale in a separate pass (:244-249);
//   * mask select: masked -> -inf (:254-277);
//   * m_tile = maximumf-reduce from -inf (:282-288), m_new = maximumf(m_acc,
//     m_tile) (:291-296), alpha = exp(m_acc - m_new) (:299-305),
//     P = exp(S - m_new) (:308-323), P_sum = 0 + P... (:326-332),
//     l_new = alpha*l_acc + P_sum (:335-341), O_acc = alpha*O_acc (:344-347),
//     O_acc = O_acc + P*V over s in order (:351-370), state copy (:373-374);
//   * O = O_acc / l_acc, copied out (:379-386).
// `math.exp` lowers to the C library's expf, so std::exp(float) is used.
// Build with -ffp-contract=off: MLIR's arith ops without fast-math flags are
// never fused into FMAs.  Loops are ordered so the compiler may vectorise
// ACROSS output elements while each element's own reduction order is unchanged
// (the S and PV reductions run over d and s in ascending order for every
// element), so results are bit-identical to the scalar loop nest.
//
// Extensions beyond the reference op (which is rank-2 f32 with an explicit i1
// mask): batch x head slices with grouped-query head mapping (kv head =
// q head / (Hq/Hkv)); causal masking computed on the fly (equal to passing the
// i1 mask mask[i][j] = j > i); partial edge tiles (the reference requires N to
// be a multiple of T and reads out of bounds otherwise — here keys beyond Nk do
// not exist and rows beyond Nq are not computed); and LSE = m_acc + log(l_acc).
//
// Parity status: the reference ships no numeric test, golden vector or
// runnable CPU pipeline (no MLIR in this environment), so this restatement is
// "parity unpinned" against the reference binary; it is pinned against
// known-answer cases and an independent float64 two-pass softmax in tests/.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// arith.maximumf: IEEE-754-2019 maximum — NaN propagates, -0 < +0.
inline float maximumf(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  if (a == 0.0f && b == 0.0f) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}

struct SliceArgs {
  const float* Q;  // [Nq, D] row stride ldq
  const float* K;  // [Nk, D] row stride ldk
  const float* V;  // [Nk, D] row stride ldv
  float* O;        // [Nq, D] row stride ldo
  float* lse;      // [Nq] or null
  const uint8_t* mask;  // [Nq, Nk] row stride ldm (bytes) or null
  int64_t ldq, ldk, ldv, ldo, ldm;
  int64_t Nq, Nk, D;
  float scale;
  int causal;
  int64_t T;
};

// One Q tile [i0, i0+rows) of one slice: the body of the outer affine.for.
__attribute__((target_clones("avx512f", "avx2", "default")))
void q_tile(const SliceArgs& a, int64_t i0) {
  const int64_t T = a.T, D = a.D;
  const int64_t rows = std::min<int64_t>(T, a.Nq - i0);
  const float ninf = -std::numeric_limits<float>::infinity();

  std::vector<float> O_acc(static_cast<size_t>(rows * D), 0.0f);
  std::vector<float> m_acc(static_cast<size_t>(rows), ninf);
  std::vector<float> l_acc(static_cast<size_t>(rows), 0.0f);
  std::vector<float> S(static_cast<size_t>(rows * T));
  std::vector<float> Kt(static_cast<size_t>(D * T));
  std::vector<float> m_tile(static_cast<size_t>(rows)), m_new(static_cast<size_t>(rows)),
      alpha(static_cast<size_t>(rows)), P_sum(static_cast<size_t>(rows)),
      l_new(static_cast<size_t>(rows));

  for (int64_t j0 = 0; j0 < a.Nk; j0 += T) {
    const int64_t cols = std::min<int64_t>(T, a.Nk - j0);
    // K tile transposed into Kt[d][c] (a copy, no arithmetic) so the S loop
    // below runs unit-stride across c.
    for (int64_t c = 0; c < cols; ++c)
      for (int64_t d = 0; d < D; ++d) Kt[d * T + c] = a.K[(j0 + c) * a.ldk + d];

    // 1. S_tile = 0; S[r,c] = S[r,c] + Q[r,d]*K[c,d], d ascending.
    for (int64_t r = 0; r < rows; ++r) {
      float* Sr = &S[r * T];
      for (int64_t c = 0; c < cols; ++c) Sr[c] = 0.0f;
      const float* Qr = a.Q + (i0 + r) * a.ldq;
      for (int64_t d = 0; d < D; ++d) {
        const float q = Qr[d];
        const float* Kd = &Kt[d * T];
        for (int64_t c = 0; c < cols; ++c) {
          const float prod = q * Kd[c];
          Sr[c] = Sr[c] + prod;
        }
      }
    }
    // 2. S *= scale.
    for (int64_t r = 0; r < rows; ++r) {
      float* Sr = &S[r * T];
      for (int64_t c = 0; c < cols; ++c) Sr[c] = Sr[c] * a.scale;
    }
    // 3. Mask select: masked -> -inf.
    if (a.mask) {
      for (int64_t r = 0; r < rows; ++r) {
        const uint8_t* Mr = a.mask + (i0 + r) * a.ldm + j0;
        float* Sr = &S[r * T];
        for (int64_t c = 0; c < cols; ++c) Sr[c] = Mr[c] ? ninf : Sr[c];
      }
    } else if (a.causal) {
      for (int64_t r = 0; r < rows; ++r) {
        float* Sr = &S[r * T];
        for (int64_t c = 0; c < cols; ++c) Sr[c] = (j0 + c > i0 + r) ? ninf : Sr[c];
      }
    }
    // 4. Online softmax update.
    for (int64_t r = 0; r < rows; ++r) {
      const float* Sr = &S[r * T];
      float mt = ninf;
      for (int64_t c = 0; c < cols; ++c) mt = maximumf(Sr[c], mt);
      m_tile[r] = mt;
      m_new[r] = maximumf(m_acc[r], m_tile[r]);
      alpha[r] = std::exp(m_acc[r] - m_new[r]);
    }
    for (int64_t r = 0; r < rows; ++r) {
      float* Sr = &S[r * T];  // reused as P_tile
      const float mn = m_new[r];
      for (int64_t c = 0; c < cols; ++c) Sr[c] = std::exp(Sr[c] - mn);
      float ps = 0.0f;
      for (int64_t c = 0; c < cols; ++c) ps = ps + Sr[c];
      P_sum[r] = ps;
      l_new[r] = alpha[r] * l_acc[r] + P_sum[r];
    }
    // O_acc[r,:] = alpha[r] * O_acc[r,:]
    for (int64_t r = 0; r < rows; ++r) {
      float* Or = &O_acc[r * D];
      const float al = alpha[r];
      for (int64_t d = 0; d < D; ++d) Or[d] = al * Or[d];
    }
    // O_acc[r,c] = O_acc[r,c] + P[r,s]*V[s,c], s ascending.
    for (int64_t r = 0; r < rows; ++r) {
      float* Or = &O_acc[r * D];
      const float* Pr = &S[r * T];
      for (int64_t s = 0; s < cols; ++s) {
        const float p = Pr[s];
        const float* Vs = a.V + (j0 + s) * a.ldv;
        for (int64_t d = 0; d < D; ++d) {
          const float pv = p * Vs[d];
          Or[d] = Or[d] + pv;
        }
      }
    }
    for (int64_t r = 0; r < rows; ++r) {
      m_acc[r] = m_new[r];
      l_acc[r] = l_new[r];
    }
  }
  // Final rescale and copy-out.
  for (int64_t r = 0; r < rows; ++r) {
    float* dst = a.O + (i0 + r) * a.ldo;
    const float* Or = &O_acc[r * D];
    const float lv = l_acc[r];
    for (int64_t d = 0; d < D; ++d) dst[d] = Or[d] / lv;
    if (a.lse) a.lse[i0 + r] = m_acc[r] + std::log(l_acc[r]);
  }
}

}  // namespace

extern "C" {

// Rank-2 form of the reference op: Q [Nq,D], K/V [Nk,D], O [Nq,D], all
// contiguous f32; mask [Nq,Nk] bytes (1 = masked) or null; lse optional.
int oracle_attn_fused_f32(const float* Q, const float* K, const float* V, float scale,
                          const uint8_t* mask, int causal, float* O, float* lse, int64_t Nq,
                          int64_t Nk, int64_t D, int64_t T) {
  // Empty extents run the same loop nest: no query row does nothing; no key
  // leaves O_acc = 0 and l = 0, so O = 0/0 = NaN and LSE = -inf.
  if (Nq < 0 || Nk < 0 || D <= 0 || T <= 0) return -1;
  if (Nq == 0) return 0;
  if (!Q || !O || (Nk > 0 && (!K || !V))) return -1;
  SliceArgs a{Q, K, V, O, lse, mask, D, D, D, D, Nk, Nq, Nk, D, scale, causal, T};
  for (int64_t i0 = 0; i0 < Nq; i0 += T) q_tile(a, i0);
  return 0;
}

// Batched form over contiguous [B,H,N,D] f32 arrays with grouped-query heads.
// Work items are (slice, q-tile) pairs, optionally restricted to the listed
// slices (`slices`, `nslices` > 0) and to every `tile_stride`-th q tile
// starting at `tile_offset` (used to time a bounded sample).  Runs on
// `nthreads` OpenMP threads (<= 0: all).  Returns 0 or -1.
int oracle_attn_batched(const float* Q, const float* K, const float* V, float* O, float* lse,
                        int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk, int64_t D,
                        float scale, int causal, const uint8_t* mask, int64_t T, int nthreads,
                        const int64_t* slices, int64_t nslices, int64_t tile_offset,
                        int64_t tile_stride) {
  if (B < 0 || Hq < 0 || Hkv <= 0 || Hq % Hkv || Nq < 0 || Nk < 0 || D <= 0 || T <= 0)
    return -1;
  if (B == 0 || Hq == 0 || Nq == 0) return 0;  // no query row: nothing to compute
  if (!Q || !O || (Nk > 0 && (!K || !V))) return -1;
  if (tile_stride <= 0) tile_stride = 1;
  const int64_t group = Hq / Hkv;
  const int64_t ntiles = (Nq + T - 1) / T;
  std::vector<int64_t> sl;
  if (slices && nslices > 0) {
    sl.assign(slices, slices + nslices);
  } else {
    for (int64_t s = 0; s < B * Hq; ++s) sl.push_back(s);
  }
  std::vector<std::pair<int64_t, int64_t>> work;
  for (int64_t s : sl)
    for (int64_t t = tile_offset; t < ntiles; t += tile_stride) work.emplace_back(s, t);
#ifdef _OPENMP
  const int nt = nthreads > 0 ? nthreads : omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
#endif
  for (int64_t w = 0; w < static_cast<int64_t>(work.size()); ++w) {
    const int64_t s = work[w].first, t = work[w].second;
    const int64_t b = s / Hq, h = s % Hq, hk = h / group;
    const float* Qs = Q + (b * Hq + h) * Nq * D;
    const float* Ks = K + (b * Hkv + hk) * Nk * D;
    const float* Vs = V + (b * Hkv + hk) * Nk * D;
    float* Os = O + (b * Hq + h) * Nq * D;
    float* Ls = lse ? lse + (b * Hq + h) * Nq : nullptr;
    const uint8_t* Ms = mask ? mask + (b * Hq + h) * Nq * Nk : nullptr;
    SliceArgs a{Qs, Ks, Vs, Os, Ls, Ms, D, D, D, D, Nk, Nq, Nk, D, scale, causal, T};
    q_tile(a, t * T);
  }
  return 0;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
