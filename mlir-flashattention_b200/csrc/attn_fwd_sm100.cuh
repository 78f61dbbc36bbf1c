// attn_fwd_sm100.cuh — fused attention forward for B200 (sm_100a).
//
// Computes, for every (batch, q-head) slice, the `attention.fused` op of the
// reference (include/Attention/AttentionOps.td:20-54):
//     O = softmax(Q·Kᵀ·scale, masked -> -inf) · V
// with the online-softmax recurrence its TilingPass emits
// (lib/Attention/TilingPass.cpp:279-374: running max m, running sum l, O
// rescaled by alpha = exp(m_old - m_new)), restated for the tensor cores:
//
//   Persistent: one CTA per SM walks a work list of Q-tile pairs (two Q
//   tiles of 128 rows of one slice); see item_index / decode_item.
//   warp 8      TMA producer: the pair's Q tiles, then K_j / V_j tiles (128
//               keys) through an NS-stage shared-memory ring (mbarrier
//               full/empty) that runs on across pairs.
//   warp 9      MMA issuer (converged warp, one elected lane issues):
//               S_t = Q_t·K_jᵀ into TMEM (SS form), O_t += P_t·V_j with P_t
//               read from TMEM (TS form); order per KV step
//               P·V_0(j), S_0(j'), P·V_1(j), S_1(j') where j' is the next
//               KV tile of the pair's list (PairSched); each S GEMM is
//               issued once the P·V GEMM reading P from its TMEM columns has
//               completed (gate_S), and each P·V GEMM in two halves of 64
//               keys as the softmax publishes the halves of P (kHalfP).
//               d = 64 ("early S", P in columns of its own) and e4m3 (early
//               S, P in shared memory, P·V in the SS form): S_0(j'), S_1(j')
//               as soon as each softmax has read its S, then P·V_0(j),
//               P·V_1(j).
//   warps 0-3   softmax for Q tile 0, warps 4-7 for Q tile 1: one thread per
//               query row reads its S row from TMEM, applies the mask, updates
//               (m, l) in registers, writes P (bf16 / f16) back into the S
//               columns (d = 64: P's own columns; e4m3: a shared-memory
//               tile) and rescales its O row in
//               TMEM when m moved; at the end of a pair it writes O / l
//               (through a shared-memory box per warp and a TMA tensor
//               store) and the LSE.
//   warps 10-11 idle (they complete warpgroup 2 for the register split).
//   The two Q tiles ping-pong: while one softmax group works, the tensor
//   cores run the other tile's GEMMs.  Registers: launched at 168 per thread
//   (three warps share each SM sub-partition), the softmax warpgroups raise
//   theirs to 224 and warpgroup 2 lowers its to 56 (setmaxnreg).
//
// TMEM (512 columns): S0/P0 [0,128) S1/P1 [128,256) O0 [256,256+D)
// O1 [256+D, 256+2D); at d = 64 P0 [384,448) P1 [448,512); e4m3 P_t lives
// in two 128 x 128-byte shared-memory tiles (step n in tile n & 1).
// Exponentials are base 2 with the scale folded in:
// p = 2^(s·scale·log2e − m).  The running max only moves when it grows by
// more than 2^8 (values of p stay <= 256, exact in bf16/e4m3 range), which
// skips most O rescales; the final O/l and LSE are unaffected by the choice.
//
// Mask modes: none; causal (mask[i][j] = j > i): KV tiles wholly above the
// diagonal are never loaded or multiplied (the FULL / MASKED / BOUNDARY tile
// split of the reference design, Design.md:412-419) and only diagonal and
// ragged-edge tiles apply a per-element mask; dense: the op's i1 mask operand
// (TilingPass.cpp:254-277), whose 128 x 128 blocks classify_mask_tiles
// classifies first: empty blocks are skipped like the causal ones, full
// blocks need no mask bytes, partial blocks are read per row and KV tile.
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
  int num_bh;                // B * Hq
  float scale_log2;          // scale * log2(e) (* q/k descales for e4m3)
  float o_scale;             // v descale for e4m3, else 1
  int out_kind;              // 0: O is bf16, 1: fp32, 2: f16
  // Dense i1 mask (one byte per element, 1 = masked), mode 2 only.
  const uint8_t* mask;
  int64_t m_sb, m_sh, m_sn;  // byte strides: batch, head, row (column stride 1)
  int mask_vec;              // 1: rows 16-byte aligned (vector loads)
  // e4m3 per-block dequantisation factors (nullptr = not used): one per
  // 128-row block of Q ([num_bh][nqb]) and of K ([B*Hkv][nkb]), one per
  // kv head for V ([B*Hkv]).
  const float* qd_blk;
  const float* kd_blk;
  const float* vd_head;
  int nqb, nkb;
  // Dense mode: class of every (mask slice, Q tile, KV tile) block of the
  // mask (kTileFull / kTilePartial / kTileEmpty, see classify_mask_tiles);
  // byte strides per batch and head (0 for a broadcast mask), rows of nkt.
  const uint8_t* tile_cls;
  int64_t cls_sb, cls_sh;
  int nkt;
  // Dense mode: work items (slice-major index) ordered by decreasing number
  // of KV tiles visited (order_dense_items), for the persistent schedule.
  // Causal mode without a split: null, or a permutation of the work list
  // that balances the snake's last rounds (planned by the host).
  const int* order;
  // Causal mode, KV split (split_pairs > 0): the split_pairs heaviest pair
  // indices of every slice run as two work items each, over the first and
  // the second half of the pair's KV tiles.  Each half writes its rows'
  // normalised output and log2-domain LSE to part_o / part_lse; the warp
  // that finishes second (counted in part_cnt, zeroed before the launch)
  // merges both halves into O and the LSE.
  int split_pairs;
  float4* part_o;   // [split][half][t][D/4][128 rows]
  float* part_lse;  // [split][half][t][128 rows]
  int* part_cnt;    // [split][t][4 warps]
};

// Classes of a 128 x 128 block of a dense mask (rows < Nq, keys < Nk).
constexpr uint8_t kTileFull = 0;     // nothing masked: no per-element select
constexpr uint8_t kTilePartial = 1;  // some masked, or keys past Nk
constexpr uint8_t kTileEmpty = 2;    // everything masked: never loaded or multiplied

// Mask modes of the kernel (compile-time specialisations).
constexpr int kMaskNone = 0;    // no mask operand
constexpr int kMaskCausal = 1;  // mask[i][j] = j > i, computed
constexpr int kMaskDense = 2;   // explicit i1 mask read from memory

// Input element types of the tensor-core kernel.
constexpr int kEltBF16 = 0;
constexpr int kEltE4M3 = 1;
constexpr int kEltF16 = 2;

template <int D, int ELT>
struct FwdCfg {
  static constexpr bool FP8 = ELT == kEltE4M3;
  static constexpr int kEB = FP8 ? 1 : 2;               // bytes per input element
  static constexpr int kBoxCols = 128 / kEB;            // elements per 128-byte row
  static constexpr int kNBox = (D * kEB) / 128;         // 128-byte column boxes per tile
  static constexpr int kBoxBytes = 128 * 128;           // 128 rows x 128 bytes
  static constexpr int kTileBytes = kNBox * kBoxBytes;  // one 128-row tile
  // K / V ring depth (tiles of 128 keys): 4 at bf16 / f16 d = 128, 8 at
  // d = 64, 6 at e4m3 (whose two P buffers per Q tile take the room of two).
  static constexpr int kStages = FP8 ? 6 : (D == 64 ? 8 : 4);
  static constexpr int kKStepsS = (D * kEB) / 32;       // 32 bytes of K per MMA
  static constexpr int kKeysPerStep = 32 / kEB;         // keys per P·V MMA
  static constexpr int kKStepsPV = 128 / kKeysPerStep;
  // Operand format field: kind::f16 has F16 = 0, BF16 = 1; kind::f8f6f4 E4M3 = 0.
  static constexpr uint32_t kFmt = ELT == kEltBF16 ? 1u : 0u;
  static constexpr int kKind = FP8 ? 1 : 0;
  // TMEM: S_t at columns 128 t, O_t at 256 + D t.  At d = 128 the columns
  // are all taken: bf16 / f16 P_t overwrites S_t, so the next S_t GEMM
  // follows the P·V GEMM.  At d = 64, P_t has its own columns (384 + 64 t);
  // e4m3 P_t (128 x 128 bytes) lives in shared memory and its P·V GEMM takes
  // the SS form.  In both the next S_t GEMM starts as soon as the softmax
  // has read S_t ("early S").
  static constexpr bool kPSmem = FP8;
  static constexpr bool kEarlyS = D == 64 || kPSmem;
  // e4m3 P: two 128 rows x 128 keys tiles per Q tile, P of step n in
  // buffer n & 1.  The P·V GEMM that last read a buffer (step n - 2) was
  // issued before the S GEMM of step n, and the commit that completes S of
  // step n tracks every earlier MMA of the issuing thread: once the softmax
  // has seen S of step n, the buffer is free.
  static constexpr int kPTile = 128 * 128;
  static constexpr int kPBytes = kPSmem ? 4 * kPTile : 0;
  // q_full, q_empty, the K / V ring, s_full[2], p_ready[4] and pv_done[4]
  // (e4m3: one per tile and P buffer; otherwise [t]), o_free[2], s_free[2],
  // drain.
  static constexpr int kNumBars = 2 + 2 * kStages + 2 + 4 + 4 + 2 + 2 + 1;
  // Epilogue staging: one 32-row x 128-byte box (128-byte swizzle) per
  // softmax warp, written from registers and stored to O by TMA.
  static constexpr int kStageBox = 32 * 128;
  static constexpr size_t kSmemBytes = 1024 /*align slack*/ + 2 * kTileBytes +
                                       kStages * kTileBytes + 8 * kStageBox + kPBytes +
                                       kNumBars * 8 + 16;
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(kNBox >= 1, "tile must span at least one 128-byte box");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

constexpr int kThreads = 384;
// Register split (setmaxnreg): the two softmax warpgroups raise their limit
// to kRegsSoftmax, warpgroup 2 (producer, MMA issuer, two idle warps) lowers
// its own to kRegsOther.  The shares must fit in the registers the CTA is
// launched with (kThreads x the kernel's register count), or the raise would
// wait forever; the host checks the count before the first launch.
constexpr int kRegsSoftmax = 224;
constexpr int kRegsOther = 56;
constexpr int kRegPool = 256 * kRegsSoftmax + 128 * kRegsOther;

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// Warp-uniform bounded wait: every lane waits, the warp agrees on the result.
template <bool kProbeFirst = false>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* status) {
  bool ok = mbar_wait_bounded<kProbeFirst>(bar, parity, abort, status, kWaitLimitNs);
  return __all_sync(0xffffffffu, ok);
}

// Drain wait: ignores the abort flag (waits for this CTA's own copies / MMAs
// in flight), still bounded in time.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* status) {
  int never = 0;
  mbar_wait_bounded(bar, parity, &never, status, kWaitLimitNs);
}

// Work list.  One work item = two 128-row Q tiles (a "pair") of one
// (batch, q-head) slice.  Causal items are ordered heaviest first (pair index
// descending, then slice) — longest-processing-time order; non-causal items
// slice-major so CTAs running at the same time share one slice's K/V in L2.
// The persistent CTAs take items in a snake: round r gives CTA c item
// r·G + c (r even) or r·G + G-1-c (r odd), which balances the decreasing
// causal weights across CTAs.
//
// Causal KV split (FwdParams::split_pairs = S > 0, chosen by the host when
// there are too few pairs per SM for the snake to balance): the list starts
// with the two halves of each of the S heaviest pair indices (pair
// num_pairs-1-j, j < S: half 0 of every slice, then half 1 of every slice),
// followed by the unsplit pairs, heaviest first.
struct Item {
  int bh, pair;
  int half;  // -1: the whole pair; 0 / 1: first / second half of its KV tiles
};

template <bool CAUSAL>
__device__ __forceinline__ int item_index(int round, int cta, int G, int W) {
  const int w = round * G + ((round & 1) ? (G - 1 - cta) : cta);
  return w < W ? w : -1;
}

template <bool CAUSAL, bool SPLIT>
__device__ __forceinline__ Item decode_item(int w, int num_bh, int num_pairs, int split) {
  Item it;
  it.half = -1;
  if (CAUSAL) {
    const int ns = SPLIT ? 2 * split * num_bh : 0;  // split halves come first
    if (SPLIT && w < ns) {
      const int j = w / (2 * num_bh), rem = w - j * 2 * num_bh;
      it.pair = num_pairs - 1 - j;
      it.half = rem / num_bh;
      it.bh = rem - it.half * num_bh;
    } else {
      w -= ns;
      it.pair = num_pairs - 1 - split - w / num_bh;
      it.bh = w % num_bh;
    }
  } else {
    it.bh = w / num_pairs;
    it.pair = w % num_pairs;
  }
  return it;
}

// Work items of one launch.
__host__ __device__ __forceinline__ int work_items(int num_bh, int num_pairs, int split) {
  return num_bh * (num_pairs + split);
}

// KV tiles (of 128 keys) each of the two Q tiles of `pair` needs.
template <bool CAUSAL>
__device__ __forceinline__ void kv_counts(int pair, int Nq, int Nk, int (&n_t)[2]) {
  const int nkv_all = cdiv(Nk, 128);
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = pair * 256 + 128 * t;
    if (qs >= Nq) {
      n_t[t] = 0;
    } else if (CAUSAL) {
      const int last_row = min(qs + 127, Nq - 1);
      n_t[t] = min(nkv_all, last_row / 128 + 1);
    } else {
      n_t[t] = nkv_all;
    }
  }
}

// The KV tiles one pair visits: the union, in increasing order, of the KV
// tiles either Q tile needs, and which tile needs which.  No-mask and causal
// pairs need a prefix per tile (kv_counts).  Dense-mask pairs skip KV tiles
// whose mask block is empty for a Q tile (the FULL / MASKED / BOUNDARY split
// of the reference design, Design.md:412-419, applied to an arbitrary mask);
// a Q tile whose first KV tile is empty needs none: its rows are NaN, as in
// the reference (see the softmax).
template <int MODE, bool SPLIT>
struct PairSched {
  int n_t[2];             // no-mask, causal: tile t needs KV tiles [lo, n_t[t])
  int lo;                 // first KV tile of this item (second half of a split pair: > 0)
  bool merge[2];          // split pair whose tile t has KV tiles in both halves
  const uint8_t* cls[2];  // dense: the Q tiles' class rows (nullptr: no KV tile)
  int nkt;                // dense: KV tiles per row

  __device__ __forceinline__ bool act(int t, int kt) const {
    if constexpr (MODE == kMaskDense)
      return cls[t] != nullptr && __ldg(cls[t] + kt) != kTileEmpty;
    else if constexpr (SPLIT)
      return kt >= lo && kt < n_t[t];
    else
      return kt < n_t[t];
  }
  __device__ __forceinline__ bool any(int t) const {
    if constexpr (MODE == kMaskDense) return cls[t] != nullptr;
    else if constexpr (SPLIT) return n_t[t] > lo;
    else return n_t[t] > 0;
  }
  // First KV tile Q tile t needs (any(t) must hold).
  __device__ __forceinline__ int first_t(int t) const {
    if constexpr (SPLIT) return lo;
    else return 0;
  }
  __device__ __forceinline__ int end() const {
    if constexpr (MODE == kMaskDense) return nkt;
    else return max(n_t[0], n_t[1]);
  }
  // Next KV tile of the union after kt (end() if none); next(-1) is the first.
  __device__ __forceinline__ int next(int kt) const {
    if constexpr (MODE == kMaskDense) {
      for (++kt; kt < nkt; ++kt)
        if (act(0, kt) || act(1, kt)) break;
      return kt;
    } else if constexpr (SPLIT) {
      return max(kt + 1, lo);
    } else {
      return kt + 1;
    }
  }
  // Next KV tile Q tile t needs after kt (end() if none).
  __device__ __forceinline__ int next_t(int t, int kt) const {
    if constexpr (MODE == kMaskDense) {
      for (++kt; kt < nkt; ++kt)
        if (act(t, kt)) break;
      return kt;
    } else {
      return kt + 1 < n_t[t] ? kt + 1 : end();
    }
  }
  __device__ __forceinline__ bool full(int t, int kt) const {
    if constexpr (MODE == kMaskDense) return __ldg(cls[t] + kt) == kTileFull;
    else return false;
  }
};

template <int MODE, bool SPLIT>
__device__ __forceinline__ PairSched<MODE, SPLIT> make_sched(const Item& itm, const FwdParams& p) {
  PairSched<MODE, SPLIT> sc;
  sc.lo = 0;
  sc.merge[0] = sc.merge[1] = false;
  if constexpr (MODE == kMaskDense) {
    const int b = itm.bh / p.Hq, h = itm.bh - (itm.bh / p.Hq) * p.Hq;
    sc.nkt = p.nkt;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int qt = itm.pair * 2 + t;
      const uint8_t* row = p.tile_cls + b * p.cls_sb + h * p.cls_sh +
                           static_cast<int64_t>(qt) * p.nkt;
      sc.cls[t] = (qt * 128 < p.Nq && __ldg(row) != kTileEmpty) ? row : nullptr;
      sc.n_t[t] = 0;
    }
  } else {
    kv_counts<MODE == kMaskCausal>(itm.pair, p.Nq, p.Nk, sc.n_t);
    sc.cls[0] = sc.cls[1] = nullptr;
    sc.nkt = 0;
    if (SPLIT && itm.half >= 0) {
      // Halves [0, mid) and [mid, end) of the pair's KV tiles.
      const int mid = (max(sc.n_t[0], sc.n_t[1]) + 1) / 2;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        sc.merge[t] = sc.n_t[t] > mid;
        if (itm.half == 0) sc.n_t[t] = min(sc.n_t[t], mid);
      }
      sc.lo = itm.half == 0 ? 0 : mid;
    }
  }
  return sc;
}

// 128 mask bytes of one row for keys [kbase, kbase+128): bit c of the
// returned words is set when key kbase+c is masked or does not exist.
__device__ __forceinline__ void load_mask_row(const uint8_t* mrow, int kbase, int Nk, bool vec,
                                              uint32_t (&bits)[4]) {
  bits[0] = bits[1] = bits[2] = bits[3] = 0u;
  if (vec && kbase + 128 <= Nk) {
    const uint4* src = reinterpret_cast<const uint4*>(mrow + kbase);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 v = __ldg(src + q);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb)
          if ((w[e] >> (8 * bb)) & 0xFFu) bits[q / 2] |= 1u << ((q & 1) * 16 + e * 4 + bb);
    }
  } else {
#pragma unroll 4
    for (int c = 0; c < 128; ++c)
      if (kbase + c >= Nk || mrow[kbase + c] != 0) bits[c >> 5] |= 1u << (c & 31);
  }
}

// SPLIT: the causal launch with a KV split of its heaviest pairs
// (FwdParams::split_pairs > 0); a separate specialisation, so launches
// without a split run no split logic.
template <int D, int MODE, int ELT, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV,
                          const __grid_constant__ CUtensorMap tmO, const FwdParams p) {
  constexpr bool CAUSAL = MODE == kMaskCausal;
  static_assert(!SPLIT || CAUSAL, "the KV split is a causal-mode schedule");
  constexpr bool DENSE = MODE == kMaskDense;
  using C = FwdCfg<D, ELT>;
  constexpr bool FP8 = C::FP8;
  // Early-S kernels (d = 64, e4m3) find most of their waits already
  // complete, and a non-blocking probe before the suspending wait is cheaper
  // there (e4m3 causal GQA +1 %, bf16 d = 64 causal +2-3 %); the gated
  // kernels' chain waits are mostly still pending and lose ~1.5 % with it.
  constexpr bool kProbe = C::kEarlyS;
  // Gated bf16 / f16 kernels: P is published in two halves of 64 keys
  // (p_ready[t], then p_ready[2 + t]) and the P·V GEMM is issued in two
  // halves, the first while the softmax computes the second half of P
  // (bf16 d = 128: non-causal +2.6 %, causal +0.7 % at full clock).
  constexpr bool kHalfP = !C::kEarlyS && !FP8;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + 2 * C::kTileBytes;
  uint8_t* sStage = sKV + C::kStages * C::kTileBytes;  // 1024-byte aligned
  uint8_t* sP = sStage + 8 * C::kStageBox;              // e4m3 P tiles (1024-byte aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::kPBytes);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + C::kStages;
  uint64_t* s_full = kv_empty + C::kStages;
  uint64_t* p_ready = s_full + 2;
  uint64_t* pv_done = p_ready + 4;
  uint64_t* o_free = pv_done + 4;
  uint64_t* s_free = o_free + 2;  // early S: the softmax has read S_t
  // P of step n of tile t ready / P·V GEMM n of tile t complete, and the
  // parity of that phase.  e4m3 has one barrier of each per P buffer (n & 1):
  // its softmax waits for a P·V GEMM only before an O rescale, so it may run
  // a step ahead of the MMA warp, and with one barrier per buffer no waiter
  // is ever two phases away from the barrier it waits on (P of step n + 2
  // needs S of step n + 2, which the MMA warp issues only after the P·V GEMM
  // of step n).
  auto p_bar = [&](int t, int n) { return FP8 ? &p_ready[2 * t + (n & 1)] : &p_ready[t]; };
  auto pv_bar = [&](int t, int n) { return FP8 ? &pv_done[2 * t + (n & 1)] : &pv_done[t]; };
  auto ph_par = [](int n) { return static_cast<uint32_t>((FP8 ? (n >> 1) : n) & 1); };
  uint64_t* drain = s_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x);
  const int cta = static_cast<int>(blockIdx.x);
  const int W = work_items(p.num_bh, p.num_pairs, SPLIT ? p.split_pairs : 0);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);  // one arrival per softmax warp
      mbar_init(&p_ready[2 + t], 4);
      mbar_init(&pv_done[t], 1);
      mbar_init(&pv_done[2 + t], 1);
      mbar_init(&o_free[t], 128);
      mbar_init(&s_free[t], 4);  // one arrival per softmax warp
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

  if (warp >= 8) {
    setmaxnreg_dec<kRegsOther>();
    if (warp == 8) {
      // ------------------------------------------------------------ producer
      if (lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        int ring = 0;  // K/V tiles issued so far (ring position)
        int qi = 0;    // Q pairs issued so far
        bool ok = true;
        for (int r = 0; ok; ++r) {
          const int w = item_index<CAUSAL>(r, cta, G, W);
          if (w < 0) break;
          const Item itm = decode_item<CAUSAL, SPLIT>((DENSE || p.order) ? __ldg(p.order + w) : w, p.num_bh, p.num_pairs, p.split_pairs);
          const int b = itm.bh / p.Hq, h = itm.bh - (itm.bh / p.Hq) * p.Hq, hk = h / p.group;
          const PairSched<MODE, SPLIT> sc = make_sched<MODE, SPLIT>(itm, p);
          const int kt_end = sc.end();
          int kt = sc.next(-1);
          if (kt >= kt_end) continue;  // no KV tile at all (dense: every row NaN)
          // Q buffer: free once the previous pair's last S GEMMs completed.
          if (!mbar_wait_bounded<kProbe>(q_empty, (static_cast<uint32_t>(qi) & 1u) ^ 1u,
                                         abort_flag, p.status, kWaitLimitNs)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(q_full, 2 * C::kTileBytes);
  #pragma unroll
          for (int t = 0; t < 2; ++t)
  #pragma unroll
            for (int c = 0; c < C::kNBox; ++c)
              tma_load_4d(sQ + t * C::kTileBytes + c * C::kBoxBytes, &tmQ, q_full,
                          c * C::kBoxCols, itm.pair * 256 + 128 * t, h, b);
          ++qi;
          auto load = [&](bool isv, int tile) {
            const int s = ring % C::kStages;
            const uint32_t u = static_cast<uint32_t>(ring / C::kStages);
            if (!mbar_wait_bounded<kProbe>(&kv_empty[s], (u & 1u) ^ 1u, abort_flag, p.status,
                                           kWaitLimitNs))
              return false;
            mbar_arrive_expect_tx(&kv_full[s], C::kTileBytes);
  #pragma unroll
            for (int c = 0; c < C::kNBox; ++c)
              tma_load_4d(sKV + s * C::kTileBytes + c * C::kBoxBytes, isv ? &tmV : &tmK,
                          &kv_full[s], c * C::kBoxCols, tile * 128, hk, b);
            ++ring;
            return true;
          };
          if constexpr (C::kEarlyS) {
            // The MMA warp's order: K(kt_0), then K(kt_i+1) ahead of V(kt_i),
            // then V(kt_last).
            ok = load(false, kt);
            while (ok) {
              const int kn = sc.next(kt);
              if (kn < kt_end) ok = load(false, kn);
              if (ok) ok = load(true, kt);
              if (kn >= kt_end) break;
              kt = kn;
            }
          } else {
            for (; kt < kt_end && ok; kt = sc.next(kt)) ok = load(false, kt) && load(true, kt);
          }
        }
        // Wait for every copy this thread started before the CTA may exit.
        if (qi > 0) drain_wait(q_full, static_cast<uint32_t>((qi - 1) & 1), p.status);
        for (int s = 0; s < C::kStages; ++s) {
          if (ring > s) {
            const int armed = (ring - 1 - s) / C::kStages + 1;
            drain_wait(&kv_full[s], static_cast<uint32_t>((armed - 1) & 1), p.status);
          }
        }
      }
      __syncwarp();
    } else if (warp == 9) {
      // ------------------------------------------------------------ MMA issuer
      // The whole warp runs this schedule converged (waits by every lane, the
      // MMA and commit instructions issued by one elected lane), so the
      // descriptors below stay warp-uniform.
      constexpr uint32_t idS = make_idesc(128, 128, C::kFmt, false);
      constexpr uint32_t idO = make_idesc(128, D, C::kFmt, true);
      // Descriptors of the first K step; later steps add (byte offset >> 4) to
      // the 14-bit start-address field, which cannot carry (smem < 256 KB).
      const uint64_t dQ0 = make_sdesc(smem_u32(sQ), 16, 1024);
      const uint64_t dK0 = make_sdesc(smem_u32(sKV), 16, 1024);
      const uint64_t dV0 = make_sdesc(smem_u32(sKV), C::kBoxBytes, 1024);
      const uint32_t lead = elect_one();  // the lane that issues MMAs and commits
      auto issue_S = [&](int t, int stage) {
        const uint64_t a0 = dQ0 + static_cast<uint64_t>((t * C::kTileBytes) >> 4);
        const uint64_t b0 = dK0 + static_cast<uint64_t>((stage * C::kTileBytes) >> 4);
  #pragma unroll
        for (int kk = 0; kk < C::kKStepsS; ++kk) {
          constexpr int kBox = C::kBoxBytes;
          const uint32_t off = ((kk * 32) / 128) * kBox + ((kk * 32) % 128);
          mma_ss_lead<C::kKind>(lead, tmem + t * 128, a0 + (off >> 4), b0 + (off >> 4), idS,
                                kk > 0 ? 1u : 0u);
        }
      };
      // pbuf: the P buffer of this step (e4m3 P in shared memory).
      auto issue_PV_half = [&](int t, int stage, bool acc, int half) {
        const uint64_t b0 = dV0 + static_cast<uint64_t>((stage * C::kTileBytes) >> 4);
        const uint32_t tP = tmem + t * 128;  // P_t's columns (its S columns)
  #pragma unroll
        for (int k = 0; k < C::kKStepsPV / 2; ++k) {
          const int kk = half * (C::kKStepsPV / 2) + k;
          mma_ts_lead<C::kKind>(lead, tmem + 256 + t * D, tP + kk * 8,
                                b0 + static_cast<uint64_t>((kk * C::kKeysPerStep * 128) >> 4),
                                idO, (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto issue_PV = [&](int t, int stage, bool acc, int pbuf) {
        const uint64_t b0 = dV0 + static_cast<uint64_t>((stage * C::kTileBytes) >> 4);
        if constexpr (C::kPSmem) {
          // P_t from shared memory (K-major, 128-byte swizzle, one 128-byte
          // row per query row): each MMA takes the next 32 keys' bytes.
          const uint64_t a0 = make_sdesc(smem_u32(sP + (2 * t + pbuf) * C::kPTile), 16, 1024);
  #pragma unroll
          for (int kk = 0; kk < C::kKStepsPV; ++kk)
            mma_ss_lead<C::kKind>(lead, tmem + 256 + t * D,
                                  a0 + static_cast<uint64_t>((kk * 32) >> 4),
                                  b0 + static_cast<uint64_t>((kk * C::kKeysPerStep * 128) >> 4),
                                  idO, (acc || kk > 0) ? 1u : 0u);
        } else {
          const uint32_t tP = tmem + (C::kEarlyS ? 384 + t * 64 : t * 128);  // P_t's columns
  #pragma unroll
          for (int kk = 0; kk < C::kKStepsPV; ++kk)
            mma_ts_lead<C::kKind>(lead, tmem + 256 + t * D, tP + kk * 8,
                                  b0 + static_cast<uint64_t>((kk * C::kKeysPerStep * 128) >> 4),
                                  idO, (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto wait = [&](uint64_t* bar, int phase) {
        return warp_wait<kProbe>(bar, static_cast<uint32_t>(phase & 1), abort_flag, p.status);
      };
      int ring = 0;             // ring position of this pair's K_0
      int qi = 0;               // pairs started
      int pv_cnt[2] = {0, 0};   // P·V GEMMs committed per tile (pv_done phases)
      int s_cnt[2] = {0, 0};    // early S: S GEMMs issued per tile (s_free phases)
      int p_cnt[2] = {0, 0};    // p_ready phases consumed per tile
      int items_t[2] = {0, 0};  // pairs in which tile t was active
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int w = item_index<CAUSAL>(r, cta, G, W);
        if (w < 0) break;
        const Item itm = decode_item<CAUSAL, SPLIT>((DENSE || p.order) ? __ldg(p.order + w) : w, p.num_bh, p.num_pairs, p.split_pairs);
        const PairSched<MODE, SPLIT> sc = make_sched<MODE, SPLIT>(itm, p);
        const int kt_end = sc.end();
        const int kt0 = sc.next(-1);
        if (kt0 >= kt_end) continue;  // no KV tile (the producer skips the pair too)
        int i = 0;  // position of kt in this pair's KV tile list
        if constexpr (C::kEarlyS) {
          // Ring positions (the producer's order): K of the first KV tile at
          // `ring`, then for step i K of the next tile at ring + 2i + 1 ahead
          // of V of this tile at ring + 2i + 2, the last V at ring + 2i + 1.
          auto slot = [](int pos) { return pos % C::kStages; };
          auto phs = [](int pos) { return pos / C::kStages; };
          // S_t into its TMEM columns once the softmax has read the previous S_t.
          auto issue_S_t = [&](int t, int kpos) {
            if (s_cnt[t] > 0 && !wait(&s_free[t], s_cnt[t] - 1)) return false;
            tc_fence_after();
            issue_S(t, slot(kpos));
            mma_commit_lead(lead, &s_full[t]);
            ++s_cnt[t];
            return true;
          };
          if (!wait(q_full, qi) || !wait(&kv_full[slot(ring)], phs(ring))) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int t = 0; t < 2 && ok; ++t)
            if (sc.act(t, kt0)) ok = issue_S_t(t, ring);
          if (!ok) break;
          mma_commit_lead(lead, &kv_empty[slot(ring)]);  // K free once its S GEMMs finish
          if (sc.next(kt0) >= kt_end) mma_commit_lead(lead, q_empty);  // all S GEMMs issued
          // Per KV tile: the next tile's S GEMMs first (each needs only its
          // softmax to have read the previous S), then O_t += P_t·V for each
          // Q tile whose P is ready.
          bool first_pv[2] = {true, true};
          int kn_ahead = DENSE ? sc.next(kt0) : 0;
          for (int kt = kt0; kt < kt_end && ok; ++i) {
            const int kn = DENSE ? kn_ahead : sc.next(kt);
            int kn2 = 0;
            bool act_kt[2] = {false, false}, act_kn[2] = {false, false};
            if constexpr (DENSE) {
              kn2 = kn < kt_end ? sc.next(kn) : kt_end;
#pragma unroll
              for (int t = 0; t < 2; ++t) {
                act_kt[t] = sc.act(t, kt);
                act_kn[t] = kn < kt_end && sc.act(t, kn);
              }
            }
            const bool more = kn < kt_end;
            if (more) {
              const int kpos = ring + 2 * i + 1;
              if (!wait(&kv_full[slot(kpos)], phs(kpos))) {
                ok = false;
                break;
              }
              for (int t = 0; t < 2 && ok; ++t)
                if (DENSE ? act_kn[t] : sc.act(t, kn)) ok = issue_S_t(t, kpos);
              if (!ok) break;
              mma_commit_lead(lead, &kv_empty[slot(kpos)]);
              if ((DENSE ? kn2 : sc.next(kn)) >= kt_end) mma_commit_lead(lead, q_empty);
            }
            const int vpos = ring + 2 * i + (more ? 2 : 1);
            if (!wait(&kv_full[slot(vpos)], phs(vpos))) {
              ok = false;
              break;
            }
            for (int t = 0; t < 2 && ok; ++t) {
              if (!(DENSE ? act_kt[t] : sc.act(t, kt))) continue;
              if (!warp_wait<kProbe>(p_bar(t, p_cnt[t]), ph_par(p_cnt[t]), abort_flag,
                                     p.status)) {
                ok = false;
                break;
              }
              ++p_cnt[t];
              if (first_pv[t] && items_t[t] > 0 && !wait(&o_free[t], items_t[t] - 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_PV(t, slot(vpos), !first_pv[t], (p_cnt[t] - 1) & 1);
              first_pv[t] = false;
              mma_commit_lead(lead, pv_bar(t, p_cnt[t] - 1));
            }
            if (!ok) break;
            mma_commit_lead(lead, &kv_empty[slot(vpos)]);  // V free once the P·V GEMMs finish
            kt = kn;
            kn_ahead = kn2;
          }
          if (!ok) break;
        } else {
          // Ring slots of the i-th KV tile of this pair (K, then V).
          auto kst = [&](int i) { return (ring + 2 * i) % C::kStages; };
          auto kph = [&](int i) { return (ring + 2 * i) / C::kStages; };
          auto vst = [&](int i) { return (ring + 2 * i + 1) % C::kStages; };
          auto vph = [&](int i) { return (ring + 2 * i + 1) / C::kStages; };
          // S_t's columns hold P_t, which the last P·V GEMM of tile t reads.
          // The PTX ISA orders two tcgen05.mma operations of one thread only
          // when they share cta_group, accumulator and shape (its pipelined
          // instruction pairs); the S GEMM (accumulator S_t, N = 128) and the
          // P·V GEMM (accumulator O_t, N = D) are not such a pair, so the S
          // GEMM is issued only once the P·V GEMM has completed (its commit
          // on pv_done[t]).  This also makes "S_t(j+1) complete" imply
          // "P·V_t(j) complete" for the softmax, which rewrites P_t and
          // rescales O_t after it sees S_t(j+1).
          auto gate_S = [&](int t) {
            if (pv_cnt[t] > 0 && !wait(&pv_done[t], pv_cnt[t] - 1)) return false;
            tc_fence_after();
            return true;
          };
          if (!wait(q_full, qi) || !wait(&kv_full[kst(0)], kph(0))) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int t = 0; t < 2 && ok; ++t) {
            if (!sc.act(t, kt0)) continue;
            // The previous pair's last P·V GEMM of this tile may still read P_t.
            if (!gate_S(t)) {
              ok = false;
              break;
            }
            issue_S(t, kst(0));
            mma_commit_lead(lead, &s_full[t]);
          }
          if (!ok) break;
          mma_commit_lead(lead, &kv_empty[kst(0)]);  // K free once its S GEMMs finish
          if (sc.next(kt0) >= kt_end) mma_commit_lead(lead, q_empty);  // all S GEMMs issued
          // Per KV tile, for each Q tile t that needs it: O_t += P_t·V, then
          // S_t = Q_t·Kᵀ of t's next KV tile once that P·V GEMM has completed
          // (gate_S: P_t lives in the S_t columns).  Tile t's next softmax
          // then overlaps the other tile's GEMMs.
          bool first_pv[2] = {true, true};
          int kn_ahead = DENSE ? sc.next(kt0) : 0;
          for (int kt = kt0; kt < kt_end && ok; ++i) {
            const int kn = DENSE ? kn_ahead : sc.next(kt);
            // Dense masks: every class lookup of this step up front, before any
            // wait, so none sits between a P·V issue and the S issue behind it
            // (no-mask and causal lookups are arithmetic and stay inline).
            int kn2 = 0;
            bool act_kt[2] = {false, false}, act_kn[2] = {false, false};
            if constexpr (DENSE) {
              kn2 = kn < kt_end ? sc.next(kn) : kt_end;
  #pragma unroll
              for (int t = 0; t < 2; ++t) {
                act_kt[t] = sc.act(t, kt);
                act_kn[t] = kn < kt_end && sc.act(t, kn);
              }
            }
            bool k_next = false;
            auto wait_k_next = [&]() {
              if (!k_next) k_next = wait(&kv_full[kst(i + 1)], kph(i + 1));
              return k_next;
            };
            if (!wait(&kv_full[vst(i)], vph(i))) {
              ok = false;
              break;
            }
            for (int t = 0; t < 2 && ok; ++t) {
              if (!(DENSE ? act_kt[t] : sc.act(t, kt))) continue;
              if (!wait(&p_ready[t], p_cnt[t])) {
                ok = false;
                break;
              }
              // The first P·V GEMM of a pair overwrites O_t: the previous pair's
              // epilogue must have read it.
              if (first_pv[t] && items_t[t] > 0 && !wait(&o_free[t], items_t[t] - 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
              if constexpr (kHalfP) {
                // Keys 0-63 of P_t are stored: their half of the GEMM, then
                // keys 64-127 once the softmax has stored them.
                issue_PV_half(t, vst(i), !first_pv[t], 0);
                if (!wait(&p_ready[2 + t], p_cnt[t])) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                issue_PV_half(t, vst(i), true, 1);
              } else {
                issue_PV(t, vst(i), !first_pv[t], 0);
              }
              ++p_cnt[t];
              first_pv[t] = false;
              mma_commit_lead(lead, &pv_done[t]);
              ++pv_cnt[t];
              if (DENSE ? act_kn[t] : (kn < kt_end && sc.act(t, kn))) {
                if (!wait_k_next() || !gate_S(t)) {
                  ok = false;
                  break;
                }
                issue_S(t, kst(i + 1));
                mma_commit_lead(lead, &s_full[t]);
              }
            }
            if (!ok) break;
            if constexpr (DENSE) {
              // A Q tile that skipped kt but needs kn gets its S GEMM here.
              for (int t = 0; t < 2 && ok; ++t) {
                if (act_kt[t] || !act_kn[t]) continue;
                if (!wait_k_next() || !gate_S(t)) {
                  ok = false;
                  break;
                }
                issue_S(t, kst(i + 1));
                mma_commit_lead(lead, &s_full[t]);
              }
              if (!ok) break;
            }
            mma_commit_lead(lead, &kv_empty[vst(i)]);  // V free once the P·V GEMMs finish
            if (kn < kt_end) {
              if (!wait_k_next()) {
                ok = false;
                break;
              }
              mma_commit_lead(lead, &kv_empty[kst(i + 1)]);  // K free once its S GEMMs finish
              if ((DENSE ? kn2 : sc.next(kn)) >= kt_end) mma_commit_lead(lead, q_empty);
            }
            kt = kn;
            kn_ahead = kn2;
          }
        }
        for (int t = 0; t < 2; ++t)
          if (sc.any(t)) ++items_t[t];
        ring += 2 * i;
        ++qi;
      }
      // Drain every MMA this warp issued before TMEM is released.
      mma_commit_lead(lead, drain);
      if (lane == 0) drain_wait(drain, 0, p.status);
      __syncwarp();
    }
    // Warps 10 and 11 only complete warpgroup 2 for the register split.
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;  // Q tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tP = tmem + lane_off + (C::kEarlyS ? 384 + t * 64 : t * 128);
    const uint32_t tO = tmem + lane_off + 256 + t * D;
    const float sl2_base = p.scale_log2;  // scale·log2(e) (· per-tensor descales)
    const bool pos = sl2_base >= 0.f;      // descales are positive: the sign is scale's
    const float mask_val = pos ? -INFINITY : INFINITY;
    int steps = 0;  // S tiles consumed so far (s_full / pv_done phases)
    bool ok = true;
    // e4m3 and d = 64 (no dense mask): the next work item, decoded ahead while
    // the epilogue waits for the last P·V GEMM (c5 +2 %, bf16 d = 64 causal
    // +3 %; the gated bf16 / f16 kernels' wait is shorter and measured slower
    // with the extra work in front of it; the d = 64 dense kernels would spill).
    constexpr bool kPreDecode = FP8 || (C::kEarlyS && !DENSE);
    int pre_rr = -1, pre_w = -1;
    Item pre_itm;
    for (int rr = 0; ok; ++rr) {
      int w;
      Item itm0;
      if (pre_rr == rr) {
        w = pre_w;
        itm0 = pre_itm;
      } else {
        w = item_index<CAUSAL>(rr, cta, G, W);
        if (w >= 0)
          itm0 = decode_item<CAUSAL, SPLIT>((DENSE || p.order) ? __ldg(p.order + w) : w, p.num_bh,
                                             p.num_pairs, p.split_pairs);
      }
      if (w < 0) break;
      const Item itm = itm0;
      const PairSched<MODE, SPLIT> sc = make_sched<MODE, SPLIT>(itm, p);
      const int b = itm.bh / p.Hq, h = itm.bh - (itm.bh / p.Hq) * p.Hq;
      const int qs = itm.pair * 256 + 128 * t;
      const int row = qs + r;
      if (!sc.any(t)) {
        if constexpr (DENSE) {
          // Every row of this Q tile is masked over its first KV tile: NaN,
          // as in the reference (see nan_row below); no GEMM is involved.
          if (qs < p.Nq && row < p.Nq) {
            const int64_t obase = static_cast<int64_t>(b) * p.o_sb +
                                  static_cast<int64_t>(h) * p.o_sh +
                                  static_cast<int64_t>(row) * p.o_sn;
            const float nan = __int_as_float(0x7fc00000);
            if (p.out_kind == 1) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.o) + obase);
#pragma unroll
              for (int i = 0; i < D / 4; ++i) dst[i] = make_float4(nan, nan, nan, nan);
            } else {
              const uint32_t q = p.out_kind == 2 ? 0x7e007e00u : 0x7fc07fc0u;
              uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.o) + obase);
#pragma unroll
              for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(q, q, q, q);
            }
            if (p.lse) p.lse[static_cast<int64_t>(itm.bh) * p.Nq + row] = nan;
          }
        }
        continue;
      }
      const int kt_end = sc.end();
      float m = -INFINITY;
      float l = 0.f;
      // e4m3 per-block factors: the Q block's folds into this tile's exponent
      // scale, the K block's into each step's, the V head's into the epilogue.
      float sl2_q = sl2_base, vd = 1.f, kd_cur = 1.f;
      const float* kd_row = nullptr;
      if constexpr (FP8) {
        const int bk = b * (p.Hq / p.group) + h / p.group;
        if (p.qd_blk) sl2_q *= __ldg(p.qd_blk + static_cast<int64_t>(itm.bh) * p.nqb + itm.pair * 2 + t);
        if (p.vd_head) vd = __ldg(p.vd_head + bk);
        if (p.kd_blk) {
          kd_row = p.kd_blk + static_cast<int64_t>(bk) * p.nkb;
          kd_cur = __ldg(kd_row + sc.first_t(t));  // the factor of this tile's first KV block
        }
      }
      // Dense masks: the reference's loop (TilingPass.cpp:291-305) evaluates
      // exp(-inf - -inf) = NaN when a row is masked over its whole first KV
      // tile, and that NaN reaches O; such rows are NaN here too.
      bool nan_row = false;
      const uint8_t* mrow = nullptr;
      if constexpr (DENSE)
        mrow = p.mask + b * p.m_sb + h * p.m_sh + static_cast<int64_t>(min(row, p.Nq - 1)) * p.m_sn;
      bool first = true;
      for (int kt = sc.first_t(t); kt < kt_end; ++steps) {
        const int kn = sc.next_t(t, kt);
        // Dense: mask bits only for partial blocks (full ones mask nothing).
        const bool sel = DENSE && !sc.full(t, kt);
        uint32_t mbits[4];
        if constexpr (DENSE) {
          if (sel) load_mask_row(mrow, kt * 128, p.Nk, p.mask_vec != 0, mbits);
        }
        if (!warp_wait<kProbe>(&s_full[t], static_cast<uint32_t>(steps & 1), abort_flag,
                               p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sl2 = sl2_q;
        if constexpr (FP8) {
          if (kd_row) {
            sl2 *= kd_cur;
            if (kn < kt_end) kd_cur = __ldg(kd_row + kn);  // next step's, loaded early
          }
        }
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
        if constexpr (C::kEarlyS) {
          // S_t has been read: the next S GEMM of this tile may overwrite it.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[t]);
        }
        const int kbase = kt * 128;
        if constexpr (DENSE) {
          if (sel) {
#pragma unroll
            for (int c = 0; c < 128; ++c)
              if ((mbits[c >> 5] >> (c & 31)) & 1u) s[c] = mask_val;
          }
        }
        const bool edge = !DENSE && ((kbase + 128 > p.Nk) || (CAUSAL && kbase + 127 > qs));
        if (edge) {
          const int lim = CAUSAL ? min(row + 1, p.Nk) : p.Nk;  // keys < lim are visible
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (kbase + c >= lim) s[c] = mask_val;
        }
        float red;
        if (pos) {
          float a0 = max3(s[0], s[1], s[2]), a1 = max3(s[3], s[4], s[5]);
#pragma unroll
          for (int c = 6; c < 126; c += 4) {
            a0 = max3(a0, s[c], s[c + 1]);
            a1 = max3(a1, s[c + 2], s[c + 3]);
          }
          red = max3(a0, a1, fmaxf(s[126], s[127]));
        } else {
          float a0 = min3(s[0], s[1], s[2]), a1 = min3(s[3], s[4], s[5]);
#pragma unroll
          for (int c = 6; c < 126; c += 4) {
            a0 = min3(a0, s[c], s[c + 1]);
            a1 = min3(a1, s[c + 2], s[c + 3]);
          }
          red = min3(a0, a1, fminf(s[126], s[127]));
        }
        if constexpr (DENSE) {
          if (kt == 0) nan_row = red == mask_val;
        }
        const float m_cand = red * sl2;
        float alpha = 1.f;
        if (m_cand > m + 8.f) {  // m = -inf: any finite candidate moves it
          alpha = ex2(m - m_cand);
          m = m_cand;
        }
        const float neg_m = (m == -INFINITY) ? 0.f : -m;
        // x = s·sl2 − m and the row sums on packed fp32 pairs.
        const uint64_t sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(neg_m, neg_m);
        if constexpr (kHalfP) {
          // O_t rescaled first (the previous P·V GEMM has completed: its S GEMM
          // followed it), then P in two halves, each published as it is stored.
          const bool need_h = !first && (alpha != 1.f);
          first = false;
          if (__any_sync(0xffffffffu, need_h)) {
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
          uint64_t ha0 = f2_pack(0.f, 0.f), ha1 = ha0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t pk[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int cc = 32 * h + c;
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(s[2 * cc], s[2 * cc + 1]), sl2x2, negm2), x0, x1);
              const float e0 = ex2(x0), e1 = ex2(x1);
              const uint64_t pr = f2_pack(e0, e1);
              if (c & 1) ha1 = f2_add(ha1, pr); else ha0 = f2_add(ha0, pr);
              pk[c] = ELT == kEltF16 ? pack_f16(e0, e1) : pack_bf16(e0, e1);
            }
            tmem_st32(tP + 32 * h, pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(h == 0 ? &p_ready[t] : &p_ready[2 + t]);
          }
          float q0, q1;
          f2_unpack(f2_add(ha0, ha1), q0, q1);
          l = l * alpha + (q0 + q1);
          kt = kn;
          continue;
        }
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(s[2 * c], s[2 * c + 1]), sl2x2, negm2), x0, x1);
          s[2 * c] = ex2(x0);
          s[2 * c + 1] = ex2(x1);
        }
        uint64_t acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
        if constexpr (!FP8) {
          uint32_t pk[64];
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const uint64_t pr = f2_pack(s[2 * c], s[2 * c + 1]);
            if (c & 1) acc1 = f2_add(acc1, pr); else acc0 = f2_add(acc0, pr);
            pk[c] = ELT == kEltF16 ? pack_f16(s[2 * c], s[2 * c + 1])
                                   : pack_bf16(s[2 * c], s[2 * c + 1]);
          }
          if constexpr (C::kEarlyS) {
            // P_t's columns and O_t: the previous P·V GEMM of this tile reads
            // the one and accumulates into the other, so it must be complete
            // before P_t is rewritten or O_t rescaled.  (Without early S the
            // MMA warp issues this S GEMM only after that P·V GEMM completed,
            // so the completion of the S GEMM implies it.)
            if (steps > 0 && !warp_wait<kProbe>(&pv_done[t],
                                                static_cast<uint32_t>((steps - 1) & 1),
                                                abort_flag, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          tmem_st32(tP + 0, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
          tmem_st32(tP + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
        } else {
          uint32_t pk[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            acc0 = f2_add(acc0, f2_pack(s[4 * c], s[4 * c + 1]));
            acc1 = f2_add(acc1, f2_pack(s[4 * c + 2], s[4 * c + 3]));
            pk[c] = pack_e4m3x4(s[4 * c], s[4 * c + 1], s[4 * c + 2], s[4 * c + 3]);
          }
          // P buffer steps & 1 is free (see kPTile); the row's 128 bytes as 8
          // chunks of 16 (128-byte swizzle: chunk c of row r at position
          // c ^ (r & 7), conflict-free), then made visible to the tensor core
          // (async proxy) before the warp's arrival on p_ready.
          uint8_t* prow = sP + (2 * t + (steps & 1)) * C::kPTile + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) * 16)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          fence_proxy_async_smem();
        }
        float q0, q1;
        f2_unpack(f2_add(acc0, acc1), q0, q1);
        l = l * alpha + (q0 + q1);
        const bool need = !first && (alpha != 1.f);
        first = false;
        if (__any_sync(0xffffffffu, need)) {
          if constexpr (FP8) {
            // O_t: the previous P·V GEMM of this tile accumulates into it.
            if (!warp_wait<kProbe>(pv_bar(t, steps - 1), ph_par(steps - 1), abort_flag,
                                   p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
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
        __syncwarp();
        if (lane == 0) mbar_arrive(p_bar(t, steps));
        kt = kn;
      }
      if (!ok) break;
      // -------------------------------------------------------- epilogue
      // Work that does not read O, done while the last P·V GEMM completes:
      // 1/l and (kPreDecode) the row's LSE and the next work item.  A split pair's
      // halves merge their LSE below.
      const float inv_l = nan_row ? __int_as_float(0x7fc00000) : p.o_scale * vd / l;
      auto store_lse = [&]() {
        if (!(SPLIT && sc.merge[t]) && row < p.Nq && p.lse)
          p.lse[static_cast<int64_t>(itm.bh) * p.Nq + row] =
              nan_row ? __int_as_float(0x7fc00000) : (m + __log2f(l)) * 0.69314718055994531f;
      };
      if constexpr (kPreDecode) {
        store_lse();
        pre_rr = rr + 1;
        pre_w = item_index<CAUSAL>(pre_rr, cta, G, W);
        if (pre_w >= 0)
          pre_itm = decode_item<CAUSAL, SPLIT>((DENSE || p.order) ? __ldg(p.order + pre_w) : pre_w, p.num_bh,
                                               p.num_pairs, p.split_pairs);
      }
      // The tile's last P·V GEMM has completed.
      if (!warp_wait<kProbe>(pv_bar(t, steps - 1), ph_par(steps - 1), abort_flag,
                             p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if constexpr (SPLIT) {
        if (sc.merge[t]) {
          // Half of a split pair: this warp's 32 rows go to the partial
          // buffers (normalised O, LSE in the log2 domain; a row with no
          // visible key in this half has weight 0), and the warp that comes
          // second merges both halves, always as half 0 + half 1 so the
          // result does not depend on which finished last.
          const int sidx = (p.num_pairs - 1 - itm.pair) * p.num_bh + itm.bh;
          const int slot = (sidx * 2 + itm.half) * 2 + t;
          const float inv = l > 0.f ? p.o_scale * vd / l : 0.f;
          float4* mine = p.part_o + static_cast<int64_t>(slot) * (D / 4) * 128 + r;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
            if (c == D / 32 - 1) {
              tc_fence_before();
              mbar_arrive(&o_free[t]);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
              mine[(c * 8 + i) * 128] = make_float4(
                  __uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                  __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
          }
          p.part_lse[slot * 128 + r] = l > 0.f ? m + __log2f(l) : -INFINITY;
          __threadfence();
          __syncwarp();
          int old = 0;
          if (lane == 0) old = atomicAdd(p.part_cnt + (sidx * 2 + t) * 4 + quarter, 1);
          old = __shfl_sync(0xffffffffu, old, 0);
          if (old == 0) continue;  // the other half is still running and will merge
          __threadfence();
          const int s0 = (sidx * 2) * 2 + t, s1 = (sidx * 2 + 1) * 2 + t;
          const float la = __ldcg(p.part_lse + s0 * 128 + r);
          const float lb = __ldcg(p.part_lse + s1 * 128 + r);
          const float mx = fmaxf(la, lb);
          const float ea = ex2(la - mx), eb = ex2(lb - mx);
          const float sum = ea + eb, wa = ea / sum, wb = eb / sum;
          if (row < p.Nq) {
            const float4* h0 = p.part_o + static_cast<int64_t>(s0) * (D / 4) * 128 + r;
            const float4* h1 = p.part_o + static_cast<int64_t>(s1) * (D / 4) * 128 + r;
            auto mix = [&](int c4) {
              const float4 x = __ldcg(h0 + c4 * 128), y = __ldcg(h1 + c4 * 128);
              return make_float4(fmaf(wb, y.x, wa * x.x), fmaf(wb, y.y, wa * x.y),
                                 fmaf(wb, y.z, wa * x.z), fmaf(wb, y.w, wa * x.w));
            };
            const int64_t obase = static_cast<int64_t>(b) * p.o_sb +
                                  static_cast<int64_t>(h) * p.o_sh +
                                  static_cast<int64_t>(row) * p.o_sn;
            if (p.out_kind == 1) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.o) + obase);
#pragma unroll 4
              for (int c4 = 0; c4 < D / 4; ++c4) dst[c4] = mix(c4);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.o) + obase);
              const bool f16 = p.out_kind == 2;
              auto pk = [&](float x, float y) { return f16 ? pack_f16(x, y) : pack_bf16(x, y); };
#pragma unroll 4
              for (int c8 = 0; c8 < D / 8; ++c8) {
                const float4 u = mix(2 * c8), v = mix(2 * c8 + 1);
                dst[c8] = make_uint4(pk(u.x, u.y), pk(u.z, u.w), pk(v.x, v.y), pk(v.z, v.w));
              }
            }
            if (p.lse)
              p.lse[static_cast<int64_t>(itm.bh) * p.Nq + row] =
                  (mx + __log2f(sum)) * 0.69314718055994531f;
          }
          continue;
        }
      }
      // O leaves through this warp's staging box: each thread writes its row's
      // 128-byte slice (8 x 16 bytes, 128-byte swizzle: chunk c of row r at
      // chunk position c ^ (r & 7), conflict-free), then one lane stores the
      // 32 x 128-byte box with TMA; rows past Nq fall outside the tensor and
      // are not written.  The previous box's store must have read the buffer.
      {
        uint8_t* stg = sStage + warp * C::kStageBox;
        const int y = qs + quarter * 32;
        // Stage the 32 words of one 128-byte box and store it with TMA.
        auto store_box = [&](const uint32_t (&w)[32], int c0) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) * 16)) =
                make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_4d(&tmO, stg, c0, y, h, b);
            bulk_commit_group();
          }
        };
        if (p.out_kind != 1) {
          const bool f16 = p.out_kind == 2;
          // 64 columns of the row (two TMEM chunks) scaled and packed.
          auto pack_box = [&](const uint32_t(&lo)[32], const uint32_t(&hi)[32], uint32_t(&w)[32]) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float a0 = __uint_as_float(lo[2 * i]) * inv_l, a1 = __uint_as_float(lo[2 * i + 1]) * inv_l;
              const float b0 = __uint_as_float(hi[2 * i]) * inv_l, b1 = __uint_as_float(hi[2 * i + 1]) * inv_l;
              w[i] = f16 ? pack_f16(a0, a1) : pack_bf16(a0, a1);
              w[16 + i] = f16 ? pack_f16(b0, b1) : pack_bf16(b0, b1);
            }
          };
          if constexpr (!FP8) {
            // bf16 / f16 inputs: the whole O row in one TMEM round trip, O_t
            // released to the next pair at once, then one box per 64 columns
            // (c3 +1.8 %; the e4m3 kernel measured faster with the per-box
            // form below).
            uint32_t o[D / 32][32];
#pragma unroll
            for (int c = 0; c < D / 32; ++c) tmem_ld32(tO + c * 32, o[c]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&o_free[t]);
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 64) {
              uint32_t w[32];
              pack_box(o[c0 / 32], o[c0 / 32 + 1], w);
              store_box(w, c0);
            }
          } else {
#pragma unroll 1
            for (int c0 = 0; c0 < D; c0 += 64) {
              uint32_t lo[32], hi[32], w[32];
              tmem_ld32(tO + c0, lo);
              tmem_ld32(tO + c0 + 32, hi);
              tmem_wait_ld();
              if (c0 + 64 >= D) {
                // O_t has been read into registers: the next pair may overwrite it.
                tc_fence_before();
                mbar_arrive(&o_free[t]);
              }
              pack_box(lo, hi, w);
              store_box(w, c0);
            }
          }
        } else {
          // f32: 32 columns per box.
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t o[32], w[32];
            tmem_ld32(tO + c0, o);
            tmem_wait_ld();
            if (c0 + 32 >= D) {
              // O_t has been read into registers: the next pair may overwrite it.
              tc_fence_before();
              mbar_arrive(&o_free[t]);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(__uint_as_float(o[i]) * inv_l);
            store_box(w, c0);
          }
        }
      }
      if constexpr (!kPreDecode) store_lse();
    }
  }

  // ---------------------------------------------------------------- teardown
  if (warp < 8 && lane == 0) bulk_wait_all();  // this warp's O stores are complete
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Classes of the 128 x 128 blocks of a dense mask, for the dense mode's KV
// tile skipping.  One warp per block (8 per CTA): on the vector path lanes
// 8r..8r+7 read row r's 128 bytes as 16-byte words, four rows per load, so
// every load instruction takes four whole 128-byte lines; the warp ORs "some
// key visible" and "some key masked" over the block's rows (rows >= Nq
// ignored) and writes kTileEmpty, kTilePartial (also every block reaching past
// Nk) or kTileFull.  Reads each distinct mask slice once: HBM-bound.
constexpr int kClassifyWarps = 8;

__global__ void __launch_bounds__(kClassifyWarps * 32)
    classify_mask_tiles(const uint8_t* __restrict__ mask, int64_t m_sb, int64_t m_sh,
                        int64_t m_sn, int Hm, int nqt, int Nq, int Nk, int nkt, int vec,
                        uint8_t* __restrict__ cls, int* __restrict__ row_count,
                        int64_t nblocks) {
  const int lane = static_cast<int>(threadIdx.x) & 31;
  const int64_t blk = static_cast<int64_t>(blockIdx.x) * kClassifyWarps + (threadIdx.x >> 5);
  if (blk >= nblocks) return;  // whole warps only
  const int kt = static_cast<int>(blk % nkt);
  const int64_t sq = blk / nkt;  // slice * nqt + qt
  const int qt = static_cast<int>(sq % nqt);
  const int slice = static_cast<int>(sq / nqt);
  const int bm = slice / Hm, hm = slice - (slice / Hm) * Hm;
  const uint8_t* base = mask + bm * m_sb + hm * m_sh;
  const int row0 = qt * 128, kbase = kt * 128;
  const int rows = min(128, Nq - row0);
  bool vis = false, msk = false;
  if (vec && kbase + 128 <= Nk) {
    const int sub = lane >> 3, word = lane & 7;  // row within a group of 4, 16-byte word
    for (int r = sub; r < rows; r += 4) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(row0 + r) * m_sn +
                                                           kbase) + word);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        msk |= w[e] != 0u;
        vis |= ((w[e] - 0x01010101u) & ~w[e] & 0x80808080u) != 0u;  // some byte is 0
      }
    }
  } else {
    const int lim = min(128, Nk - kbase);
    for (int r = 0; r < rows; ++r) {
      const uint8_t* mrow = base + static_cast<int64_t>(row0 + r) * m_sn + kbase;
      for (int c = lane; c < lim; c += 32) {
        const bool m = mrow[c] != 0;
        msk |= m;
        vis |= !m;
      }
    }
  }
  const bool any_vis = __any_sync(0xffffffffu, vis);
  const bool any_msk = __any_sync(0xffffffffu, msk);
  if (lane == 0) {
    cls[blk] = !any_vis ? kTileEmpty : ((any_msk || kbase + 128 > Nk) ? kTilePartial : kTileFull);
    if (any_vis) atomicAdd(row_count + sq, 1);  // non-empty blocks per (slice, Q tile)
  }
}

// Work list order for the dense mode: pairs sorted by decreasing weight
// (the KV tiles their two Q tiles visit: the non-empty blocks counted per
// (slice, Q tile) by classify_mask_tiles, 0 for a tile whose first block is
// empty), so the persistent CTAs' snake takes the heaviest pairs first, as
// the causal mode's fixed order does.  One CTA: weights, a counting sort over
// at most kOrderBuckets weights (more: the slice-major identity order),
// scatter.
// Items of equal weight keep their slice-major order.
constexpr int kOrderBuckets = 4096;

__global__ void __launch_bounds__(1024)
    order_dense_items(const uint8_t* __restrict__ cls, const int* __restrict__ row_count,
                      int64_t cls_sb, int64_t cls_sh, int Hq, int num_bh, int num_pairs, int nqt,
                      int nkt, uint16_t* __restrict__ weight, int* __restrict__ order) {
  __shared__ int start[kOrderBuckets];
  const int items = num_bh * num_pairs;
  const int nb = 2 * nkt + 1;
  if (nb > kOrderBuckets) {
    for (int i = threadIdx.x; i < items; i += blockDim.x) order[i] = i;
    return;
  }
  for (int k = threadIdx.x; k < nb; k += blockDim.x) start[k] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int bh = i / num_pairs, pair = i - (i / num_pairs) * num_pairs;
    const int b = bh / Hq, h = bh - (bh / Hq) * Hq;
    int wgt = 0;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int qt = 2 * pair + t;
      if (qt >= nqt) continue;
      const int64_t r = (b * cls_sb + h * cls_sh) / nkt + qt;  // (slice, Q tile)
      if (cls[r * nkt] == kTileEmpty) continue;  // NaN tile: no KV tile visited
      wgt += row_count[r];
    }
    weight[i] = static_cast<uint16_t>(wgt);
    atomicAdd(&start[wgt], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // heaviest first: exclusive sum over decreasing weights
    int acc = 0;
    for (int k = nb - 1; k >= 0; --k) {
      const int c = start[k];
      start[k] = acc;
      acc += c;
    }
  }
  __syncthreads();
  // Stable scatter (equal weights keep the slice-major order, so the result
  // and the schedule are the same on every call): a chunk of blockDim items at
  // a time, warps in turn, each weight group of a warp placed by its leader.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int c0 = 0; c0 < items; c0 += blockDim.x) {
    const int i = c0 + static_cast<int>(threadIdx.x);
    const bool valid = i < items;
    const int wgt = valid ? static_cast<int>(weight[i]) : -1;
    const unsigned same = __match_any_sync(0xffffffffu, wgt);
    const int leader = __ffs(same) - 1;
    const int rank = __popc(same & ((1u << lane) - 1u));
    for (int wj = 0; wj < nwarps; ++wj) {
      if (warp == wj) {
        int base = 0;
        if (lane == leader && valid) {
          base = start[wgt];
          start[wgt] = base + __popc(same);
        }
        base = __shfl_sync(0xffffffffu, base, leader);
        if (valid) order[base + rank] = i;
      }
      __syncthreads();
    }
  }
}

}  // namespace attn_sm100
