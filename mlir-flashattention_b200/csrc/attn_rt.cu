// attn_rt.cu — host runtime behind include/attn_rt.h.
//
// This is the boundary where the reference's CPU lowering of `attention.fused`
// (lib/Attention/TilingPass.cpp:155-392) is replaced: the op's operands arrive
// here (as an AttnDesc or as MLIR memref descriptors), are checked with the
// reference verifier's rules (lib/Attention/AttentionOps.cpp:33-59), and the
// sm_100a kernels are launched.  No CPU fallback exists: without an sm_100
// device every entry point returns ATTN_ERR_NO_DEVICE.
#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/attn_rt.h"
#include "attn_fwd_f32.cuh"
#include "attn_fwd_sm100.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};

// NVTX range over one entry point's host work (validation, staging copies,
// launches), so that a timeline tool shows each call beside its kernels.
// Header-only NVTX: without an attached tool the calls do nothing.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(ATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CUDA_TRY(call)                                   \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);  \
  } while (0)

// ----------------------------------------------------------------- devices
constexpr int kMaxDevices = 64;
constexpr int kStageBufs = 2;

struct Staging {
  // One set of device buffers for a chunk of (batch, kv-head) groups.
  void* q = nullptr;
  void* k = nullptr;
  void* v = nullptr;
  void* o = nullptr;
  float* lse = nullptr;
  size_t q_bytes = 0, k_bytes = 0, v_bytes = 0, o_bytes = 0, lse_bytes = 0;
  cudaEvent_t h2d_done = nullptr, comp_done = nullptr, d2h_done = nullptr;
};

struct DevState {
  std::mutex mu;
  bool ready = false;
  int sm_count = 0;
  int32_t* status = nullptr;
  cudaStream_t s_compute = nullptr, s_h2d = nullptr, s_d2h = nullptr;
  Staging stage[kStageBufs];
  std::mutex whole_mu;    // guards `whole` (held across one staged call)
  void* whole = nullptr;  // whole-operand staging of host f32 / dense-mask calls (grow-only)
  size_t whole_bytes = 0;
  // Stream-ordered per-call scratch (dense-mask block classes, KV-split
  // partials) comes from this pool, which keeps its memory between calls
  // (release threshold unlimited): repeated calls do not map and unmap
  // device memory, and each call's scratch stays private to its stream.
  cudaMemPool_t pool = nullptr;
};

DevState g_dev[kMaxDevices];

int init_device(int device) {
  if (device < 0 || device >= kMaxDevices) return fail(ATTN_ERR_INVALID, "bad device %d", device);
  DevState& st = g_dev[device];
  std::lock_guard<std::mutex> lk(st.mu);
  if (st.ready) return ATTN_OK;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= device)
    return fail(ATTN_ERR_NO_DEVICE, "no CUDA device %d visible", device);
  CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(ATTN_ERR_NO_DEVICE, "device %d is sm_%d%d; this runtime is built for sm_100a",
                device, prop.major, prop.minor);
  st.sm_count = prop.multiProcessorCount;
  CUDA_TRY(cudaMalloc(&st.status, sizeof(int32_t)));
  CUDA_TRY(cudaMemset(st.status, 0, sizeof(int32_t)));
  CUDA_TRY(cudaStreamCreateWithFlags(&st.s_compute, cudaStreamNonBlocking));
  CUDA_TRY(cudaStreamCreateWithFlags(&st.s_h2d, cudaStreamNonBlocking));
  CUDA_TRY(cudaStreamCreateWithFlags(&st.s_d2h, cudaStreamNonBlocking));
  for (auto& sb : st.stage) {
    CUDA_TRY(cudaEventCreateWithFlags(&sb.h2d_done, cudaEventDisableTiming));
    CUDA_TRY(cudaEventCreateWithFlags(&sb.comp_done, cudaEventDisableTiming));
    CUDA_TRY(cudaEventCreateWithFlags(&sb.d2h_done, cudaEventDisableTiming));
  }
  cudaMemPoolProps pp{};
  pp.allocType = cudaMemAllocationTypePinned;
  pp.location.type = cudaMemLocationTypeDevice;
  pp.location.id = device;
  CUDA_TRY(cudaMemPoolCreate(&st.pool, &pp));
  uint64_t keep = ~0ull;
  CUDA_TRY(cudaMemPoolSetAttribute(st.pool, cudaMemPoolAttrReleaseThreshold, &keep));
  st.ready = true;
  return ATTN_OK;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(ATTN_ERR_NO_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
  return ATTN_OK;
}

// ------------------------------------------------------------ tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 4-D map over (head_dim, rows, heads, batch) with a 128-byte x 128-row box
// and 128-byte swizzle.  Strides in elements; a unit dimension gets a
// synthetic stride (never stepped along).
// 4-D tensor map [B, H, N, D] (element strides), 128-byte swizzle; the box
// is 128 bytes of D by `box_rows` rows.
int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int eb, int64_t D,
             int64_t N, int64_t H, int64_t B, int64_t s_n, int64_t s_h, int64_t s_b,
             int box_rows = 128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ATTN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (N == 1) s_n = D;
  if (H == 1) s_h = s_n * N;
  if (B == 1) s_b = s_h * H;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_n * eb), static_cast<cuuint64_t>(s_h * eb),
                           static_cast<cuuint64_t>(s_b * eb)};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16 != 0 || strides[i] >= (1ull << 40))
      return fail(ATTN_ERR_ALIGN, "tensor stride %llu bytes is not a multiple of 16",
                  static_cast<unsigned long long>(strides[i]));
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / eb), static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ATTN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return ATTN_OK;
}

// Multiprocessor count of the current device (cached per device).
int sm_count(int* out) {
  static std::atomic<int> cache[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(ATTN_ERR_INVALID, "bad device %d", dev);
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    cache[dev].store(n, std::memory_order_relaxed);
  }
  *out = n;
  return ATTN_OK;
}

// Stream-ordered scratch: from the current device's pool when the runtime
// state is set up (attn_fwd, memref entries), else from the device's default
// pool.  Freed with cudaFreeAsync on the same stream after the kernels.
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices && g_dev[dev].pool)
    return cudaMallocFromPoolAsync(p, bytes, g_dev[dev].pool, s);
  return cudaMallocAsync(p, bytes, s);
}

// KV tiles (of 128 keys) Q tile t of `pair` needs; the kernel's kv_counts.
int pair_tiles(int pair, int t, int64_t Nq, int64_t Nk, bool causal) {
  const int64_t nkv = (Nk + 127) / 128, qs = int64_t(pair) * 256 + 128 * t;
  if (qs >= Nq) return 0;
  if (!causal) return static_cast<int>(nkv);
  return static_cast<int>(std::min<int64_t>(nkv, std::min<int64_t>(qs + 127, Nq - 1) / 128 + 1));
}

// Causal launches with few pairs per SM are bounded by their heaviest pairs,
// which alone take longer than the average CTA's share (one head of
// N = 16384: 64 pairs for 148 CTAs).  The kernel can run the S heaviest pair
// indices of every slice as two halves of their KV tiles (merged in the
// epilogue).  This picks S by replaying the kernel's work order and snake
// assignment on the host and keeping the S with the shortest slowest CTA (0
// unless that gains 2 %).  Costs, in KV steps of a pair: the item's steps,
// +3 per item (Q load, pipeline start and drain, epilogue) and +4 more per
// half (partial write, merge); fitted to B200 timings of 4 heads of
// N = 16384 with S forced from 0 to 64 and of one such head, which the model
// reproduces within 3 %.  Splitting then pays only with very few pairs per
// SM (one head: 1.28x), not for 4 heads (256 pairs on 148 SMs).
int choose_split(int num_bh, int num_pairs, int64_t Nq, int64_t Nk, int G) {
  const int64_t W = int64_t(num_bh) * num_pairs;
  if (num_pairs < 2 || W >= 4ll * G || G <= 0) return 0;
  std::vector<int64_t> load(G);
  std::vector<int> steps(num_pairs), mid(num_pairs);
  for (int pr = 0; pr < num_pairs; ++pr) {
    steps[pr] = std::max(pair_tiles(pr, 0, Nq, Nk, true), pair_tiles(pr, 1, Nq, Nk, true));
    mid[pr] = (steps[pr] + 1) / 2;
  }
  auto makespan = [&](int S) {  // in KV steps
    std::fill(load.begin(), load.end(), 0);
    int64_t w = 0;
    auto add = [&](int64_t cost, int count) {
      for (int k = 0; k < count; ++k, ++w) {
        const int64_t round = w / G, c = w % G;
        load[(round & 1) ? G - 1 - c : c] += cost;
      }
    };
    for (int j = 0; j < S; ++j) {
      const int pr = num_pairs - 1 - j;
      add(mid[pr] + 7, num_bh);
      add(steps[pr] - mid[pr] + 7, num_bh);
    }
    for (int pr = num_pairs - 1 - S; pr >= 0; --pr) add(steps[pr] + 3, num_bh);
    return *std::max_element(load.begin(), load.end());
  };
  const int64_t base = makespan(0);
  int best = 0;
  int64_t best_t = base;
  const int step = std::max(1, num_pairs / 32);
  for (int S = 1; S <= num_pairs; S += (S < 8 ? 1 : step)) {
    const int64_t t = makespan(S);
    if (t < best_t) {
      best_t = t;
      best = S;
    }
  }
  return best_t * 50 < base * 49 ? best : 0;
}

// Causal launches with a few items per CTA (B8 H16 N1024: 512 pairs of 2-8
// KV steps on 148 CTAs) are unbalanced by the snake's last rounds: with the
// costs above (steps + 3) its slowest CTA has 32 units against an average of
// 27.7.  The kernel can instead read the work list through a permutation
// (FwdParams::order): every CTA keeps its snake positions (so its number of
// items), and the items are dealt heaviest first to the CTA with the lowest
// load plus its remaining positions times the average remaining item cost
// (29 units for that shape).  Used only when the model gains at least 2 %;
// the permutation is planned once per device and shape, kept in device
// memory for the life of the process (at most kMaxOrders shapes per device),
// and planned before any stream capture by a first call of the shape.
constexpr size_t kMaxOrders = 64;
struct OrderEntry {
  int num_bh, num_pairs, G;
  int64_t Nq, Nk;
  int* order;  // device permutation, or nullptr: the snake is as good
};
std::mutex g_order_mu;
std::vector<OrderEntry> g_orders[kMaxDevices];

// Host plan: perm[position] = item, or an empty vector to keep the snake.
std::vector<int> plan_causal_order(int num_bh, int num_pairs, int64_t Nq, int64_t Nk, int G) {
  const int64_t W = int64_t(num_bh) * num_pairs;
  std::vector<int> perm;
  if (G <= 0 || W <= G || W >= 8ll * G) return perm;
  // Item w is pair num_pairs - 1 - w / num_bh (decode_item, no split):
  // non-increasing cost in w.
  std::vector<int64_t> cost(W);
  for (int64_t w = 0; w < W; ++w) {
    const int pr = num_pairs - 1 - static_cast<int>(w / num_bh);
    cost[w] = std::max(pair_tiles(pr, 0, Nq, Nk, true), pair_tiles(pr, 1, Nq, Nk, true)) + 3;
  }
  std::vector<std::vector<int>> pos(G);
  for (int64_t w = 0; w < W; ++w) {
    const int64_t round = w / G, c = w % G;
    pos[(round & 1) ? G - 1 - c : c].push_back(static_cast<int>(w));
  }
  int64_t snake = 0, total = 0;
  for (int c = 0; c < G; ++c) {
    int64_t s = 0;
    for (int w : pos[c]) s += cost[w];
    snake = std::max(snake, s);
  }
  for (int64_t w = 0; w < W; ++w) total += cost[w];
  std::vector<int64_t> load(G, 0);
  std::vector<std::vector<int>> got(G);
  int64_t rem_sum = total, rem_n = W, span = 0;
  for (int64_t w = 0; w < W; ++w) {
    const double avg = rem_n > 1 ? double(rem_sum - cost[w]) / double(rem_n - 1) : 0.0;
    int best = -1;
    double best_key = 0.0;
    for (int c = 0; c < G; ++c) {
      const int64_t left = static_cast<int64_t>(pos[c].size() - got[c].size());
      if (left <= 0) continue;
      const double key = double(load[c] + cost[w]) + double(left - 1) * avg;
      if (best < 0 || key < best_key) {
        best = c;
        best_key = key;
      }
    }
    load[best] += cost[w];
    got[best].push_back(static_cast<int>(w));
    span = std::max(span, load[best]);
    rem_sum -= cost[w];
    --rem_n;
  }
  if (span * 50 >= snake * 49) return perm;
  perm.assign(W, -1);
  for (int c = 0; c < G; ++c)
    for (size_t k = 0; k < pos[c].size(); ++k) perm[pos[c][k]] = got[c][k];
  std::vector<char> seen(W, 0);
  for (int v : perm) {
    if (v < 0 || v >= W || seen[v]) return std::vector<int>();  // not a permutation: keep the snake
    seen[v] = 1;
  }
  return perm;
}

// The device permutation for this shape (planned and uploaded on first use),
// or nullptr for the plain snake.
int causal_order(int num_bh, int num_pairs, int64_t Nq, int64_t Nk, int G, const int** out) {
  *out = nullptr;
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return ATTN_OK;
  std::lock_guard<std::mutex> lock(g_order_mu);
  for (const OrderEntry& e : g_orders[dev])
    if (e.num_bh == num_bh && e.num_pairs == num_pairs && e.G == G && e.Nq == Nq && e.Nk == Nk) {
      *out = e.order;
      return ATTN_OK;
    }
  if (g_orders[dev].size() >= kMaxOrders) return ATTN_OK;
  OrderEntry e{num_bh, num_pairs, G, Nq, Nk, nullptr};
  const std::vector<int> perm = plan_causal_order(num_bh, num_pairs, Nq, Nk, G);
  if (!perm.empty()) {
    CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&e.order), perm.size() * sizeof(int)));
    const cudaError_t ce =
        cudaMemcpy(e.order, perm.data(), perm.size() * sizeof(int), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
      cudaFree(e.order);
      return cuda_fail(ce, "cudaMemcpy (work order)");
    }
  }
  g_orders[dev].push_back(e);
  *out = e.order;
  return ATTN_OK;
}

// -------------------------------------------------------------- launches
template <int D, int MODE, int ELT>
int launch_sm100(const AttnDesc& d, int32_t* status, cudaStream_t stream, bool may_split) {
  using C = attn_sm100::FwdCfg<D, ELT>;
  constexpr bool FP8 = C::FP8;
  constexpr bool kCausal = MODE == attn_sm100::kMaskCausal;
  auto kern = attn_sm100::attn_fwd_sm100_kernel<D, MODE, ELT, false>;
  // The causal mode also has the KV-split specialisation.
  auto kern_split = attn_sm100::attn_fwd_sm100_kernel<D, MODE, ELT, kCausal>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  static int launch_regs = 0;
  std::call_once(once, [&] {
    for (auto k : {kern, kern_split}) {
      if (attr_err != cudaSuccess) break;
      attr_err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(C::kSmemBytes));
      cudaFuncAttributes fa{};
      if (attr_err == cudaSuccess) attr_err = cudaFuncGetAttributes(&fa, k);
      launch_regs = launch_regs == 0 ? fa.numRegs : std::min(launch_regs, fa.numRegs);
    }
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute");
  // The kernel re-divides its registers between warpgroups (setmaxnreg); a
  // build whose launch register count cannot cover the split must not run.
  if (launch_regs * attn_sm100::kThreads < attn_sm100::kRegPool)
    return fail(ATTN_ERR_UNSUPPORTED,
                "kernel built with %d registers per thread; the register split needs %d",
                launch_regs, attn_sm100::kRegPool / attn_sm100::kThreads);
  const CUtensorMapDataType dt =
      FP8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
          : (ELT == attn_sm100::kEltF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  const int eb = FP8 ? 1 : 2;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, d.q, dt, eb, d.D, d.Nq, d.Hq, d.B, d.q_stride[2], d.q_stride[1],
                     d.q_stride[0])) != ATTN_OK)
    return rc;
  if ((rc = make_map(&mk, d.k, dt, eb, d.D, d.Nk, d.Hkv, d.B, d.k_stride[2], d.k_stride[1],
                     d.k_stride[0])) != ATTN_OK)
    return rc;
  if ((rc = make_map(&mv, d.v, dt, eb, d.D, d.Nk, d.Hkv, d.B, d.v_stride[2], d.v_stride[1],
                     d.v_stride[0])) != ATTN_OK)
    return rc;
  // O is written by TMA tensor stores of 32-row boxes (one per softmax warp).
  CUtensorMap mo;
  const CUtensorMapDataType dto = d.out_dtype == ATTN_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : d.out_dtype == ATTN_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if ((rc = make_map(&mo, d.o, dto, d.out_dtype == ATTN_F32 ? 4 : 2, d.D, d.Nq, d.Hq, d.B,
                     d.o_stride[2], d.o_stride[1], d.o_stride[0], 32)) != ATTN_OK)
    return rc;
  attn_sm100::FwdParams p{};
  p.o = d.o;
  p.o_sb = d.o_stride[0];
  p.o_sh = d.o_stride[1];
  p.o_sn = d.o_stride[2];
  p.lse = d.lse;
  p.status = status;
  p.Hq = static_cast<int>(d.Hq);
  p.group = static_cast<int>(d.Hq / d.Hkv);
  p.Nq = static_cast<int>(d.Nq);
  p.Nk = static_cast<int>(d.Nk);
  p.num_pairs = static_cast<int>((d.Nq + 255) / 256);
  float sl2 = d.scale * 1.4426950408889634f;
  if (FP8) sl2 *= d.q_descale * d.k_descale;
  if (sl2 == 0.f) sl2 = 1e-30f;  // scale 0: uniform weights without 0*inf
  p.scale_log2 = sl2;
  p.o_scale = FP8 ? d.v_descale : 1.f;
  if (FP8) {
    p.qd_blk = d.q_descale_blocks;
    p.kd_blk = d.k_descale_blocks;
    p.vd_head = d.v_descale_heads;
    p.nqb = static_cast<int>((d.Nq + 127) / 128);
    p.nkb = static_cast<int>((d.Nk + 127) / 128);
  }
  p.out_kind = d.out_dtype == ATTN_F32 ? 1 : (d.out_dtype == ATTN_F16 ? 2 : 0);
  if (MODE == attn_sm100::kMaskDense) {
    p.mask = d.mask;
    p.m_sb = d.mask_stride[0];
    p.m_sh = d.mask_stride[1];
    p.m_sn = d.mask_stride[2];
    const bool rows_aligned = (reinterpret_cast<uintptr_t>(d.mask) & 15u) == 0 &&
                              (d.Nq == 1 || d.mask_stride[2] % 16 == 0) &&
                              (d.Hq == 1 || d.mask_stride[1] % 16 == 0) &&
                              (d.B == 1 || d.mask_stride[0] % 16 == 0);
    p.mask_vec = rows_aligned ? 1 : 0;
  }
  p.num_bh = static_cast<int>(d.B * d.Hq);
  // Dense masks: classify the mask's 128 x 128 blocks first (stream-ordered
  // scratch, freed after the attention kernel) so that fully masked KV tiles
  // are skipped and unmasked ones need no per-element select.
  uint8_t* cls = nullptr;
  if (MODE == attn_sm100::kMaskDense) {
    const int64_t nqt = (d.Nq + 127) / 128, nkt = (d.Nk + 127) / 128;
    const int64_t Bm = (d.B == 1 || d.mask_stride[0] == 0) ? 1 : d.B;
    const int64_t Hm = (d.Hq == 1 || d.mask_stride[1] == 0) ? 1 : d.Hq;
    const int64_t blocks = Bm * Hm * nqt * nkt;  // one warp each
    const int64_t ctas = (blocks + attn_sm100::kClassifyWarps - 1) / attn_sm100::kClassifyWarps;
    const int64_t items = static_cast<int64_t>(p.num_bh) * p.num_pairs;
    if (ctas >= (1ll << 31)) return fail(ATTN_ERR_SHAPE, "dense mask too large to classify");
    // One scratch block: classes, non-empty blocks per (slice, Q tile) (i32),
    // item weights (u16), the work order (i32).
    auto r256 = [](size_t n) { return (n + 255) / 256 * 256; };
    const size_t cls_bytes = r256(static_cast<size_t>(blocks));
    const size_t cnt_bytes = r256(static_cast<size_t>(Bm * Hm * nqt) * 4);
    const size_t w_bytes = r256(static_cast<size_t>(items) * 2);
    cudaError_t e = scratch_alloc(reinterpret_cast<void**>(&cls),
                                  cls_bytes + cnt_bytes + w_bytes + static_cast<size_t>(items) * 4,
                                  stream);
    if (e != cudaSuccess) return cuda_fail(e, "stream-ordered scratch (mask tile classes)");
    int* row_count = reinterpret_cast<int*>(cls + cls_bytes);
    uint16_t* weights = reinterpret_cast<uint16_t*>(cls + cls_bytes + cnt_bytes);
    int* order = reinterpret_cast<int*>(cls + cls_bytes + cnt_bytes + w_bytes);
    e = cudaMemsetAsync(row_count, 0, cnt_bytes, stream);
    if (e != cudaSuccess) {
      cudaFreeAsync(cls, stream);
      return cuda_fail(e, "cudaMemsetAsync (mask block counts)");
    }
    attn_sm100::classify_mask_tiles<<<static_cast<unsigned>(ctas), attn_sm100::kClassifyWarps * 32,
                                      0, stream>>>(
        d.mask, Bm == 1 ? 0 : d.mask_stride[0], Hm == 1 ? 0 : d.mask_stride[1], d.mask_stride[2],
        static_cast<int>(Hm), static_cast<int>(nqt), static_cast<int>(d.Nq),
        static_cast<int>(d.Nk), static_cast<int>(nkt), p.mask_vec, cls, row_count, blocks);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
      cudaFreeAsync(cls, stream);
      return cuda_fail(e, "classify_mask_tiles launch");
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    p.tile_cls = cls;
    p.cls_sb = Bm == 1 ? 0 : Hm * nqt * nkt;
    p.cls_sh = Hm == 1 ? 0 : nqt * nkt;
    p.nkt = static_cast<int>(nkt);
    attn_sm100::order_dense_items<<<1, 1024, 0, stream>>>(
        cls, row_count, p.cls_sb, p.cls_sh, p.Hq, p.num_bh, p.num_pairs, static_cast<int>(nqt),
        p.nkt, weights, order);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
      cudaFreeAsync(cls, stream);
      return cuda_fail(e, "order_dense_items launch");
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    p.order = order;
  }
  // Persistent launch: one CTA per SM (TMEM and shared memory allow one),
  // each walking its share of the (slice, Q-tile pair) work list.
  int sms = 0;
  if ((rc = sm_count(&sms)) != ATTN_OK) {
    if (cls) cudaFreeAsync(cls, stream);
    return rc;
  }
  // Causal KV split of the heaviest pairs when the schedule's tail needs it
  // (never on the no-allocation path: its scratch is stream-ordered).
  unsigned char* part = nullptr;
  if (kCausal && may_split) p.split_pairs = choose_split(p.num_bh, p.num_pairs, d.Nq, d.Nk, sms);
  if (p.split_pairs > 0) {
    const size_t nsplit = static_cast<size_t>(p.split_pairs) * p.num_bh;
    auto r256 = [](size_t n) { return (n + 255) / 256 * 256; };
    const size_t o_bytes = r256(nsplit * 4 * 128 * D * sizeof(float));
    const size_t l_bytes = r256(nsplit * 4 * 128 * sizeof(float));
    const size_t c_bytes = r256(nsplit * 8 * sizeof(int));
    cudaError_t e = scratch_alloc(reinterpret_cast<void**>(&part), o_bytes + l_bytes + c_bytes,
                                  stream);
    if (e != cudaSuccess) return cuda_fail(e, "stream-ordered scratch (KV-split partials)");
    p.part_o = reinterpret_cast<float4*>(part);
    p.part_lse = reinterpret_cast<float*>(part + o_bytes);
    p.part_cnt = reinterpret_cast<int*>(part + o_bytes + l_bytes);
    e = cudaMemsetAsync(p.part_cnt, 0, c_bytes, stream);
    if (e != cudaSuccess) {
      cudaFreeAsync(part, stream);
      return cuda_fail(e, "cudaMemsetAsync (KV-split counters)");
    }
  }
  const int64_t items = attn_sm100::work_items(p.num_bh, p.num_pairs, p.split_pairs);
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(items, sms)));
  // Causal, unsplit: the work list through a balancing permutation where the
  // snake leaves a long tail (never on the no-allocation path, which plans
  // nothing).
  if (kCausal && may_split && p.split_pairs == 0) {
    const int* order = nullptr;
    if ((rc = causal_order(p.num_bh, p.num_pairs, d.Nq, d.Nk, static_cast<int>(grid.x), &order)) !=
        ATTN_OK) {
      if (cls) cudaFreeAsync(cls, stream);
      return rc;
    }
    p.order = order;
  }
  (p.split_pairs > 0 ? kern_split : kern)<<<grid, attn_sm100::kThreads, C::kSmemBytes, stream>>>(
      mq, mk, mv, mo, p);
  cudaError_t e = cudaGetLastError();
  if (cls) cudaFreeAsync(cls, stream);
  if (part) cudaFreeAsync(part, stream);
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd_sm100 launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ATTN_OK;
}

// fp32, head_dim 64 or 128 with every operand row 16-byte aligned: the
// register-tiled kernel.
template <int D>
int launch_f32_tiled(const AttnDesc& d, cudaStream_t stream) {
  auto kern = attn_f32::attn_fwd_f32_tiled<D>;
  constexpr size_t smem = attn_f32::f32_tiled_smem_bytes<D>();
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem));
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute");
  attn_f32::F32Params p{};
  p.q = static_cast<const float*>(d.q);
  p.k = static_cast<const float*>(d.k);
  p.v = static_cast<const float*>(d.v);
  p.o = static_cast<float*>(d.o);
  p.lse = d.lse;
  p.mask = d.mask;
  p.q_sb = d.q_stride[0]; p.q_sh = d.q_stride[1]; p.q_sn = d.q_stride[2];
  p.k_sb = d.k_stride[0]; p.k_sh = d.k_stride[1]; p.k_sn = d.k_stride[2];
  p.v_sb = d.v_stride[0]; p.v_sh = d.v_stride[1]; p.v_sn = d.v_stride[2];
  p.o_sb = d.o_stride[0]; p.o_sh = d.o_stride[1]; p.o_sn = d.o_stride[2];
  p.m_sb = d.mask_stride[0]; p.m_sh = d.mask_stride[1]; p.m_sn = d.mask_stride[2];
  p.Hq = static_cast<int>(d.Hq);
  p.group = static_cast<int>(d.Hq / d.Hkv);
  p.Nq = static_cast<int>(d.Nq);
  p.Nk = static_cast<int>(d.Nk);
  p.D = D;
  p.mask_kind = d.mask_kind;
  p.scale = d.scale;
  p.vec4 = 1;
  dim3 grid(static_cast<unsigned>((d.Nq + attn_f32::kTBM - 1) / attn_f32::kTBM),
            static_cast<unsigned>(d.B * d.Hq));
  kern<<<grid, attn_f32::kTThreads, smem, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd_f32_tiled launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ATTN_OK;
}

// Rows of Q, K, V and O start on 16-byte boundaries (float4 access).
bool f32_rows_aligned(const AttnDesc& d) {
  auto ok = [](const void* p, const int64_t* st) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && st[0] % 4 == 0 && st[1] % 4 == 0 &&
           st[2] % 4 == 0;
  };
  return ok(d.q, d.q_stride) && ok(d.k, d.k_stride) && ok(d.v, d.v_stride) &&
         ok(d.o, d.o_stride);
}

template <int DMAX>
int launch_f32(const AttnDesc& d, cudaStream_t stream) {
  auto kern = attn_f32::attn_fwd_f32_kernel<DMAX>;
  constexpr size_t smem = attn_f32::f32_smem_bytes<DMAX>();
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem));
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute");
  attn_f32::F32Params p{};
  p.q = static_cast<const float*>(d.q);
  p.k = static_cast<const float*>(d.k);
  p.v = static_cast<const float*>(d.v);
  p.o = static_cast<float*>(d.o);
  p.lse = d.lse;
  p.mask = d.mask;
  p.q_sb = d.q_stride[0]; p.q_sh = d.q_stride[1]; p.q_sn = d.q_stride[2];
  p.k_sb = d.k_stride[0]; p.k_sh = d.k_stride[1]; p.k_sn = d.k_stride[2];
  p.v_sb = d.v_stride[0]; p.v_sh = d.v_stride[1]; p.v_sn = d.v_stride[2];
  p.o_sb = d.o_stride[0]; p.o_sh = d.o_stride[1]; p.o_sn = d.o_stride[2];
  p.m_sb = d.mask_stride[0]; p.m_sh = d.mask_stride[1]; p.m_sn = d.mask_stride[2];
  p.Hq = static_cast<int>(d.Hq);
  p.group = static_cast<int>(d.Hq / d.Hkv);
  p.Nq = static_cast<int>(d.Nq);
  p.Nk = static_cast<int>(d.Nk);
  p.D = static_cast<int>(d.D);
  p.mask_kind = d.mask_kind;
  p.scale = d.scale;
  p.vec4 = (d.D % 4 == 0 && d.k_stride[2] % 4 == 0 && d.v_stride[2] % 4 == 0 &&
            d.k_stride[1] % 4 == 0 && d.v_stride[1] % 4 == 0 && d.k_stride[0] % 4 == 0 &&
            d.v_stride[0] % 4 == 0 && (reinterpret_cast<uintptr_t>(d.k) & 15u) == 0 &&
            (reinterpret_cast<uintptr_t>(d.v) & 15u) == 0) ? 1 : 0;
  dim3 grid(static_cast<unsigned>((d.Nq + attn_f32::kRows - 1) / attn_f32::kRows),
            static_cast<unsigned>(d.B * d.Hq));
  kern<<<grid, attn_f32::kRows * 32, smem, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd_f32 launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ATTN_OK;
}

// Failure-detection self-test: one CTA waits, with the bounded wait every
// kernel here uses, on an mbarrier that nothing ever arrives on.
__global__ void probe_timeout_kernel(uint64_t limit_ns, int32_t* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    attn_sm100::mbar_init(&bar, 1);
    abort_flag = 0;
    attn_sm100::fence_mbar_init();
  }
  __syncthreads();
  attn_sm100::mbar_wait_bounded(&bar, 0, &abort_flag, status, limit_ns);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Empty extents, handled as the reference's loop nest (TilingPass.cpp:188,208)
// handles them: no query row (B, Hq or Nq = 0) computes nothing; no key
// (Nk = 0) runs no KV step, leaving O_acc = 0 and l = 0, so every output row
// is 0/0 = NaN and the LSE m + ln l is -inf.  Sets the two flags; the full
// validation (validate) applies only to calls with rows and keys.
int check_empty(const AttnDesc& d, bool* no_rows, bool* no_keys) {
  *no_rows = *no_keys = false;
  if (d.B < 0 || d.Hq < 0 || d.Hkv < 0 || d.Nq < 0 || d.Nk < 0 || d.D < 0)
    return fail(ATTN_ERR_SHAPE, "extents must not be negative");
  const bool rows = d.B == 0 || d.Hq == 0 || d.Nq == 0;
  if (!rows && d.Nk != 0) return ATTN_OK;
  if (d.flags != 0) return fail(ATTN_ERR_INVALID, "flags must be 0");
  if (d.dtype != ATTN_F32 && d.dtype != ATTN_BF16 && d.dtype != ATTN_F16 && d.dtype != ATTN_E4M3)
    return fail(ATTN_ERR_DTYPE, "unknown dtype %d", d.dtype);
  if (d.out_dtype != ATTN_F32 && d.out_dtype != ATTN_BF16 && d.out_dtype != ATTN_F16)
    return fail(ATTN_ERR_DTYPE, "unknown output dtype %d", d.out_dtype);
  if (d.mask_kind < ATTN_MASK_NONE || d.mask_kind > ATTN_MASK_DENSE)
    return fail(ATTN_ERR_INVALID, "unknown mask kind %d", d.mask_kind);
  if (d.Hq > 0 && (d.Hkv <= 0 || d.Hq % d.Hkv != 0))
    return fail(ATTN_ERR_SHAPE, "query heads (%lld) must be a multiple of key/value heads (%lld)",
                (long long)d.Hq, (long long)d.Hkv);
  *no_rows = rows;
  *no_keys = !rows;
  if (*no_keys && d.D > 0 && !d.o) return fail(ATTN_ERR_INVALID, "null output pointer");
  return ATTN_OK;
}

// Output of a call without keys, in device memory: O rows NaN, LSE -inf.
__global__ void fill_no_keys(void* o, int out_kind, int64_t sb, int64_t sh, int64_t sn, int64_t Hq,
                             int64_t Nq, int64_t D, float* lse, int64_t rows) {
  const int64_t total = rows * D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / D, c = i - (i / D) * D;  // r = (b * Hq + h) * Nq + n
    const int64_t n = r % Nq, bh = r / Nq, b = bh / Hq, h = bh % Hq;
    const int64_t off = b * sb + h * sh + n * sn + c;
    if (out_kind == 1)
      static_cast<float*>(o)[off] = __int_as_float(0x7fc00000);
    else
      static_cast<uint16_t*>(o)[off] = out_kind == 2 ? 0x7e00 : 0x7fc0;
    if (lse && c == 0) lse[r] = -INFINITY;
  }
}

// The same in host memory (host memref operands).
void fill_no_keys_host(const AttnDesc& d) {
  for (int64_t b = 0; b < d.B; ++b)
    for (int64_t h = 0; h < d.Hq; ++h)
      for (int64_t n = 0; n < d.Nq; ++n) {
        const int64_t off = b * d.o_stride[0] + h * d.o_stride[1] + n * d.o_stride[2];
        for (int64_t c = 0; c < d.D; ++c) {
          if (d.out_dtype == ATTN_F32) {
            static_cast<float*>(d.o)[off + c] = std::numeric_limits<float>::quiet_NaN();
          } else {
            static_cast<uint16_t*>(d.o)[off + c] = d.out_dtype == ATTN_F16 ? 0x7e00 : 0x7fc0;
          }
        }
        if (d.lse) d.lse[(b * d.Hq + h) * d.Nq + n] = -std::numeric_limits<float>::infinity();
      }
}

int validate(const AttnDesc& d) {
  if (!d.q || !d.k || !d.v || !d.o) return fail(ATTN_ERR_INVALID, "null Q/K/V/output pointer");
  if (d.flags != 0) return fail(ATTN_ERR_INVALID, "flags must be 0");
  if (d.B <= 0 || d.Hq <= 0 || d.Hkv <= 0 || d.Nq <= 0 || d.Nk <= 0 || d.D <= 0)
    return fail(ATTN_ERR_SHAPE, "all extents must be positive (B=%lld Hq=%lld Hkv=%lld Nq=%lld "
                "Nk=%lld D=%lld)", (long long)d.B, (long long)d.Hq, (long long)d.Hkv,
                (long long)d.Nq, (long long)d.Nk, (long long)d.D);
  if (d.Hq % d.Hkv != 0)
    return fail(ATTN_ERR_SHAPE, "query heads (%lld) must be a multiple of key/value heads (%lld)",
                (long long)d.Hq, (long long)d.Hkv);
  if (d.Nq >= (1ll << 31) || d.Nk >= (1ll << 31) || d.B * d.Hq >= (1ll << 31))
    return fail(ATTN_ERR_SHAPE, "extent too large");
  if (d.mask_kind < ATTN_MASK_NONE || d.mask_kind > ATTN_MASK_DENSE)
    return fail(ATTN_ERR_INVALID, "unknown mask kind %d", d.mask_kind);
  if (d.mask_kind == ATTN_MASK_DENSE && !d.mask)
    return fail(ATTN_ERR_INVALID, "dense mask requested without a mask pointer");
  if (!std::isfinite(d.scale)) return fail(ATTN_ERR_INVALID, "scale must be finite");
  const bool blocks = d.q_descale_blocks || d.k_descale_blocks || d.v_descale_heads;
  if (blocks && d.dtype != ATTN_E4M3)
    return fail(ATTN_ERR_DTYPE, "per-block descales apply to e4m3 inputs only");
  for (const float* b : {d.q_descale_blocks, d.k_descale_blocks, d.v_descale_heads})
    if ((reinterpret_cast<uintptr_t>(b) & 3u) != 0)
      return fail(ATTN_ERR_ALIGN, "per-block descale arrays must be 4-byte aligned");
  switch (d.dtype) {
    case ATTN_F32:
      if (d.out_dtype != ATTN_F32)
        return fail(ATTN_ERR_DTYPE, "f32 inputs produce an f32 output");
      if (d.D > 256) return fail(ATTN_ERR_UNSUPPORTED, "f32 path supports head_dim <= 256");
      return ATTN_OK;
    case ATTN_BF16:
    case ATTN_F16:
    case ATTN_E4M3: {
      if (d.out_dtype != ATTN_BF16 && d.out_dtype != ATTN_F32 && d.out_dtype != ATTN_F16)
        return fail(ATTN_ERR_DTYPE, "output must be bf16, f16 or f32");
      if (d.dtype != ATTN_E4M3 && d.D != 64 && d.D != 128)
        return fail(ATTN_ERR_UNSUPPORTED, "bf16/f16 path supports head_dim 64 or 128 (got %lld)",
                    (long long)d.D);
      if (d.dtype == ATTN_E4M3 && d.D != 128)
        return fail(ATTN_ERR_UNSUPPORTED, "e4m3 path supports head_dim 128 (got %lld)",
                    (long long)d.D);
      if (d.dtype == ATTN_E4M3 && !(d.q_descale > 0.f && d.k_descale > 0.f && d.v_descale > 0.f))
        return fail(ATTN_ERR_INVALID, "e4m3 descales must be positive");
      if (!aligned16(d.q) || !aligned16(d.k) || !aligned16(d.v) || !aligned16(d.o))
        return fail(ATTN_ERR_ALIGN, "Q/K/V/output must be 16-byte aligned");
      const int64_t ob = d.out_dtype == ATTN_F32 ? 4 : 2;
      for (int i = 0; i < 3; ++i)
        if ((d.o_stride[i] * ob) % 16 != 0 &&
            !((i == 0 && d.B == 1) || (i == 1 && d.Hq == 1) || (i == 2 && d.Nq == 1)))
          return fail(ATTN_ERR_ALIGN, "output strides must be multiples of 16 bytes");
      return ATTN_OK;
    }
    default:
      return fail(ATTN_ERR_DTYPE, "unknown dtype %d", d.dtype);
  }
}

template <int D, int ELT>
int dispatch_mode(const AttnDesc& d, int32_t* status, cudaStream_t s, bool may_split) {
  switch (d.mask_kind) {
    case ATTN_MASK_CAUSAL:
      return launch_sm100<D, attn_sm100::kMaskCausal, ELT>(d, status, s, may_split);
    case ATTN_MASK_DENSE:
      return launch_sm100<D, attn_sm100::kMaskDense, ELT>(d, status, s, may_split);
    default: return launch_sm100<D, attn_sm100::kMaskNone, ELT>(d, status, s, may_split);
  }
}

// may_split = false: no stream-ordered scratch (the no-allocation entry).
int dispatch(const AttnDesc& d, int32_t* status, cudaStream_t s, bool may_split = true) {
  if (d.dtype == ATTN_F32) {
    if ((d.D == 64 || d.D == 128) && f32_rows_aligned(d))
      return d.D == 64 ? launch_f32_tiled<64>(d, s) : launch_f32_tiled<128>(d, s);
    if (d.D <= 64) return launch_f32<64>(d, s);
    if (d.D <= 128) return launch_f32<128>(d, s);
    return launch_f32<256>(d, s);
  }
  using namespace attn_sm100;
  if (d.dtype == ATTN_BF16)
    return d.D == 64 ? dispatch_mode<64, kEltBF16>(d, status, s, may_split)
                     : dispatch_mode<128, kEltBF16>(d, status, s, may_split);
  if (d.dtype == ATTN_F16)
    return d.D == 64 ? dispatch_mode<64, kEltF16>(d, status, s, may_split)
                     : dispatch_mode<128, kEltF16>(d, status, s, may_split);
  return dispatch_mode<128, kEltE4M3>(d, status, s, may_split);
}

// ------------------------------------------------- memref-descriptor layer
struct View {
  char* ptr = nullptr;
  int64_t size[4] = {1, 1, 1, 1};   // B, H, N, D
  int64_t stride[4] = {0, 0, 0, 1};
};

View view2(const AttnMemRef2D* m, int eb) {
  View v;
  v.ptr = static_cast<char*>(m->aligned) + m->offset * eb;
  v.size[2] = m->sizes[0];
  v.size[3] = m->sizes[1];
  v.stride[2] = m->strides[0];
  v.stride[3] = m->strides[1];
  v.stride[1] = m->sizes[0] * m->strides[0];
  v.stride[0] = v.stride[1];
  return v;
}

View view4(const AttnMemRef4D* m, int eb) {
  View v;
  v.ptr = static_cast<char*>(m->aligned) + m->offset * eb;
  for (int i = 0; i < 4; ++i) {
    v.size[i] = m->sizes[i];
    v.stride[i] = m->strides[i];
  }
  return v;
}

bool is_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// The reference verifier's shape rules (AttentionOps.cpp:48-56), extended to
// batch/head extents; V's head_dim is also checked (the reference does not).
int verify_views(const View& Q, const View& K, const View& V, const View& O) {
  if (K.size[3] != Q.size[3]) return fail(ATTN_ERR_SHAPE, "K head_dim must equal Q head_dim");
  if (V.size[2] != K.size[2]) return fail(ATTN_ERR_SHAPE, "V seq_len must equal K seq_len");
  if (O.size[2] != Q.size[2]) return fail(ATTN_ERR_SHAPE, "output seq_q must equal Q seq_q");
  if (O.size[3] != Q.size[3]) return fail(ATTN_ERR_SHAPE, "output head_dim must equal Q head_dim");
  if (V.size[3] != Q.size[3]) return fail(ATTN_ERR_SHAPE, "V head_dim must equal Q head_dim");
  if (K.size[0] != Q.size[0] || V.size[0] != Q.size[0] || O.size[0] != Q.size[0])
    return fail(ATTN_ERR_SHAPE, "batch extents must match");
  if (V.size[1] != K.size[1] || O.size[1] != Q.size[1])
    return fail(ATTN_ERR_SHAPE, "head extents must match");
  for (const View* v : {&Q, &K, &V, &O})
    if (v->stride[3] != 1) return fail(ATTN_ERR_STRIDE, "head_dim must be the unit-stride dimension");
  return ATTN_OK;
}

AttnDesc desc_from_views(int dtype, int out_dtype, int mask_kind, const View& Q, const View& K,
                         const View& V, const View& O, float scale) {
  AttnDesc d{};
  d.dtype = dtype;
  d.out_dtype = out_dtype;
  d.mask_kind = mask_kind;
  d.B = Q.size[0];
  d.Hq = Q.size[1];
  d.Hkv = K.size[1];
  d.Nq = Q.size[2];
  d.Nk = K.size[2];
  d.D = Q.size[3];
  for (int i = 0; i < 3; ++i) {
    d.q_stride[i] = Q.stride[i];
    d.k_stride[i] = K.stride[i];
    d.v_stride[i] = V.stride[i];
    d.o_stride[i] = O.stride[i];
  }
  d.q = Q.ptr;
  d.k = K.ptr;
  d.v = V.ptr;
  d.o = O.ptr;
  d.scale = scale;
  d.q_descale = d.k_descale = d.v_descale = 1.f;
  return d;
}

size_t elem_bytes(int dt) {
  return dt == ATTN_F32 ? 4 : (dt == ATTN_BF16 || dt == ATTN_F16) ? 2 : 1;
}

int ensure(void** p, size_t* have, size_t need) {
  if (*have >= need) return ATTN_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  CUDA_TRY(cudaMalloc(p, need));
  *have = need;
  return ATTN_OK;
}

// Copy `rows` x `D` elements of slice (b, h) between host and device, the
// device side dense ([rows][D]).
cudaError_t copy_slice(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                       size_t rows, cudaMemcpyKind kind, cudaStream_t s) {
  // Dense rows: one linear copy (a 2D copy of 256-byte rows runs slower).
  if (dpitch == width && spitch == width) return cudaMemcpyAsync(dst, src, width * rows, kind, s);
  return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, kind, s);
}

// True if a [B, H, N, D] operand with element strides st is densely packed.
bool packed4(const int64_t st[3], int64_t H, int64_t N, int64_t D) {
  return st[2] == D && st[1] == N * D && st[0] == H * N * D;
}

// Run a call whose operands live in host memory: chunks of (batch, kv-head)
// groups are staged through device buffers, with the H2D copy of chunk c+1,
// the kernels of chunk c and the D2H copy of chunk c-1 overlapped on three
// streams.  Synchronous: returns when O (and LSE) are in host memory.
int run_staged(const AttnDesc& hd, int device) {
  NvtxRange range("attn_rt: host-memref staging");
  DevState& st = g_dev[device];
  std::lock_guard<std::mutex> lk(st.mu);  // one staged call per device at a time
  const size_t eb = elem_bytes(hd.dtype), ob = elem_bytes(hd.out_dtype);
  const int64_t group = hd.Hq / hd.Hkv;
  const int64_t ngroups = hd.B * hd.Hkv;
  // 16 chunks: measured best for c4 over PCIe (8: 9.65 ms, 16: 9.33, 32: 10.08).
  const int64_t per_chunk = std::max<int64_t>(1, (ngroups + 15) / 16);
  const int64_t nchunks = (ngroups + per_chunk - 1) / per_chunk;
  const size_t q_slice = static_cast<size_t>(hd.Nq * hd.D) * eb;
  const size_t kv_slice = static_cast<size_t>(hd.Nk * hd.D) * eb;
  const size_t o_slice = static_cast<size_t>(hd.Nq * hd.D) * ob;
  for (auto& sb : st.stage) {
    int rc;
    if ((rc = ensure(&sb.q, &sb.q_bytes, q_slice * group * per_chunk)) != ATTN_OK) return rc;
    if ((rc = ensure(&sb.k, &sb.k_bytes, kv_slice * per_chunk)) != ATTN_OK) return rc;
    if ((rc = ensure(&sb.v, &sb.v_bytes, kv_slice * per_chunk)) != ATTN_OK) return rc;
    if ((rc = ensure(&sb.o, &sb.o_bytes, o_slice * group * per_chunk)) != ATTN_OK) return rc;
    if (hd.lse) {
      void* l = sb.lse;
      if ((rc = ensure(&l, &sb.lse_bytes, sizeof(float) * hd.Nq * group * per_chunk)) != ATTN_OK)
        return rc;
      sb.lse = static_cast<float*>(l);
    }
  }

  for (int64_t c = 0; c < nchunks; ++c) {
    Staging& sb = st.stage[c % kStageBufs];
    const int64_t g0 = c * per_chunk;
    const int64_t gn = std::min<int64_t>(per_chunk, ngroups - g0);
    if (c >= kStageBufs) CUDA_TRY(cudaStreamWaitEvent(st.s_h2d, sb.d2h_done, 0));
    // Packed operands: a chunk of consecutive (batch, kv-head) groups is one
    // contiguous range of Q, K, V (and O, LSE): one linear copy each.
    const bool packed = packed4(hd.q_stride, hd.Hq, hd.Nq, hd.D) &&
                        packed4(hd.k_stride, hd.Hkv, hd.Nk, hd.D) &&
                        packed4(hd.v_stride, hd.Hkv, hd.Nk, hd.D) &&
                        packed4(hd.o_stride, hd.Hq, hd.Nq, hd.D);
    if (packed) {
      CUDA_TRY(cudaMemcpyAsync(sb.k, static_cast<const char*>(hd.k) + g0 * kv_slice,
                               gn * kv_slice, cudaMemcpyHostToDevice, st.s_h2d));
      CUDA_TRY(cudaMemcpyAsync(sb.v, static_cast<const char*>(hd.v) + g0 * kv_slice,
                               gn * kv_slice, cudaMemcpyHostToDevice, st.s_h2d));
      CUDA_TRY(cudaMemcpyAsync(sb.q, static_cast<const char*>(hd.q) + g0 * group * q_slice,
                               gn * group * q_slice, cudaMemcpyHostToDevice, st.s_h2d));
    }
    for (int64_t g = 0; g < gn && !packed; ++g) {
      const int64_t b = (g0 + g) / hd.Hkv, hk = (g0 + g) % hd.Hkv;
      const char* ks = static_cast<const char*>(hd.k) + (b * hd.k_stride[0] + hk * hd.k_stride[1]) * eb;
      const char* vs = static_cast<const char*>(hd.v) + (b * hd.v_stride[0] + hk * hd.v_stride[1]) * eb;
      CUDA_TRY(copy_slice(static_cast<char*>(sb.k) + g * kv_slice, hd.D * eb, ks,
                          hd.k_stride[2] * eb, hd.D * eb, hd.Nk, cudaMemcpyHostToDevice, st.s_h2d));
      CUDA_TRY(copy_slice(static_cast<char*>(sb.v) + g * kv_slice, hd.D * eb, vs,
                          hd.v_stride[2] * eb, hd.D * eb, hd.Nk, cudaMemcpyHostToDevice, st.s_h2d));
      for (int64_t i = 0; i < group; ++i) {
        const int64_t h = hk * group + i;
        const char* qs = static_cast<const char*>(hd.q) + (b * hd.q_stride[0] + h * hd.q_stride[1]) * eb;
        CUDA_TRY(copy_slice(static_cast<char*>(sb.q) + (g * group + i) * q_slice, hd.D * eb, qs,
                            hd.q_stride[2] * eb, hd.D * eb, hd.Nq, cudaMemcpyHostToDevice,
                            st.s_h2d));
      }
    }
    CUDA_TRY(cudaEventRecord(sb.h2d_done, st.s_h2d));
    CUDA_TRY(cudaStreamWaitEvent(st.s_compute, sb.h2d_done, 0));
    // The chunk on the device is [gn, group, N, D] dense: B' = gn, Hq' = group, Hkv' = 1.
    AttnDesc dd = hd;
    dd.B = gn;
    dd.Hq = group;
    dd.Hkv = 1;
    dd.q = sb.q;
    dd.k = sb.k;
    dd.v = sb.v;
    dd.o = sb.o;
    dd.lse = hd.lse ? sb.lse : nullptr;
    dd.q_stride[2] = hd.D; dd.q_stride[1] = hd.Nq * hd.D; dd.q_stride[0] = group * hd.Nq * hd.D;
    dd.o_stride[2] = hd.D; dd.o_stride[1] = hd.Nq * hd.D; dd.o_stride[0] = group * hd.Nq * hd.D;
    dd.k_stride[2] = hd.D; dd.k_stride[1] = hd.Nk * hd.D; dd.k_stride[0] = hd.Nk * hd.D;
    dd.v_stride[2] = hd.D; dd.v_stride[1] = hd.Nk * hd.D; dd.v_stride[0] = hd.Nk * hd.D;
    dd.mask = nullptr;
    if (hd.mask_kind == ATTN_MASK_DENSE)
      return fail(ATTN_ERR_UNSUPPORTED, "dense masks on host memrefs are not staged");
    int rc = validate(dd);
    if (rc != ATTN_OK) return rc;
    rc = dispatch(dd, st.status, st.s_compute, /*may_split=*/false);
    if (rc != ATTN_OK) return rc;
    CUDA_TRY(cudaEventRecord(sb.comp_done, st.s_compute));
    CUDA_TRY(cudaStreamWaitEvent(st.s_d2h, sb.comp_done, 0));
    if (packed) {
      CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(hd.o) + g0 * group * o_slice, sb.o,
                               gn * group * o_slice, cudaMemcpyDeviceToHost, st.s_d2h));
      if (hd.lse)
        CUDA_TRY(cudaMemcpyAsync(hd.lse + g0 * group * hd.Nq, sb.lse,
                                 sizeof(float) * gn * group * hd.Nq, cudaMemcpyDeviceToHost,
                                 st.s_d2h));
    }
    for (int64_t g = 0; g < gn && !packed; ++g) {
      const int64_t b = (g0 + g) / hd.Hkv, hk = (g0 + g) % hd.Hkv;
      for (int64_t i = 0; i < group; ++i) {
        const int64_t h = hk * group + i;
        char* os = static_cast<char*>(hd.o) + (b * hd.o_stride[0] + h * hd.o_stride[1]) * ob;
        CUDA_TRY(copy_slice(os, hd.o_stride[2] * ob,
                            static_cast<char*>(sb.o) + (g * group + i) * o_slice, hd.D * ob,
                            hd.D * ob, hd.Nq, cudaMemcpyDeviceToHost, st.s_d2h));
        if (hd.lse) {
          float* ls = hd.lse + (b * hd.Hq + h) * hd.Nq;
          CUDA_TRY(cudaMemcpyAsync(ls, sb.lse + (g * group + i) * hd.Nq, sizeof(float) * hd.Nq,
                                   cudaMemcpyDeviceToHost, st.s_d2h));
        }
      }
    }
    CUDA_TRY(cudaEventRecord(sb.d2h_done, st.s_d2h));
  }
  CUDA_TRY(cudaStreamSynchronize(st.s_d2h));
  CUDA_TRY(cudaStreamSynchronize(st.s_compute));
  int32_t code = 0;
  CUDA_TRY(cudaMemcpy(&code, st.status, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (code != 0) {
    CUDA_TRY(cudaMemset(st.status, 0, sizeof(int32_t)));
    return fail(code, "kernel reported %s", attn_rt_status_string(code));
  }
  return ATTN_OK;
}

// Common body of every _mlir_ciface_ entry: device operands run in place on
// the runtime's stream; host operands go through run_staged.
int run_views(int dtype, int out_dtype, int mask_kind, const View& Q, const View& K,
              const View& V, const View& O, float scale, float qd, float kd, float vd,
              const View* L, const View* M) {
  int rc = verify_views(Q, K, V, O);
  if (rc != ATTN_OK) return rc;
  int dev = 0;
  if ((rc = current_device(&dev)) != ATTN_OK) return rc;
  if ((rc = init_device(dev)) != ATTN_OK) return rc;
  AttnDesc d = desc_from_views(dtype, out_dtype, mask_kind, Q, K, V, O, scale);
  d.q_descale = qd;
  d.k_descale = kd;
  d.v_descale = vd;
  if (L && L->size[0] * L->size[1] * L->size[2] * L->size[3] == 0) L = nullptr;  // not requested
  if (L) {
    if (L->size[0] != Q.size[0] || L->size[1] != Q.size[1] || L->size[2] != Q.size[2])
      return fail(ATTN_ERR_SHAPE, "LSE must be [B, H, seq_q]");
    if (L->stride[2] != 1 || L->stride[1] != Q.size[2] || L->stride[0] != Q.size[1] * Q.size[2])
      return fail(ATTN_ERR_STRIDE, "LSE must be contiguous");
    d.lse = reinterpret_cast<float*>(L->ptr);
  }
  if (M) {
    if (M->size[2] != Q.size[2] || M->size[3] != K.size[2])
      return fail(ATTN_ERR_SHAPE, "mask must be [seq_q, seq_k]");
    if (M->stride[3] != 1) return fail(ATTN_ERR_STRIDE, "mask columns must be unit-stride");
    if ((M->size[0] != 1 && M->size[0] != Q.size[0]) || (M->size[1] != 1 && M->size[1] != Q.size[1]))
      return fail(ATTN_ERR_SHAPE, "mask batch/head extents must be 1 or match Q");
    d.mask = reinterpret_cast<const uint8_t*>(M->ptr);
    d.mask_stride[0] = M->size[0] == 1 ? 0 : M->stride[0];  // extent 1 broadcasts
    d.mask_stride[1] = M->size[1] == 1 ? 0 : M->stride[1];
    d.mask_stride[2] = M->stride[2];
  }
  bool no_rows = false, no_keys = false;
  if ((rc = check_empty(d, &no_rows, &no_keys)) != ATTN_OK) return rc;
  if (no_rows) return ATTN_OK;
  if (no_keys && !is_device_ptr(d.o)) {
    fill_no_keys_host(d);
    return ATTN_OK;
  }
  const bool dev_q = no_keys || is_device_ptr(d.q);
  if (dev_q) {
    if (!is_device_ptr(d.k) || !is_device_ptr(d.v) || !is_device_ptr(d.o) ||
        (d.lse && !is_device_ptr(d.lse)) || (d.mask && !is_device_ptr(d.mask)))
      return fail(ATTN_ERR_INVALID, "operands mix host and device memory");
    DevState& st = g_dev[dev];
    if ((rc = attn_fwd(&d, st.s_compute)) != ATTN_OK) return rc;
    return attn_rt_check_status(dev, st.s_compute);
  }
  if (d.mask_kind == ATTN_MASK_DENSE || d.dtype == ATTN_F32) {
    // Small reference-shaped calls (f32, dense masks): stage whole operands.
    const size_t eb = elem_bytes(d.dtype), ob = elem_bytes(d.out_dtype);
    auto span = [](const int64_t* st, int64_t B, int64_t H, int64_t N, int64_t Dd) {
      return ((B - 1) * st[0] + (H - 1) * st[1] + (N - 1) * st[2] + Dd);
    };
    const size_t qn = span(d.q_stride, d.B, d.Hq, d.Nq, d.D) * eb;
    const size_t kn = span(d.k_stride, d.B, d.Hkv, d.Nk, d.D) * eb;
    const size_t vn = span(d.v_stride, d.B, d.Hkv, d.Nk, d.D) * eb;
    const size_t on = span(d.o_stride, d.B, d.Hq, d.Nq, d.D) * ob;
    const size_t mn = d.mask ? static_cast<size_t>((d.B - 1) * d.mask_stride[0] +
                                                   (d.Hq - 1) * d.mask_stride[1] +
                                                   (d.Nq - 1) * d.mask_stride[2] + d.Nk)
                             : 0;
    const size_t ln = d.lse ? sizeof(float) * d.B * d.Hq * d.Nq : 0;
    const size_t total = qn + kn + vn + on + mn + ln + 6 * 256;
    DevState& st = g_dev[dev];
    // One staged call per device at a time; the buffer is kept for the next.
    std::lock_guard<std::mutex> lk(st.whole_mu);
    if ((rc = ensure(&st.whole, &st.whole_bytes, total)) != ATTN_OK) return rc;
    char* buf = static_cast<char*>(st.whole);
    auto carve = [&](size_t n) { char* p = buf; buf += (n + 255) / 256 * 256; return p; };
    char* dq = carve(qn); char* dk = carve(kn); char* dv = carve(vn); char* dout = carve(on);
    char* dm = mn ? carve(mn) : nullptr;
    char* dl = ln ? carve(ln) : nullptr;
    cudaStream_t s = st.s_compute;
    auto cleanup = [&](int code) {
      if (code != ATTN_OK) cudaStreamSynchronize(s);  // nothing may still use the buffer
      return code;
    };
    if (cudaMemcpyAsync(dq, d.q, qn, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(dk, d.k, kn, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(dv, d.v, vn, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        (dm && cudaMemcpyAsync(dm, d.mask, mn, cudaMemcpyHostToDevice, s) != cudaSuccess))
      return cleanup(cuda_fail(cudaGetLastError(), "staging copy"));
    AttnDesc dd = d;
    dd.q = dq; dd.k = dk; dd.v = dv; dd.o = dout;
    dd.mask = reinterpret_cast<const uint8_t*>(dm);
    dd.lse = reinterpret_cast<float*>(dl);
    if ((rc = attn_fwd(&dd, s)) != ATTN_OK) return cleanup(rc);
    if (cudaMemcpyAsync(const_cast<void*>(static_cast<const void*>(d.o)), dout, on,
                        cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        (dl && cudaMemcpyAsync(d.lse, dl, ln, cudaMemcpyDeviceToHost, s) != cudaSuccess))
      return cleanup(cuda_fail(cudaGetLastError(), "staging copy back"));
    rc = attn_rt_check_status(dev, s);
    return cleanup(rc);
  }
  int vrc = validate(d);
  if (vrc != ATTN_OK) return vrc;
  return run_staged(d, dev);
}

}  // namespace

// =================================================================== C ABI
extern "C" {

int attn_rt_version(void) { return (1 << 16) | 1; }

int64_t attn_rt_launch_count(void) { return g_launches.load(); }

int attn_rt_alloc(void** ptr, size_t bytes) {
  if (!ptr || bytes == 0) return fail(ATTN_ERR_INVALID, "attn_rt_alloc: null pointer or 0 bytes");
  *ptr = nullptr;
  int dev = 0, rc;
  if ((rc = current_device(&dev)) != ATTN_OK) return rc;
  if ((rc = init_device(dev)) != ATTN_OK) return rc;
  CUDA_TRY(cudaMalloc(ptr, bytes));
  return ATTN_OK;
}

int attn_rt_free(void* ptr) {
  if (!ptr) return ATTN_OK;
  CUDA_TRY(cudaFree(ptr));
  return ATTN_OK;
}

int attn_rt_copy(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ATTN_OK;
  if (!dst || !src) return fail(ATTN_ERR_INVALID, "attn_rt_copy: null pointer");
  if (stream) {
    CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  } else {
    CUDA_TRY(cudaMemcpy(dst, src, bytes, cudaMemcpyDefault));
  }
  return ATTN_OK;
}

const char* attn_rt_last_error(void) { return g_last_error.c_str(); }

const char* attn_rt_status_string(int code) {
  switch (code) {
    case ATTN_OK: return "ok";
    case ATTN_ERR_INVALID: return "invalid argument";
    case ATTN_ERR_SHAPE: return "shape mismatch";
    case ATTN_ERR_STRIDE: return "unsupported stride";
    case ATTN_ERR_DTYPE: return "unsupported dtype";
    case ATTN_ERR_ALIGN: return "misaligned pointer or stride";
    case ATTN_ERR_CUDA: return "CUDA error";
    case ATTN_ERR_TIMEOUT: return "device wait timed out";
    case ATTN_ERR_UNSUPPORTED: return "unsupported variant";
    case ATTN_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

int attn_rt_init(int device) { return init_device(device); }

int attn_rt_causal_split(int64_t slices, int64_t Nq, int64_t Nk, int sms) {
  if (slices <= 0 || Nq <= 0 || Nk <= 0 || sms <= 0 || slices * ((Nq + 255) / 256) >= (1ll << 31))
    return 0;
  return choose_split(static_cast<int>(slices), static_cast<int>((Nq + 255) / 256), Nq, Nk, sms);
}

int attn_rt_probe_timeout(int64_t limit_ns) {
  if (limit_ns <= 0 || limit_ns > 2000000000ll)
    return fail(ATTN_ERR_INVALID, "probe limit must be in (0, 2 s]");
  int dev = 0, rc;
  if ((rc = current_device(&dev)) != ATTN_OK) return rc;
  if ((rc = init_device(dev)) != ATTN_OK) return rc;
  DevState& st = g_dev[dev];
  probe_timeout_kernel<<<1, 32, 0, st.s_compute>>>(static_cast<uint64_t>(limit_ns), st.status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "probe launch");
  return attn_rt_check_status(dev, st.s_compute);
}

int attn_rt_check_status(int device, void* stream) {
  int rc = init_device(device);
  if (rc != ATTN_OK) return rc;
  DevState& st = g_dev[device];
  CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int32_t code = 0;
  CUDA_TRY(cudaMemcpy(&code, st.status, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (code != 0) {
    CUDA_TRY(cudaMemset(st.status, 0, sizeof(int32_t)));
    return fail(code, "kernel reported %s", attn_rt_status_string(code));
  }
  return ATTN_OK;
}

int attn_fwd(const AttnDesc* desc, void* stream) {
  NvtxRange range("attn_fwd");
  if (!desc) return fail(ATTN_ERR_INVALID, "null descriptor");
  bool no_rows = false, no_keys = false;
  int rc = check_empty(*desc, &no_rows, &no_keys);
  if (rc != ATTN_OK) return rc;
  if (no_rows) return ATTN_OK;
  if (!no_keys && (rc = validate(*desc)) != ATTN_OK) return rc;
  int dev = 0;
  if ((rc = current_device(&dev)) != ATTN_OK) return rc;
  if ((rc = init_device(dev)) != ATTN_OK) return rc;
  {
    // Kernels read these with TMA and plain loads: host memory would fault.
    const AttnDesc& d = *desc;
    const void* need[] = {no_keys ? nullptr : d.q, no_keys ? nullptr : d.k,
                          no_keys ? nullptr : d.v, d.o, d.lse, d.mask, d.q_descale_blocks,
                          d.k_descale_blocks, d.v_descale_heads};
    for (const void* ptr : need)
      if (ptr && !is_device_ptr(ptr))
        return fail(ATTN_ERR_INVALID,
                    "attn_fwd takes device pointers; host buffers go through the memref "
                    "entries or attn_fwd_host_noalloc");
  }
  if (no_keys) {
    const AttnDesc& d = *desc;
    const int64_t rows = d.B * d.Hq * d.Nq;
    if (rows * d.D == 0) return ATTN_OK;
    const int out_kind = d.out_dtype == ATTN_F32 ? 1 : (d.out_dtype == ATTN_F16 ? 2 : 0);
    const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((rows * d.D + 255) / 256, 4096));
    fill_no_keys<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        d.o, out_kind, d.o_stride[0], d.o_stride[1], d.o_stride[2], d.Hq, d.Nq, d.D, d.lse, rows);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "fill_no_keys launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return ATTN_OK;
  }
  int32_t* status = desc->status ? desc->status : g_dev[dev].status;
  return dispatch(*desc, status, static_cast<cudaStream_t>(stream));
}

#define F32_2D(NAME, KIND)                                                                   \
  int32_t NAME(AttnMemRef2D* Q, AttnMemRef2D* K, AttnMemRef2D* V, float scale,               \
               AttnMemRef2D* O) {                                                            \
    if (!Q || !K || !V || !O) return fail(ATTN_ERR_INVALID, "null memref descriptor");        \
    return run_views(ATTN_F32, ATTN_F32, KIND, view2(Q, 4), view2(K, 4), view2(V, 4),         \
                     view2(O, 4), scale, 1.f, 1.f, 1.f, nullptr, nullptr);                    \
  }
F32_2D(_mlir_ciface_attn_fused_f32_nomask, ATTN_MASK_NONE)
F32_2D(_mlir_ciface_attn_fused_f32_causal, ATTN_MASK_CAUSAL)

int32_t _mlir_ciface_attn_fused_f32_mask(AttnMemRef2D* Q, AttnMemRef2D* K, AttnMemRef2D* V,
                                         float scale, AttnMemRef2D* mask, AttnMemRef2D* O) {
  if (!Q || !K || !V || !O || !mask) return fail(ATTN_ERR_INVALID, "null memref descriptor");
  View M = view2(mask, 1);
  return run_views(ATTN_F32, ATTN_F32, ATTN_MASK_DENSE, view2(Q, 4), view2(K, 4), view2(V, 4),
                   view2(O, 4), scale, 1.f, 1.f, 1.f, nullptr, &M);
}

#define F32_4D(NAME, KIND)                                                                   \
  int32_t NAME(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V, float scale,               \
               AttnMemRef4D* O) {                                                            \
    if (!Q || !K || !V || !O) return fail(ATTN_ERR_INVALID, "null memref descriptor");        \
    return run_views(ATTN_F32, ATTN_F32, KIND, view4(Q, 4), view4(K, 4), view4(V, 4),         \
                     view4(O, 4), scale, 1.f, 1.f, 1.f, nullptr, nullptr);                    \
  }
F32_4D(_mlir_ciface_attn_fused_f32_nomask_4d, ATTN_MASK_NONE)
F32_4D(_mlir_ciface_attn_fused_f32_causal_4d, ATTN_MASK_CAUSAL)

#define BF16_4D(NAME, KIND)                                                                  \
  int32_t NAME(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V, float scale,               \
               AttnMemRef4D* O, AttnMemRef4D* LSE) {                                         \
    if (!Q || !K || !V || !O) return fail(ATTN_ERR_INVALID, "null memref descriptor");        \
    View L;                                                                                  \
    if (LSE) L = view4(LSE, 4);                                                              \
    return run_views(ATTN_BF16, ATTN_BF16, KIND, view4(Q, 2), view4(K, 2), view4(V, 2),       \
                     view4(O, 2), scale, 1.f, 1.f, 1.f, LSE ? &L : nullptr, nullptr);         \
  }
BF16_4D(_mlir_ciface_attn_fused_bf16_nomask_4d, ATTN_MASK_NONE)
BF16_4D(_mlir_ciface_attn_fused_bf16_causal_4d, ATTN_MASK_CAUSAL)

#define F16_4D(NAME, KIND)                                                                   \
  int32_t NAME(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V, float scale,               \
               AttnMemRef4D* O, AttnMemRef4D* LSE) {                                         \
    if (!Q || !K || !V || !O) return fail(ATTN_ERR_INVALID, "null memref descriptor");        \
    View L;                                                                                  \
    if (LSE) L = view4(LSE, 4);                                                              \
    return run_views(ATTN_F16, ATTN_F16, KIND, view4(Q, 2), view4(K, 2), view4(V, 2),         \
                     view4(O, 2), scale, 1.f, 1.f, 1.f, LSE ? &L : nullptr, nullptr);         \
  }
F16_4D(_mlir_ciface_attn_fused_f16_nomask_4d, ATTN_MASK_NONE)
F16_4D(_mlir_ciface_attn_fused_f16_causal_4d, ATTN_MASK_CAUSAL)

int32_t _mlir_ciface_attn_fused_bf16_mask_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                             float scale, AttnMemRef4D* mask, AttnMemRef4D* O,
                                             AttnMemRef4D* LSE) {
  if (!Q || !K || !V || !O || !mask) return fail(ATTN_ERR_INVALID, "null memref descriptor");
  View L, M = view4(mask, 1);
  if (LSE) L = view4(LSE, 4);
  return run_views(ATTN_BF16, ATTN_BF16, ATTN_MASK_DENSE, view4(Q, 2), view4(K, 2), view4(V, 2),
                   view4(O, 2), scale, 1.f, 1.f, 1.f, LSE ? &L : nullptr, &M);
}

// The op's own mask form, i1 [seq_q, seq_k] (AttentionOps.td:26-28,40), on
// rank-4 operands: one mask broadcast over every (batch, head) slice.
int32_t _mlir_ciface_attn_fused_bf16_mask2d_4d(AttnMemRef4D* Q, AttnMemRef4D* K,
                                               AttnMemRef4D* V, float scale, AttnMemRef2D* mask,
                                               AttnMemRef4D* O, AttnMemRef4D* LSE) {
  if (!Q || !K || !V || !O || !mask) return fail(ATTN_ERR_INVALID, "null memref descriptor");
  View L, M = view2(mask, 1);  // extents 1 x 1 x seq_q x seq_k: broadcast
  if (LSE) L = view4(LSE, 4);
  return run_views(ATTN_BF16, ATTN_BF16, ATTN_MASK_DENSE, view4(Q, 2), view4(K, 2), view4(V, 2),
                   view4(O, 2), scale, 1.f, 1.f, 1.f, LSE ? &L : nullptr, &M);
}

#define E4M3_4D(NAME, KIND)                                                                  \
  int32_t NAME(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V, float scale, float qd,     \
               float kd, float vd, AttnMemRef4D* O, AttnMemRef4D* LSE) {                     \
    if (!Q || !K || !V || !O) return fail(ATTN_ERR_INVALID, "null memref descriptor");        \
    View L;                                                                                  \
    if (LSE) L = view4(LSE, 4);                                                              \
    return run_views(ATTN_E4M3, ATTN_BF16, KIND, view4(Q, 1), view4(K, 1), view4(V, 1),       \
                     view4(O, 2), scale, qd, kd, vd, LSE ? &L : nullptr, nullptr);            \
  }
E4M3_4D(_mlir_ciface_attn_fused_e4m3_nomask_4d, ATTN_MASK_NONE)
E4M3_4D(_mlir_ciface_attn_fused_e4m3_causal_4d, ATTN_MASK_CAUSAL)

}  // extern "C"

// ======================================================= no-allocation entry
// attn_fwd_host_noalloc: the host-buffer call of the memref entries, for
// callers that must not allocate device memory.  Its device scratch (the
// kernel status word and the staging buffers for Q, K, V, O and LSE) lives
// in the file-scope array below instead of in cudaMalloc'd buffers.
namespace {

constexpr size_t kNoAllocScratchBytes = ATTN_NOALLOC_SCRATCH_BYTES;
constexpr size_t kNoAllocStatusBytes = 256;  // status word, padded to 256 B

// Module-scope device memory: every GPU that loads this library holds these
// bytes until the process exits.  In host code `g_noalloc_scratch` only names
// the symbol; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDev {
  std::mutex mu;
  bool ready = false;            // set once the address below is known
  unsigned char* ptr = nullptr;  // device address of g_noalloc_scratch
};
NoAllocDev g_noalloc[kMaxDevices];

// Once per device, with that device current: check the architecture and
// resolve the array's device address.  Allocates nothing.  Only success is
// remembered: a call that fails here (for instance one made inside a stream
// capture) leaves the device unset, so a later call can try again.
int noalloc_setup(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return fail(ATTN_ERR_INVALID, "bad device %d", device);
  NoAllocDev& nd = g_noalloc[device];
  std::lock_guard<std::mutex> lock(nd.mu);
  if (!nd.ready) {
    int major = 0;
    cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return cuda_fail(e, "attn_fwd_host_noalloc set-up: cudaDeviceGetAttribute");
    }
    if (major != 10)
      return fail(ATTN_ERR_NO_DEVICE, "device %d is not sm_100; attn_fwd_host_noalloc needs one",
                  device);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return cuda_fail(e, "attn_fwd_host_noalloc set-up: cudaGetSymbolAddress");
    }
    nd.ptr = static_cast<unsigned char*>(p);
    nd.ready = true;
  }
  *out = nd.ptr;
  return ATTN_OK;
}

size_t round256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace

extern "C" int attn_fwd_host_noalloc(const AttnDesc* desc, void* stream_) {
  NvtxRange range("attn_fwd_host_noalloc");
  if (!desc) return fail(ATTN_ERR_INVALID, "null descriptor");
  const AttnDesc& hd = *desc;
  if (hd.mask_kind == ATTN_MASK_DENSE)
    return fail(ATTN_ERR_UNSUPPORTED, "attn_fwd_host_noalloc supports no-mask and causal calls");
  if (hd.q_descale_blocks || hd.k_descale_blocks || hd.v_descale_heads)
    return fail(ATTN_ERR_UNSUPPORTED, "attn_fwd_host_noalloc takes per-tensor descales only");
  // Host buffers only: a device pointer here would be handed to host-to-
  // device copies (or, without keys, written from the host).
  const void* host_bufs[] = {hd.q, hd.k, hd.v, hd.o, hd.lse};
  for (const void* ptr : host_bufs)
    if (ptr && is_device_ptr(ptr))
      return fail(ATTN_ERR_INVALID,
                  "attn_fwd_host_noalloc takes host buffers; pass device-resident operands "
                  "to attn_fwd");
  bool no_rows = false, no_keys = false;
  int rc = check_empty(hd, &no_rows, &no_keys);
  if (rc != ATTN_OK) return rc;
  if (no_rows) return ATTN_OK;
  if (no_keys) {
    fill_no_keys_host(hd);
    return ATTN_OK;
  }
  // Shape, type and scale rules only: every chunk is re-packed into dense,
  // 256-byte aligned staging regions (validated again below), so the host
  // buffers' own alignment and strides place no constraint on the kernel.
  if (!hd.q || !hd.k || !hd.v || !hd.o)
    return fail(ATTN_ERR_INVALID, "null Q/K/V/output pointer");
  {
    AttnDesc chk = hd;
    alignas(256) static unsigned char aligned_dummy[256];
    chk.q = chk.k = chk.v = chk.o = aligned_dummy;
    chk.o_stride[2] = hd.D;
    chk.o_stride[1] = hd.Nq * hd.D;
    chk.o_stride[0] = hd.Hq * hd.Nq * hd.D;
    if ((rc = validate(chk)) != ATTN_OK) return rc;
  }
  int dev = 0;
  if ((rc = current_device(&dev)) != ATTN_OK) return rc;
  unsigned char* base = nullptr;
  if ((rc = noalloc_setup(dev, &base)) != ATTN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream_);

  // Scratch needed per (batch, kv-head) group: the group's q-heads of Q, O
  // and LSE, and its one kv-head of K and V, each region 256-byte aligned.
  const size_t eb = elem_bytes(hd.dtype), ob = elem_bytes(hd.out_dtype);
  const int64_t group = hd.Hq / hd.Hkv;
  const int64_t ngroups = hd.B * hd.Hkv;
  const size_t q_slice = static_cast<size_t>(hd.Nq * hd.D) * eb;
  const size_t kv_slice = static_cast<size_t>(hd.Nk * hd.D) * eb;
  const size_t o_slice = static_cast<size_t>(hd.Nq * hd.D) * ob;
  const size_t l_slice = hd.lse ? sizeof(float) * static_cast<size_t>(hd.Nq) : 0;
  const size_t per_group =
      round256(group * q_slice) + 2 * round256(kv_slice) + round256(group * o_slice) +
      round256(group * l_slice);
  const size_t room = kNoAllocScratchBytes - kNoAllocStatusBytes;
  if (per_group > room)
    return fail(ATTN_ERR_SHAPE,
                "attn_fwd_host_noalloc: one (batch, kv-head) group needs %zu bytes of device "
                "scratch but the static scratch holds %zu bytes (ATTN_NOALLOC_SCRATCH_BYTES "
                "minus %zu for the status word); use the memref entries instead",
                per_group, room, kNoAllocStatusBytes);
  const int64_t per_chunk = std::min<int64_t>(ngroups, static_cast<int64_t>(room / per_group));

  int32_t* status = reinterpret_cast<int32_t*>(base);
  // Once anything is enqueued, copies from and into the caller's buffers may
  // be in flight: every error return after that point first waits for the
  // stream, so the caller may free or reuse its buffers as soon as the call
  // returns.
#define NOALLOC_TRY(call)                            \
  do {                                               \
    cudaError_t e_ = (call);                         \
    if (e_ != cudaSuccess) {                         \
      const int c_ = cuda_fail(e_, #call);           \
      cudaStreamSynchronize(s);                      \
      return c_;                                     \
    }                                                \
  } while (0)
  auto bail = [&](int code) {
    cudaStreamSynchronize(s);
    return code;
  };
  // The array keeps the previous call's contents: the status word must start
  // at zero.  (Staging regions are fully overwritten before they are read.)
  NOALLOC_TRY(cudaMemsetAsync(status, 0, sizeof(int32_t), s));
  unsigned char* dq = base + kNoAllocStatusBytes;
  unsigned char* dk = dq + round256(per_chunk * group * q_slice);
  unsigned char* dv = dk + round256(per_chunk * kv_slice);
  unsigned char* dout = dv + round256(per_chunk * kv_slice);
  float* dl = reinterpret_cast<float*>(dout + round256(per_chunk * group * o_slice));

  for (int64_t g0 = 0; g0 < ngroups; g0 += per_chunk) {
    const int64_t gn = std::min<int64_t>(per_chunk, ngroups - g0);
    for (int64_t g = 0; g < gn; ++g) {
      const int64_t b = (g0 + g) / hd.Hkv, hk = (g0 + g) % hd.Hkv;
      const char* ks = static_cast<const char*>(hd.k) + (b * hd.k_stride[0] + hk * hd.k_stride[1]) * eb;
      const char* vs = static_cast<const char*>(hd.v) + (b * hd.v_stride[0] + hk * hd.v_stride[1]) * eb;
      NOALLOC_TRY(cudaMemcpy2DAsync(dk + g * kv_slice, hd.D * eb, ks, hd.k_stride[2] * eb,
                                 hd.D * eb, hd.Nk, cudaMemcpyHostToDevice, s));
      NOALLOC_TRY(cudaMemcpy2DAsync(dv + g * kv_slice, hd.D * eb, vs, hd.v_stride[2] * eb,
                                 hd.D * eb, hd.Nk, cudaMemcpyHostToDevice, s));
      for (int64_t i = 0; i < group; ++i) {
        const int64_t h = hk * group + i;
        const char* qs = static_cast<const char*>(hd.q) + (b * hd.q_stride[0] + h * hd.q_stride[1]) * eb;
        NOALLOC_TRY(cudaMemcpy2DAsync(dq + (g * group + i) * q_slice, hd.D * eb, qs,
                                   hd.q_stride[2] * eb, hd.D * eb, hd.Nq,
                                   cudaMemcpyHostToDevice, s));
      }
    }
    AttnDesc dd = hd;
    dd.B = gn;
    dd.Hq = group;
    dd.Hkv = 1;
    dd.q = dq; dd.k = dk; dd.v = dv; dd.o = dout;
    dd.lse = hd.lse ? dl : nullptr;
    dd.q_stride[2] = hd.D; dd.q_stride[1] = hd.Nq * hd.D; dd.q_stride[0] = group * hd.Nq * hd.D;
    dd.o_stride[2] = hd.D; dd.o_stride[1] = hd.Nq * hd.D; dd.o_stride[0] = group * hd.Nq * hd.D;
    dd.k_stride[2] = hd.D; dd.k_stride[1] = hd.Nk * hd.D; dd.k_stride[0] = hd.Nk * hd.D;
    dd.v_stride[2] = hd.D; dd.v_stride[1] = hd.Nk * hd.D; dd.v_stride[0] = hd.Nk * hd.D;
    dd.status = status;
    if ((rc = validate(dd)) != ATTN_OK) return bail(rc);
    if ((rc = dispatch(dd, status, s, /*may_split=*/false)) != ATTN_OK) return bail(rc);
    for (int64_t g = 0; g < gn; ++g) {
      const int64_t b = (g0 + g) / hd.Hkv, hk = (g0 + g) % hd.Hkv;
      for (int64_t i = 0; i < group; ++i) {
        const int64_t h = hk * group + i;
        char* os = static_cast<char*>(hd.o) + (b * hd.o_stride[0] + h * hd.o_stride[1]) * ob;
        NOALLOC_TRY(cudaMemcpy2DAsync(os, hd.o_stride[2] * ob, dout + (g * group + i) * o_slice,
                                   hd.D * ob, hd.D * ob, hd.Nq, cudaMemcpyDeviceToHost, s));
        if (hd.lse)
          NOALLOC_TRY(cudaMemcpyAsync(hd.lse + (b * hd.Hq + h) * hd.Nq, dl + (g * group + i) * hd.Nq,
                                   sizeof(float) * hd.Nq, cudaMemcpyDeviceToHost, s));
      }
    }
  }
  int32_t code = 0;
  NOALLOC_TRY(cudaMemcpyAsync(&code, status, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  NOALLOC_TRY(cudaStreamSynchronize(s));
#undef NOALLOC_TRY
  if (code != 0) return fail(code, "kernel reported %s", attn_rt_status_string(code));
  return ATTN_OK;
}
