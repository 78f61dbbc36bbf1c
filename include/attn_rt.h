/*
 * attn_rt.h — C ABI of the B200 (sm_100a) runtime behind the `attention.fused` op.
 *
 * The reference project (luisroayerdi/MLIR-FlashAttention) defines one op,
 *   attention.fused ins(%Q, %K, %V) scale(%s) [mask(%m)] outs(%O)
 * (include/Attention/AttentionOps.td:20-54) and lowers it to a CPU loop nest
 * (lib/Attention/TilingPass.cpp:155-392).  This library replaces that lowering:
 * a pass rewrites the op into calls to the `_mlir_ciface_attn_fused_*` symbols
 * below (MLIR's memref-descriptor C interface, the calling convention shown in
 * the reference at examples/MatMUL/main.c:4-7,38-41), and every call ends in
 * `attn_fwd`, which launches the hand-written sm_100a kernels.
 *
 * Semantics of one (batch, head) slice, identical to the reference op:
 *   O = softmax(Q·Kᵀ·scale, masked entries -> -inf) · V
 * The reference op is rank-2 f32 only; this ABI adds rank-4 [B,H,N,D] views,
 * bf16, f16 and fp8-e4m3 inputs (fp32 accumulation), grouped-query heads (Hq a
 * multiple of Hkv), and an optional log-sum-exp output.
 *
 * Ownership and threading.  The caller owns every buffer; O (and LSE) are
 * written in place, as the op's memory effects declare (AttentionOps.cpp:15-30).
 * The runtime keeps only a per-device status word and, for host memrefs,
 * per-device staging buffers, both created on first use behind a mutex.
 * Calls on different streams may run concurrently.
 *
 * Errors.  Every entry point returns 0 on success or a negative ATTN_ERR_* code
 * and never aborts.  `attn_rt_last_error()` returns the message of the last
 * failure on the calling thread; shape errors reuse the reference verifier's
 * wording (AttentionOps.cpp:39-56).
 */
#ifndef ATTN_RT_H
#define ATTN_RT_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ATTN_API __attribute__((visibility("default")))
#else
#define ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define ATTN_OK                 0
#define ATTN_ERR_INVALID       -1  /* null descriptor or pointer                   */
#define ATTN_ERR_SHAPE         -2  /* shapes inconsistent (verifier rules)         */
#define ATTN_ERR_STRIDE        -3  /* head_dim not unit-stride or strides unusable */
#define ATTN_ERR_DTYPE         -4  /* unsupported element type combination         */
#define ATTN_ERR_ALIGN         -5  /* pointer/stride not 16-byte aligned           */
#define ATTN_ERR_CUDA          -6  /* a CUDA runtime/driver call failed            */
#define ATTN_ERR_TIMEOUT       -7  /* a bounded on-device wait expired             */
#define ATTN_ERR_UNSUPPORTED   -8  /* valid op, variant not built (e.g. head_dim)  */
#define ATTN_ERR_NO_DEVICE     -9  /* no sm_100 device visible                     */

/* ---- element types and mask kinds --------------------------------------- */
#define ATTN_F32   0
#define ATTN_BF16  1
#define ATTN_E4M3  2
#define ATTN_F16   3

#define ATTN_MASK_NONE    0  /* no mask operand                                   */
#define ATTN_MASK_CAUSAL  1  /* mask[i][j] = (j > i): the causal generic           */
#define ATTN_MASK_DENSE   2  /* explicit i1 mask, one byte per element, 1 = masked */

/*
 * One attention call over B x Hq independent (batch, head) slices.
 * Strides are in ELEMENTS for q/k/v/o ([0]=batch, [1]=head, [2]=row; the
 * head_dim stride must be 1) and in BYTES for the dense mask.
 * All data pointers are device pointers.
 */
typedef struct AttnDesc {
  int32_t dtype;        /* ATTN_F32 / ATTN_BF16 / ATTN_F16 / ATTN_E4M3: Q, K, V  */
  int32_t out_dtype;    /* ATTN_F32, ATTN_BF16 or ATTN_F16: type of O           */
  int32_t mask_kind;    /* ATTN_MASK_*                                          */
  int32_t flags;        /* reserved, must be 0                                  */
  int64_t B, Hq, Hkv, Nq, Nk, D;
  int64_t q_stride[3], k_stride[3], v_stride[3], o_stride[3];
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;                /* optional [B,Hq,Nq] fp32 contiguous, natural log  */
  const uint8_t* mask;       /* ATTN_MASK_DENSE only                             */
  int64_t mask_stride[3];    /* bytes: batch, head, row; column stride is 1      */
  float scale;               /* multiplies Q·Kᵀ (the op's `scale` operand)        */
  float q_descale;           /* e4m3 only: dequantisation factors; else 1        */
  float k_descale;
  float v_descale;
  int32_t* status;           /* optional device word for kernel status; if null
                                the runtime's per-device word is used            */
  /* e4m3 only, optional (NULL = not used): per-block dequantisation factors,
   * fp32 device arrays, contiguous, positive and finite, applied on top of the
   * per-tensor factors above.  One block = 128 rows, the tile of the
   * reference's TilingPass (AttentionPasses.td:46):
   *   q_descale_blocks [B, Hq,  ceil(Nq / 128)]  Q rows [128 i, 128 i + 128)
   *   k_descale_blocks [B, Hkv, ceil(Nk / 128)]  K rows [128 j, 128 j + 128)
   *   v_descale_heads  [B, Hkv]                  all of V for one kv head
   * Score (r, c) = scale * qd * kd * q_descale_blocks[b,h,r/128] *
   * k_descale_blocks[b,h/(Hq/Hkv),c/128] * (Q8[r] . K8[c]); O is multiplied
   * by vd * v_descale_heads[b,h/(Hq/Hkv)].  Device path (attn_fwd) only. */
  const float* q_descale_blocks;
  const float* k_descale_blocks;
  const float* v_descale_heads;
} AttnDesc;

/* Asynchronous launch on `stream` (a cudaStream_t; NULL = legacy default).
 * Replaces the loop nest TilingPass.cpp:188-386 emits for one attention.fused.
 * Empty extents behave as that loop nest does: B, Hq or Nq = 0 computes
 * nothing (ATTN_OK); Nk = 0 runs no KV step, so every row of O is 0/0 = NaN
 * and the LSE is -inf.  The first causal call of a shape with few work items
 * per SM plans a balanced work order and keeps it in device memory (one
 * cudaMalloc and a synchronous copy per device and shape, at most 64 shapes):
 * make that first call outside stream capture. */
ATTN_API int attn_fwd(const AttnDesc* desc, void* stream);

/* Select and initialise `device` (idempotent): checks for sm_100, creates the
 * per-device status word.  Called implicitly by attn_fwd. */
ATTN_API int attn_rt_init(int device);

/* Schedule of causal tensor-core calls (no counterpart in the reference).
 * A causal launch with few Q-tile pairs per SM is bounded by its heaviest
 * pairs; the runtime then runs the S heaviest pair indices of every slice as
 * two work items over the first and second half of their KV tiles and merges
 * the halves in the kernel (stream-ordered scratch: 128 x (D + 1) floats per
 * Q tile and half).  Returns the S a causal call with `slices` (batch x
 * q-head) slices of Nq x Nk would use on a device with `sm_count` SMs
 * (0: no split).  attn_fwd_host_noalloc never splits. */
ATTN_API int attn_rt_causal_split(int64_t slices, int64_t Nq, int64_t Nk, int sm_count);

/* Synchronise `stream`, read and clear the device status word written by the
 * kernels of `device`; returns ATTN_OK or the first recorded ATTN_ERR_*. */
ATTN_API int attn_rt_check_status(int device, void* stream);

/* Failure-detection self-test (no counterpart in the reference): launches one
 * CTA that waits, with the bounded mbarrier wait every kernel here uses, on a
 * barrier nothing arrives on, giving up after `limit_ns` (<= 2 s).  Returns
 * ATTN_ERR_TIMEOUT when the bound works; the device stays usable. */
ATTN_API int attn_rt_probe_timeout(int64_t limit_ns);

/* Human-readable name of a status code. */
ATTN_API const char* attn_rt_status_string(int code);

/* Message of the last failure on the calling thread ("" if none). */
ATTN_API const char* attn_rt_last_error(void);

/* ABI version, (major << 16) | minor. */
ATTN_API int attn_rt_version(void);

/* Number of kernel launches attn_fwd issued in this process (all devices). */
ATTN_API int64_t attn_rt_launch_count(void);

/* Device memory helpers for callers that keep operands resident across calls
 * (a lowered program that copies its memrefs to the GPU once and passes
 * device memrefs to the entries below, instead of host memrefs that are
 * staged on every call).  The allocation is on the current device, 256-byte
 * aligned; `bytes` must be positive.  attn_rt_copy copies `bytes` between any
 * two host or device addresses: asynchronously on `stream` when it is
 * non-null, else synchronously. */
ATTN_API int attn_rt_alloc(void** ptr, size_t bytes);
ATTN_API int attn_rt_free(void* ptr);
ATTN_API int attn_rt_copy(void* dst, const void* src, size_t bytes, void* stream);

/* ---- MLIR memref-descriptor interface ------------------------------------
 * MLIR passes a memref<...> to an `llvm.emit_c_interface` function as a pointer
 * to {allocated, aligned, offset, sizes[R], strides[R]} (strides in elements).
 * The element type is fixed by the symbol name.  The buffers may be host or
 * device memory: host buffers are staged through device memory in chunks of
 * slices with copies overlapped with compute, and the call returns after O is
 * back in host memory.  These calls are synchronous.
 * Symbol naming: attn_fused_<dtype>_<variant>[_4d], variant in
 * {nomask, causal, mask}; the lowering pass picks it from the mask operand.  */
typedef struct AttnMemRef2D {
  void* allocated;
  void* aligned;
  int64_t offset;
  int64_t sizes[2];
  int64_t strides[2];
} AttnMemRef2D;

typedef struct AttnMemRef4D {
  void* allocated;
  void* aligned;
  int64_t offset;
  int64_t sizes[4];
  int64_t strides[4];
} AttnMemRef4D;

/* Rank-2 f32, the reference op's own form (AttentionOps.td:36-41). */
ATTN_API int32_t _mlir_ciface_attn_fused_f32_nomask(AttnMemRef2D* Q, AttnMemRef2D* K, AttnMemRef2D* V,
                                           float scale, AttnMemRef2D* O);
ATTN_API int32_t _mlir_ciface_attn_fused_f32_causal(AttnMemRef2D* Q, AttnMemRef2D* K, AttnMemRef2D* V,
                                           float scale, AttnMemRef2D* O);
ATTN_API int32_t _mlir_ciface_attn_fused_f32_mask(AttnMemRef2D* Q, AttnMemRef2D* K, AttnMemRef2D* V,
                                         float scale, AttnMemRef2D* mask, AttnMemRef2D* O);

/* Rank-4 [B,H,N,D] f32 in / f32 out. */
ATTN_API int32_t _mlir_ciface_attn_fused_f32_nomask_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                              float scale, AttnMemRef4D* O);
ATTN_API int32_t _mlir_ciface_attn_fused_f32_causal_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                              float scale, AttnMemRef4D* O);

/* Rank-4 bf16 in / bf16 out.  LSE is NULL, a zero-sized memref (not
 * requested; what the lowering pass passes), or memref<BxHxNqx1xf32>. */
ATTN_API int32_t _mlir_ciface_attn_fused_bf16_nomask_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                               float scale, AttnMemRef4D* O, AttnMemRef4D* LSE);
ATTN_API int32_t _mlir_ciface_attn_fused_bf16_causal_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                               float scale, AttnMemRef4D* O, AttnMemRef4D* LSE);

/* Rank-4 f16 in / f16 out (same kernels, f16 operand format). */
ATTN_API int32_t _mlir_ciface_attn_fused_f16_nomask_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                                       float scale, AttnMemRef4D* O, AttnMemRef4D* LSE);
ATTN_API int32_t _mlir_ciface_attn_fused_f16_causal_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                                       float scale, AttnMemRef4D* O, AttnMemRef4D* LSE);

/* Rank-4 bf16 with a general i1 mask memref<BxHxNqxNkxi1> (one byte per
 * element, 1 = masked; batch/head strides may be 0 to broadcast one mask);
 * the reference op's `mask` operand (AttentionOps.td:40, TilingPass.cpp:254-277)
 * on the tensor-core path. */
ATTN_API int32_t _mlir_ciface_attn_fused_bf16_mask_4d(AttnMemRef4D* Q, AttnMemRef4D* K,
                                                      AttnMemRef4D* V, float scale,
                                                      AttnMemRef4D* mask, AttnMemRef4D* O,
                                                      AttnMemRef4D* LSE);

/* Rank-4 bf16 operands with the op's own rank-2 i1 mask memref<NqxNkxi1>
 * (AttentionOps.td:26-28,40), applied to every (batch, head) slice.  The
 * lowering pass calls this entry when a rank-2 mask meets rank-4 operands. */
ATTN_API int32_t _mlir_ciface_attn_fused_bf16_mask2d_4d(AttnMemRef4D* Q, AttnMemRef4D* K,
                                                        AttnMemRef4D* V, float scale,
                                                        AttnMemRef2D* mask, AttnMemRef4D* O,
                                                        AttnMemRef4D* LSE);

/* Rank-4 e4m3 in (per-tensor dequantisation factors) / bf16 out. */
ATTN_API int32_t _mlir_ciface_attn_fused_e4m3_nomask_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                               float scale, float q_descale, float k_descale,
                                               float v_descale, AttnMemRef4D* O, AttnMemRef4D* LSE);
ATTN_API int32_t _mlir_ciface_attn_fused_e4m3_causal_4d(AttnMemRef4D* Q, AttnMemRef4D* K, AttnMemRef4D* V,
                                               float scale, float q_descale, float k_descale,
                                               float v_descale, AttnMemRef4D* O, AttnMemRef4D* LSE);

/* ---- entry point that allocates no device memory -------------------------
 * No counterpart in the reference.
 *
 * Same operation as the memref entries above on HOST buffers (desc->q, k, v,
 * o and lse are host pointers; dtype f32, bf16 or e4m3; mask kind none or
 * causal), but without any device allocation.  It is meant for callers that
 * cannot call cudaMalloc: e.g. a host program (such as MLIR-lowered CPU code
 * operating on host memrefs) running in a process whose device memory is
 * already reserved by another allocator (a serving engine or framework
 * caching allocator that holds nearly all HBM), or one that must not take the
 * implicit device synchronisation cudaMalloc/cudaFree may cause.
 *
 * Its device scratch — the kernel status word and the staging buffers for
 * Q, K, V, O and LSE — is one file-scope __device__ array of
 * ATTN_NOALLOC_SCRATCH_BYTES, which every GPU that loads the library holds
 * until the process exits.  Work is staged through it in chunks of whole
 * (batch, kv-head) groups; a call whose single group needs more than
 * ATTN_NOALLOC_SCRATCH_BYTES - 256 bytes is rejected with ATTN_ERR_SHAPE and
 * a message giving both sizes.
 *
 * Host buffers may have any alignment and row strides (each chunk is
 * re-packed into aligned staging regions); device pointers are refused with
 * ATTN_ERR_INVALID (device-resident operands go to attn_fwd).
 *
 * The first call on each device resolves the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  A set-up that fails is not remembered, so a
 * later call retries it.  Copies and kernels run on `stream` and the call
 * returns after O (and LSE) are back in host memory; an error after the
 * first copy was enqueued also waits for `stream` before returning, so the
 * caller may reuse its buffers whatever the outcome.  All calls share the one
 * array, which keeps the previous call's contents (the status word is
 * cleared at the start of each call): calls that overlap on the GPU — from
 * several threads or streams of one process — race and must be serialised by
 * the caller.  Calls no cudaMalloc, cudaFree or allocating library routine. */
#define ATTN_NOALLOC_SCRATCH_BYTES (64u << 20)
ATTN_API int attn_fwd_host_noalloc(const AttnDesc* desc, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ATTN_RT_H */
