//===- RuntimeLoweringPass.cpp - attention.fused -> B200 runtime calls ---===//
//
// Pass `--attention-to-runtime` for the reference's Attention dialect
// (luisroayerdi/MLIR-FlashAttention).  It runs after `--fusion-pass`
// (lib/Attention/FusionPass.cpp) in place of `--tiling-pass`
// (lib/Attention/TilingPass.cpp) and rewrites every
//
//   attention.fused ins(%Q, %K, %V) scale(%s) [mask(%m)] outs(%O)
//
// (include/Attention/AttentionOps.td:20-54) into
//
//   %rc = func.call @attn_fused_<dtype>_<variant>[_4d](%Q, %K, %V, %s, [%m,] %O)
//   %ok = arith.cmpi eq, %rc, %c0_i32 : i32
//   cf.assert %ok, "attention.fused: runtime call failed ..."
//
// where the callee is declared `func.func private ... attributes
// {llvm.emit_c_interface}` so that, after the standard lowering to LLVM, the
// call lands on `_mlir_ciface_attn_fused_*` in libattnrt.so (include/attn_rt.h).
// The runtime launches the sm_100a kernels; the op's semantics (in-place write
// of %O, AttentionOps.cpp:15-30) are unchanged.  The runtime reports failures
// (shape, alignment, CUDA errors, a device timeout) as a negative i32 rather
// than aborting; the reference op has no error result, so the lowered program
// checks the code with cf.assert and stops with a message instead of
// continuing with a stale %O.
//
// Mask classification (the reference's mask-specialisation design,
// Design.md:402-444, which its code does not implement):
//   * no mask operand                                   -> "nomask"
//   * mask written by a linalg.fill of `false`           -> "nomask"
//   * mask written by a linalg.generic with no inputs whose body yields
//     `arith.cmpi ugt|sgt (index 1), (index 0)` or `ult|slt (index 0), (index 1)`
//     (the causal generic), or a mask value carrying the unit attribute
//     `attention.causal` on its defining op                -> "causal"
//   * anything else                                      -> "mask" (dense i1
//     operand; rank-2 f32 or rank-4 bf16, others rejected with an error).
//     On rank-4 bf16 operands the op's own [seq_q, seq_k] mask (rank 2,
//     AttentionOps.td:26-28,40) calls "mask2d" (one mask for every slice);
//     a rank-4 mask calls "mask".
//
// Shapes: every memref operand is passed through `memref.cast` to the fully
// dynamic strided type of its rank (memref<?x?xT, strided<[?, ?], offset: ?>>),
// so one declaration per callee serves every static or dynamic shape and
// layout in the module; the runtime reads sizes and strides from the
// descriptor.  (TilingPass.cpp:168-172 accepts static shapes only.)
//
// The pass is stateless.  Unlike the reference's FuncOp-anchored passes
// (AttentionPasses.td:14,27) it is anchored on the module, because it adds
// the private runtime declarations at module scope, which a pass running
// concurrently on sibling functions may not do.  Failures are reported with
// emitOpError + signalPassFailure like TilingPass.cpp:170-172,406-407.
//
// Build: only where find_package(MLIR) succeeds; see CMakeLists.txt here.
//===----------------------------------------------------------------------===//

#include "Attention/AttentionOps.h"
#include "Attention/AttentionPasses.h"
#include "mlir/Dialect/Arith/IR/Arith.h"
#include "mlir/Dialect/ControlFlow/IR/ControlFlowOps.h"
#include "mlir/Dialect/Func/IR/FuncOps.h"
#include "mlir/Dialect/Linalg/IR/Linalg.h"
#include "mlir/Dialect/MemRef/IR/MemRef.h"
#include "mlir/IR/BuiltinOps.h"
#include "mlir/IR/BuiltinTypes.h"
#include "mlir/IR/PatternMatch.h"
#include "mlir/IR/SymbolTable.h"
#include "mlir/Transforms/GreedyPatternRewriteDriver.h"

namespace mlir::attention {
#define GEN_PASS_DEF_ATTENTIONTORUNTIMEPASS
#include "Attention/AttentionPasses.h.inc"

namespace {

enum class MaskKind { None, Causal, Dense };

// True if `v` is `linalg.index <dim>` inside the generic body.
static bool isIndex(Value v, int64_t dim) {
  auto idx = v.getDefiningOp<linalg::IndexOp>();
  return idx && static_cast<int64_t>(idx.getDim()) == dim;
}

// The causal generic: no inputs, one i1 output, body yields j > i.
static bool isCausalGeneric(linalg::GenericOp g) {
  if (!g.getDpsInputs().empty() || g.getDpsInits().size() != 1) return false;
  auto yield = cast<linalg::YieldOp>(g.getBody()->getTerminator());
  if (yield.getNumOperands() != 1) return false;
  auto cmp = yield.getOperand(0).getDefiningOp<arith::CmpIOp>();
  if (!cmp) return false;
  Value a = cmp.getLhs(), b = cmp.getRhs();
  switch (cmp.getPredicate()) {
    case arith::CmpIPredicate::ugt:
    case arith::CmpIPredicate::sgt:
      return isIndex(a, 1) && isIndex(b, 0);
    case arith::CmpIPredicate::ult:
    case arith::CmpIPredicate::slt:
      return isIndex(a, 0) && isIndex(b, 1);
    default:
      return false;
  }
}

static bool isFalseFill(linalg::FillOp f) {
  auto c = f.getInputs()[0].getDefiningOp<arith::ConstantOp>();
  if (!c) return false;
  auto b = dyn_cast<BoolAttr>(c.getValue());
  if (b) return !b.getValue();
  auto i = dyn_cast<IntegerAttr>(c.getValue());
  return i && i.getValue().isZero();
}

static MaskKind classifyMask(Value mask) {
  if (!mask) return MaskKind::None;
  if (Operation* def = mask.getDefiningOp())
    if (def->hasAttr("attention.causal")) return MaskKind::Causal;
  // Find the unique writer of the mask buffer (DPS init), as FusionPass does
  // for its operands (FusionPass.cpp:40-71).
  Operation* writer = nullptr;
  for (Operation* user : mask.getUsers()) {
    auto dps = dyn_cast<DestinationStyleOpInterface>(user);
    if (!dps) continue;
    for (Value init : dps.getDpsInits())
      if (init == mask) {
        if (writer) return MaskKind::Dense;  // several writers: keep it general
        writer = user;
      }
  }
  if (!writer) return MaskKind::Dense;
  if (auto fill = dyn_cast<linalg::FillOp>(writer))
    return isFalseFill(fill) ? MaskKind::None : MaskKind::Dense;
  if (auto gen = dyn_cast<linalg::GenericOp>(writer))
    return isCausalGeneric(gen) ? MaskKind::Causal : MaskKind::Dense;
  return MaskKind::Dense;
}

static StringRef dtypeName(Type t) {
  if (t.isF32()) return "f32";
  if (t.isBF16()) return "bf16";
  if (t.isF16()) return "f16";
  if (isa<Float8E4M3FNType>(t)) return "e4m3";
  return "";
}

// The fully dynamic strided memref type of `t`'s rank and element type.
static MemRefType dynamicStridedType(MemRefType t) {
  const int64_t r = t.getRank();
  SmallVector<int64_t> shape(r, ShapedType::kDynamic), strides(r, ShapedType::kDynamic);
  auto layout = StridedLayoutAttr::get(t.getContext(), ShapedType::kDynamic, strides);
  return MemRefType::get(shape, t.getElementType(), layout, t.getMemorySpace());
}

struct FusedToRuntimeCall : public OpRewritePattern<FusedOp> {
  using OpRewritePattern::OpRewritePattern;

  LogicalResult matchAndRewrite(FusedOp op, PatternRewriter& rewriter) const override {
    auto qT = cast<MemRefType>(op.getQ().getType());
    StringRef dt = dtypeName(qT.getElementType());
    if (dt.empty()) return op.emitOpError("element type has no runtime kernel");
    const int64_t rank = qT.getRank();
    if (rank != 2 && rank != 4) return op.emitOpError("operands must be rank-2 or rank-4");

    MaskKind kind = classifyMask(op.getMask());
    if (kind == MaskKind::Dense && !((dt == "f32" && rank == 2) || (dt == "bf16" && rank == 4)))
      return op.emitOpError("a general i1 mask is supported for rank-2 f32 and rank-4 bf16 "
                            "operands");
    // A dense mask is the op's [seq_q, seq_k] (rank 2) or, on rank-4
    // operands, a per-slice [B, H, seq_q, seq_k]; each rank has its own entry
    // so the runtime reads a descriptor of the rank it was given.
    const int64_t maskRank =
        op.getMask() ? cast<MemRefType>(op.getMask().getType()).getRank() : 0;
    if (kind == MaskKind::Dense && maskRank != 2 && maskRank != rank)
      return op.emitOpError("mask must be rank 2 [seq_q, seq_k] or of the operands' rank");
    if (dt != "f32" && rank != 4)
      return op.emitOpError("bf16/f16/e4m3 operands are lowered in their rank-4 form");

    std::string callee = ("attn_fused_" + dt + "_").str();
    callee += kind == MaskKind::None     ? "nomask"
              : kind == MaskKind::Causal ? "causal"
              : (rank == 4 && maskRank == 2) ? "mask2d"
                                             : "mask";
    if (rank == 4) callee += "_4d";

    auto module = op->getParentOfType<ModuleOp>();
    if (!module) return op.emitOpError("must be nested in a module");

    // Signature first (no IR is created before every check has passed).
    auto f32 = rewriter.getF32Type();
    auto lseT = MemRefType::get({0, 0, 0, 1}, f32);  // zero-sized: LSE not requested
    SmallVector<Value> memrefs = {op.getQ(), op.getK(), op.getV()};
    if (kind == MaskKind::Dense) memrefs.push_back(op.getMask());
    memrefs.push_back(op.getOutput());
    SmallVector<Type> dynTypes;
    for (Value v : memrefs) {
      auto t = cast<MemRefType>(v.getType());
      auto d = dynamicStridedType(t);
      if (!memref::CastOp::areCastCompatible(t, d))
        return op.emitOpError("operand layout is not strided: ") << t;
      dynTypes.push_back(d);
    }
    auto lseDyn = dynamicStridedType(lseT);
    SmallVector<Type> argTypes = {dynTypes[0], dynTypes[1], dynTypes[2], f32};
    if (dt == "e4m3") argTypes.append({f32, f32, f32});
    argTypes.append(dynTypes.begin() + 3, dynTypes.end());
    if (dt != "f32") argTypes.push_back(lseDyn);
    auto fnType = rewriter.getFunctionType(argTypes, {rewriter.getI32Type()});
    auto fn = module.lookupSymbol<func::FuncOp>(callee);
    if (fn && fn.getFunctionType() != fnType)
      return op.emitOpError("runtime symbol ") << callee << " already declared with another type";
    if (!fn) {
      OpBuilder::InsertionGuard g(rewriter);
      rewriter.setInsertionPointToStart(module.getBody());
      fn = rewriter.create<func::FuncOp>(op.getLoc(), callee, fnType);
      fn.setPrivate();
      fn->setAttr("llvm.emit_c_interface", rewriter.getUnitAttr());
    }

    rewriter.setInsertionPoint(op);
    auto toDyn = [&](Value v, Type d) -> Value {
      if (v.getType() == d) return v;
      return rewriter.create<memref::CastOp>(op.getLoc(), d, v);
    };
    SmallVector<Value> args = {toDyn(op.getQ(), dynTypes[0]), toDyn(op.getK(), dynTypes[1]),
                               toDyn(op.getV(), dynTypes[2]), op.getScale()};
    if (dt == "e4m3") {
      // Per-tensor dequantisation factors ride on the op as optional f32
      // attributes (its attr-dict, AttentionOps.td:50); absent means 1.0.
      for (StringRef name : {"q_descale", "k_descale", "v_descale"}) {
        double val = 1.0;
        if (auto a = op->getAttrOfType<FloatAttr>(name)) val = a.getValueAsDouble();
        args.push_back(rewriter.create<arith::ConstantOp>(
            op.getLoc(), rewriter.getF32FloatAttr(static_cast<float>(val))));
      }
    }
    for (size_t i = 3; i < memrefs.size(); ++i) args.push_back(toDyn(memrefs[i], dynTypes[i]));
    if (dt != "f32")
      args.push_back(toDyn(rewriter.create<memref::AllocaOp>(op.getLoc(), lseT), lseDyn));
    auto call = rewriter.create<func::CallOp>(op.getLoc(), fn, args);
    Value zero = rewriter.create<arith::ConstantIntOp>(op.getLoc(), 0, 32);
    Value ok = rewriter.create<arith::CmpIOp>(op.getLoc(), arith::CmpIPredicate::eq,
                                              call.getResult(0), zero);
    rewriter.create<cf::AssertOp>(
        op.getLoc(), ok,
        ("attention.fused: runtime call " + callee +
         " failed (negative ATTN_ERR_* code; attn_rt_last_error() has the message)"));
    rewriter.eraseOp(op);
    return success();
  }
};

struct AttentionToRuntimePassImpl
    : public impl::AttentionToRuntimePassBase<AttentionToRuntimePassImpl> {
  using impl::AttentionToRuntimePassBase<AttentionToRuntimePassImpl>::AttentionToRuntimePassBase;

  void runOnOperation() override {
    RewritePatternSet patterns(&getContext());
    patterns.add<FusedToRuntimeCall>(&getContext());
    FrozenRewritePatternSet frozen(std::move(patterns));
    if (failed(applyPatternsGreedily(getOperation(), frozen))) signalPassFailure();
    // Any op the pattern refused (it emitted an error) must fail the pass.
    getOperation().walk([&](FusedOp op) {
      op.emitOpError("not lowered to the runtime");
      signalPassFailure();
    });
  }
};

}  // namespace
}  // namespace mlir::attention
