//===- AttentionToRuntime.td - pass declaration ------------*- tablegen -*-===//
//
// Declaration of the B200 runtime lowering pass, to be added to the
// reference's include/Attention/AttentionPasses.td next to FusionPass and
// TilingPass (AttentionPasses.td:14-51).  The generated base class
// impl::AttentionToRuntimePassBase is used by RuntimeLoweringPass.cpp and the
// pass is registered by the existing mlir::attention::registerPasses()
// (AttentionPasses.h:22-23), so attention-opt gains --attention-to-runtime
// without other changes.
//
//===----------------------------------------------------------------------===//

def AttentionToRuntimePass : Pass<"attention-to-runtime", "::mlir::ModuleOp"> {
  let summary = "Lower attention.fused to calls into the B200 attention runtime";
  let description = [{
    Replaces each attention.fused op (normally produced by --fusion-pass) by a
    func.call to attn_fused_<dtype>_<variant>[_4d], declared private with
    llvm.emit_c_interface so that the lowered program calls
    _mlir_ciface_attn_fused_* in libattnrt.so.  The variant is chosen from the
    mask operand: none -> nomask, a causal generic (j > i) -> causal, any
    other i1 mask -> mask (rank-2 f32, rank-4 bf16) or mask2d (a rank-2
    mask on rank-4 bf16 operands).  The returned status is checked with
    cf.assert.  Use instead of --tiling-pass.
  }];
  let dependentDialects = ["::mlir::func::FuncDialect", "::mlir::memref::MemRefDialect",
                           "::mlir::arith::ArithDialect", "::mlir::cf::ControlFlowDialect"];
}
