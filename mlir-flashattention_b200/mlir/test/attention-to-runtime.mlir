// RUN: attention-opt %s --attention-to-runtime | FileCheck %s
//
// lit test for the runtime lowering (runs where attention-opt is built with
// MLIR).  Shapes follow the reference's tiling.mlir (64x32) and fusion.mlir
// (128x64 with a 128x128 mask).

// Every operand is cast to the fully dynamic strided type of its rank, so one
// declaration per callee serves all shapes in the module.
// CHECK-DAG: func.func private @attn_fused_f32_nomask(memref<?x?xf32, strided<[?, ?], offset: ?>>, memref<?x?xf32, strided<[?, ?], offset: ?>>, memref<?x?xf32, strided<[?, ?], offset: ?>>, f32, memref<?x?xf32, strided<[?, ?], offset: ?>>) -> i32 attributes {llvm.emit_c_interface}
// CHECK-DAG: func.func private @attn_fused_f32_mask(memref<?x?xf32, strided<[?, ?], offset: ?>>, memref<?x?xf32, strided<[?, ?], offset: ?>>, memref<?x?xf32, strided<[?, ?], offset: ?>>, f32, memref<?x?xi1, strided<[?, ?], offset: ?>>, memref<?x?xf32, strided<[?, ?], offset: ?>>) -> i32 attributes {llvm.emit_c_interface}
// CHECK-DAG: func.func private @attn_fused_bf16_causal_4d(memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, f32, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xf32, strided<[?, ?, ?, ?], offset: ?>>) -> i32 attributes {llvm.emit_c_interface}
// CHECK-DAG: func.func private @attn_fused_bf16_mask2d_4d(memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, f32, memref<?x?xi1, strided<[?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xf32, strided<[?, ?, ?, ?], offset: ?>>) -> i32 attributes {llvm.emit_c_interface}
// CHECK-DAG: func.func private @attn_fused_bf16_mask_4d(memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, f32, memref<?x?x?x?xi1, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xbf16, strided<[?, ?, ?, ?], offset: ?>>, memref<?x?x?x?xf32, strided<[?, ?, ?, ?], offset: ?>>) -> i32 attributes {llvm.emit_c_interface}
// CHECK-LABEL: func.func @plain
// CHECK:       memref.cast %{{.*}} : memref<64x32xf32> to memref<?x?xf32, strided<[?, ?], offset: ?>>
// CHECK:       %[[RC:.*]] = call @attn_fused_f32_nomask
// CHECK:       %[[OK:.*]] = arith.cmpi eq, %[[RC]], %{{.*}} : i32
// CHECK:       cf.assert %[[OK]], "attention.fused: runtime call attn_fused_f32_nomask failed
// CHECK-NOT:   attention.fused
func.func @plain(%Q: memref<64x32xf32>, %K: memref<64x32xf32>, %V: memref<64x32xf32>,
                 %s: f32, %O: memref<64x32xf32>) {
  attention.fused ins(%Q, %K, %V : memref<64x32xf32>, memref<64x32xf32>, memref<64x32xf32>)
    scale(%s : f32) outs(%O : memref<64x32xf32>)
  return
}

// CHECK-LABEL: func.func @causal
// CHECK:       call @attn_fused_f32_causal
// CHECK-NOT:   attention.fused
func.func @causal(%Q: memref<128x64xf32>, %K: memref<128x64xf32>, %V: memref<128x64xf32>,
                  %s: f32, %O: memref<128x64xf32>) {
  %m = memref.alloc() : memref<128x128xi1>
  linalg.generic {indexing_maps = [affine_map<(d0, d1) -> (d0, d1)>],
                  iterator_types = ["parallel", "parallel"]} outs(%m : memref<128x128xi1>) {
  ^bb0(%out: i1):
    %i = linalg.index 0 : index
    %j = linalg.index 1 : index
    %c = arith.cmpi ugt, %j, %i : index
    linalg.yield %c : i1
  }
  attention.fused ins(%Q, %K, %V : memref<128x64xf32>, memref<128x64xf32>, memref<128x64xf32>)
    scale(%s : f32) mask(%m : memref<128x128xi1>) outs(%O : memref<128x64xf32>)
  return
}

// CHECK-LABEL: func.func @dense
// CHECK:       call @attn_fused_f32_mask
func.func @dense(%Q: memref<128x64xf32>, %K: memref<128x64xf32>, %V: memref<128x64xf32>,
                 %s: f32, %m: memref<128x128xi1>, %O: memref<128x64xf32>) {
  attention.fused ins(%Q, %K, %V : memref<128x64xf32>, memref<128x64xf32>, memref<128x64xf32>)
    scale(%s : f32) mask(%m : memref<128x128xi1>) outs(%O : memref<128x64xf32>)
  return
}

// Two shapes in one function, one of them dynamic: both calls use the single
// declaration of @attn_fused_f32_nomask.
// CHECK-LABEL: func.func @two_shapes
// CHECK:       call @attn_fused_f32_nomask
// CHECK:       memref.cast %{{.*}} : memref<?x64xf32> to memref<?x?xf32, strided<[?, ?], offset: ?>>
// CHECK:       call @attn_fused_f32_nomask
func.func @two_shapes(%Q: memref<64x32xf32>, %K: memref<64x32xf32>, %V: memref<64x32xf32>,
                      %O: memref<64x32xf32>, %Q2: memref<?x64xf32>, %K2: memref<?x64xf32>,
                      %V2: memref<?x64xf32>, %O2: memref<?x64xf32>, %s: f32) {
  attention.fused ins(%Q, %K, %V : memref<64x32xf32>, memref<64x32xf32>, memref<64x32xf32>)
    scale(%s : f32) outs(%O : memref<64x32xf32>)
  attention.fused ins(%Q2, %K2, %V2 : memref<?x64xf32>, memref<?x64xf32>, memref<?x64xf32>)
    scale(%s : f32) outs(%O2 : memref<?x64xf32>)
  return
}

// Rank-4 bf16, causal: the LSE argument is a zero-sized alloca (not requested).
// CHECK-LABEL: func.func @bf16_causal
// CHECK:       memref.alloca() : memref<0x0x0x1xf32>
// CHECK:       call @attn_fused_bf16_causal_4d
func.func @bf16_causal(%Q: memref<1x32x16384x128xbf16>, %K: memref<1x32x16384x128xbf16>,
                       %V: memref<1x32x16384x128xbf16>, %O: memref<1x32x16384x128xbf16>,
                       %s: f32) {
  %m = memref.alloc() : memref<16384x16384xi1>
  linalg.generic {indexing_maps = [affine_map<(d0, d1) -> (d0, d1)>],
                  iterator_types = ["parallel", "parallel"]} outs(%m : memref<16384x16384xi1>) {
  ^bb0(%out: i1):
    %i = linalg.index 0 : index
    %j = linalg.index 1 : index
    %c = arith.cmpi ugt, %j, %i : index
    linalg.yield %c : i1
  }
  attention.fused ins(%Q, %K, %V : memref<1x32x16384x128xbf16>, memref<1x32x16384x128xbf16>,
                                   memref<1x32x16384x128xbf16>)
    scale(%s : f32) mask(%m : memref<16384x16384xi1>) outs(%O : memref<1x32x16384x128xbf16>)
  return
}

// Rank-4 bf16 operands with the op's own rank-2 dense mask [seq_q, seq_k]:
// the mask keeps its rank-2 descriptor and goes to the mask2d entry, which
// applies it to every (batch, head) slice.
// CHECK-LABEL: func.func @bf16_dense_rank2_mask
// CHECK:       memref.cast %{{.*}} : memref<300x300xi1> to memref<?x?xi1, strided<[?, ?], offset: ?>>
// CHECK:       %[[RC:.*]] = call @attn_fused_bf16_mask2d_4d
// CHECK:       cf.assert
func.func @bf16_dense_rank2_mask(%Q: memref<1x2x300x64xbf16>, %K: memref<1x2x300x64xbf16>,
                                 %V: memref<1x2x300x64xbf16>, %m: memref<300x300xi1>,
                                 %O: memref<1x2x300x64xbf16>, %s: f32) {
  attention.fused ins(%Q, %K, %V : memref<1x2x300x64xbf16>, memref<1x2x300x64xbf16>,
                                   memref<1x2x300x64xbf16>)
    scale(%s : f32) mask(%m : memref<300x300xi1>) outs(%O : memref<1x2x300x64xbf16>)
  return
}

// A per-slice rank-4 mask keeps the rank-4 mask entry.
// CHECK-LABEL: func.func @bf16_dense_rank4_mask
// CHECK:       call @attn_fused_bf16_mask_4d
func.func @bf16_dense_rank4_mask(%Q: memref<1x2x300x64xbf16>, %K: memref<1x2x300x64xbf16>,
                                 %V: memref<1x2x300x64xbf16>, %m: memref<1x2x300x300xi1>,
                                 %O: memref<1x2x300x64xbf16>, %s: f32) {
  attention.fused ins(%Q, %K, %V : memref<1x2x300x64xbf16>, memref<1x2x300x64xbf16>,
                                   memref<1x2x300x64xbf16>)
    scale(%s : f32) mask(%m : memref<1x2x300x300xi1>) outs(%O : memref<1x2x300x64xbf16>)
  return
}
