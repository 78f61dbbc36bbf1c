// RUN: attention-opt %s --attention-to-runtime | FileCheck %s
//
// lit test for the runtime lowering (runs where attention-opt is built with
// MLIR).  Shapes follow the reference's tiling.mlir (64x32) and fusion.mlir
// (128x64 with a 128x128 mask).

// CHECK-DAG: func.func private @attn_fused_f32_nomask(memref<64x32xf32>, memref<64x32xf32>, memref<64x32xf32>, f32, memref<64x32xf32>) -> i32 attributes {llvm.emit_c_interface}
// CHECK-LABEL: func.func @plain
// CHECK:       call @attn_fused_f32_nomask
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
