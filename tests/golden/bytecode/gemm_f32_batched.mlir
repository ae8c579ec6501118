module @jit_gemm_f32 attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<2x128x128xf32>, %arg1: tensor<2x128x128xf32>) -> (tensor<2x128x128xf32>) {
    %0 = stablehlo.dot_general %arg0, %arg1, batching_dims = [0] x [0], contracting_dims = [2] x [1], precision = [DEFAULT, DEFAULT] : (tensor<2x128x128xf32>, tensor<2x128x128xf32>) -> tensor<2x128x128xf32>
    return %0 : tensor<2x128x128xf32>
  }
}
