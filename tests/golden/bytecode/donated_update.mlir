module @jit_donated_update attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<64x64xf32> {tf.aliasing_output = 0 : i32}, %arg1: tensor<64x64xf32> {jax.buffer_donor = true}, %arg2: tensor<64x64xf32> {tf.aliasing_output = 1 : i32}) -> (tensor<64x64xf32>, tensor<64x64xf32>) {
    %cst = stablehlo.constant dense<9.000000e-01> : tensor<f32>
    %0 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<64x64xf32>
    %1 = stablehlo.multiply %arg2, %0 : tensor<64x64xf32>
    %2 = stablehlo.add %1, %arg1 : tensor<64x64xf32>
    %cst_0 = stablehlo.constant dense<1.000000e-02> : tensor<f32>
    %3 = stablehlo.broadcast_in_dim %cst_0, dims = [] : (tensor<f32>) -> tensor<64x64xf32>
    %4 = stablehlo.multiply %2, %3 : tensor<64x64xf32>
    %5 = stablehlo.subtract %arg0, %4 : tensor<64x64xf32>
    return %5, %2 : tensor<64x64xf32>, tensor<64x64xf32>
  }
}
