module @jit_attention_full attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<1x2x256x64xbf16>, %arg1: tensor<1x2x256x64xbf16>, %arg2: tensor<1x2x256x64xbf16>) -> (tensor<1x2x256x64xbf16>) {
    %0 = stablehlo.dot_general %arg0, %arg1, batching_dims = [0, 1] x [0, 1], contracting_dims = [3] x [3], precision = [DEFAULT, DEFAULT] : (tensor<1x2x256x64xbf16>, tensor<1x2x256x64xbf16>) -> tensor<1x2x256x256xf32>
    %cst = stablehlo.constant dense<1.250000e-01> : tensor<f32>
    %1 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<1x2x256x256xf32>
    %2 = stablehlo.multiply %0, %1 : tensor<1x2x256x256xf32>
    %cst_0 = stablehlo.constant dense<0xFF800000> : tensor<f32>
    %3 = stablehlo.reduce(%2 init: %cst_0) applies stablehlo.maximum across dimensions = [3] : (tensor<1x2x256x256xf32>, tensor<f32>) -> tensor<1x2x256xf32>
    %4 = stablehlo.reshape %3 : (tensor<1x2x256xf32>) -> tensor<1x2x256x1xf32>
    %5 = stablehlo.reshape %4 : (tensor<1x2x256x1xf32>) -> tensor<1x2x256xf32>
    %6 = stablehlo.broadcast_in_dim %5, dims = [0, 1, 2] : (tensor<1x2x256xf32>) -> tensor<1x2x256x256xf32>
    %7 = stablehlo.subtract %2, %6 : tensor<1x2x256x256xf32>
    %8 = stablehlo.exponential %7 : tensor<1x2x256x256xf32>
    %cst_1 = stablehlo.constant dense<0.000000e+00> : tensor<f32>
    %9 = stablehlo.reduce(%8 init: %cst_1) applies stablehlo.add across dimensions = [3] : (tensor<1x2x256x256xf32>, tensor<f32>) -> tensor<1x2x256xf32>
    %10 = stablehlo.reshape %9 : (tensor<1x2x256xf32>) -> tensor<1x2x256x1xf32>
    %11 = stablehlo.reshape %10 : (tensor<1x2x256x1xf32>) -> tensor<1x2x256xf32>
    %12 = stablehlo.broadcast_in_dim %11, dims = [0, 1, 2] : (tensor<1x2x256xf32>) -> tensor<1x2x256x256xf32>
    %13 = stablehlo.divide %8, %12 : tensor<1x2x256x256xf32>
    %14 = stablehlo.convert %13 : (tensor<1x2x256x256xf32>) -> tensor<1x2x256x256xbf16>
    %15 = stablehlo.dot_general %14, %arg2, batching_dims = [0, 1] x [0, 1], contracting_dims = [3] x [2], precision = [DEFAULT, DEFAULT] : (tensor<1x2x256x256xbf16>, tensor<1x2x256x64xbf16>) -> tensor<1x2x256x64xbf16>
    return %15 : tensor<1x2x256x64xbf16>
  }
}
