module @jit_misc attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func private @scale(%arg0: tensor<4x8xf32>) -> tensor<4x8xf32> {
    %cst = stablehlo.constant dense<2.500000e-01> : tensor<f32>
    %0 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<4x8xf32>
    %1 = stablehlo.multiply %arg0, %0 : tensor<4x8xf32>
    return %1 : tensor<4x8xf32>
  }
  func.func public @main(%arg0: tensor<4x8xf32>, %arg1: tensor<4x8xui32>, %arg2: tensor<4x8xf16>) -> (tensor<4x8xf32>, tensor<4x8xi1>, tensor<4x16xf16>, tensor<2x8xf32>, tensor<8x4xf32>, tensor<4x8xi32>, tensor<12xi1>, tensor<3xf32>, tensor<4xf32>) {
    %0 = call @scale(%arg0) : (tensor<4x8xf32>) -> tensor<4x8xf32>
    %c = stablehlo.constant dense<[true, false, true, false, true, true, false, false]> : tensor<8xi1>
    %1 = stablehlo.broadcast_in_dim %c, dims = [1] : (tensor<8xi1>) -> tensor<4x8xi1>
    %c_0 = stablehlo.constant dense<7> : tensor<ui32>
    %2 = stablehlo.broadcast_in_dim %c_0, dims = [] : (tensor<ui32>) -> tensor<4x8xui32>
    %3 = stablehlo.compare  GT, %arg1, %2,  UNSIGNED : (tensor<4x8xui32>, tensor<4x8xui32>) -> tensor<4x8xi1>
    %4 = stablehlo.and %1, %3 : tensor<4x8xi1>
    %5 = stablehlo.concatenate %arg2, %arg2, dim = 1 : (tensor<4x8xf16>, tensor<4x8xf16>) -> tensor<4x16xf16>
    %6 = stablehlo.slice %0 [1:3, 0:8] : (tensor<4x8xf32>) -> tensor<2x8xf32>
    %7 = stablehlo.transpose %0, dims = [1, 0] : (tensor<4x8xf32>) -> tensor<8x4xf32>
    %8 = stablehlo.iota dim = 1 : tensor<4x8xi32>
    %c_1 = stablehlo.constant dense<[[1, -2, 3, -4, 5, -6, 7, -8], [0, 0, 0, 0, 0, 0, 0, 0], [9, 9, 9, 9, 9, 9, 9, 9], [-1, -1, -1, -1, -1, -1, -1, -2147483648]]> : tensor<4x8xi32>
    %9 = stablehlo.add %8, %c_1 : tensor<4x8xi32>
    %c_2 = stablehlo.constant dense<true> : tensor<4x8xi1>
    %10 = stablehlo.xor %4, %c_2 : tensor<4x8xi1>
    %c_3 = stablehlo.constant dense<[true, true, false, true, false, false, true, false, true, true, true, false]> : tensor<12xi1>
    %c_4 = stablehlo.constant dense<[false, true, true, true, true, false, true, false, true, false, true, true]> : tensor<12xi1>
    %11 = stablehlo.or %c_3, %c_4 : tensor<12xi1>
    %c_5 = stablehlo.constant dense<[1.5, -2.25, 0x7FC00000]> : tensor<3xf32>
    %c_6 = stablehlo.constant dense<[1.0, -0.5, 3.0, 65504.0]> : tensor<4xbf16>
    %12 = stablehlo.convert %c_6 : (tensor<4xbf16>) -> tensor<4xf32>
    return %0, %10, %5, %6, %7, %9, %11, %c_5, %12 : tensor<4x8xf32>, tensor<4x8xi1>, tensor<4x16xf16>, tensor<2x8xf32>, tensor<8x4xf32>, tensor<4x8xi32>, tensor<12xi1>, tensor<3xf32>, tensor<4xf32>
  }
}
