module @jit_gemm_bf16 attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<256x256xbf16>, %arg1: tensor<256x256xbf16>) -> (tensor<256x256xf32>) {
    %0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<256x256xbf16>, tensor<256x256xbf16>) -> tensor<256x256xf32>
    return %0 : tensor<256x256xf32>
  }
}
