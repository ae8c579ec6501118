module @jit_argreduce attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<16x100xf32>) -> (tensor<16xf32>, tensor<16xi32>) {
    %0 = stablehlo.iota dim = 1 : tensor<16x100xi32>
    %cst = stablehlo.constant dense<0xFF800000> : tensor<f32>
    %cst_0 = stablehlo.constant dense<0> : tensor<i32>
    %1:2 = stablehlo.reduce(%arg0 init: %cst), (%0 init: %cst_0) across dimensions = [1] : (tensor<16x100xf32>, tensor<16x100xi32>, tensor<f32>, tensor<i32>) -> (tensor<16xf32>, tensor<16xi32>)
         reducer(%a0: tensor<f32>, %b0: tensor<f32>) (%a1: tensor<i32>, %b1: tensor<i32>)  {
          %g = stablehlo.compare  GT, %a0, %b0,  FLOAT : (tensor<f32>, tensor<f32>) -> tensor<i1>
          %n = stablehlo.compare  NE, %a0, %a0,  FLOAT : (tensor<f32>, tensor<f32>) -> tensor<i1>
          %p = stablehlo.or %g, %n : tensor<i1>
          %e = stablehlo.compare  EQ, %a0, %b0,  FLOAT : (tensor<f32>, tensor<f32>) -> tensor<i1>
          %l = stablehlo.compare  LT, %a1, %b1,  SIGNED : (tensor<i32>, tensor<i32>) -> tensor<i1>
          %q = stablehlo.and %e, %l : tensor<i1>
          %r = stablehlo.or %p, %q : tensor<i1>
          %v = stablehlo.select %p, %a0, %b0 : tensor<i1>, tensor<f32>
          %w = stablehlo.select %r, %a1, %b1 : tensor<i1>, tensor<i32>
          stablehlo.return %v, %w : tensor<f32>, tensor<i32>
        }
    return %1#0, %1#1 : tensor<16xf32>, tensor<16xi32>
  }
}
