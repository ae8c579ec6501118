module @jit_mlp_step attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<784x512xf32>, %arg1: tensor<512xf32>, %arg2: tensor<512x10xf32>, %arg3: tensor<10xf32>, %arg4: tensor<128x784xf32>, %arg5: tensor<128xi32>) -> (tensor<f32>, tensor<784x512xf32>, tensor<512xf32>, tensor<512x10xf32>, tensor<10xf32>) {
    %0 = stablehlo.dot_general %arg4, %arg0, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<128x784xf32>, tensor<784x512xf32>) -> tensor<128x512xf32>
    %1 = stablehlo.broadcast_in_dim %arg1, dims = [1] : (tensor<512xf32>) -> tensor<128x512xf32>
    %2 = stablehlo.add %0, %1 : tensor<128x512xf32>
    %cst = stablehlo.constant dense<0.000000e+00> : tensor<f32>
    %3 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %4 = stablehlo.maximum %2, %3 : tensor<128x512xf32>
    %5 = stablehlo.dot_general %4, %arg2, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<128x512xf32>, tensor<512x10xf32>) -> tensor<128x10xf32>
    %6 = stablehlo.broadcast_in_dim %arg3, dims = [1] : (tensor<10xf32>) -> tensor<128x10xf32>
    %7 = stablehlo.add %5, %6 : tensor<128x10xf32>
    %cst_0 = stablehlo.constant dense<0xFF800000> : tensor<f32>
    %8 = stablehlo.reduce(%7 init: %cst_0) applies stablehlo.maximum across dimensions = [1] : (tensor<128x10xf32>, tensor<f32>) -> tensor<128xf32>
    %9 = stablehlo.reshape %8 : (tensor<128xf32>) -> tensor<128x1xf32>
    %10 = stablehlo.reshape %9 : (tensor<128x1xf32>) -> tensor<128xf32>
    %11 = stablehlo.broadcast_in_dim %10, dims = [0] : (tensor<128xf32>) -> tensor<128x10xf32>
    %12 = stablehlo.subtract %7, %11 : tensor<128x10xf32>
    %13 = stablehlo.exponential %12 : tensor<128x10xf32>
    %14 = stablehlo.reduce(%13 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<128x10xf32>, tensor<f32>) -> tensor<128xf32>
    %15 = stablehlo.reshape %14 : (tensor<128xf32>) -> tensor<128x1xf32>
    %16 = stablehlo.log %15 : tensor<128x1xf32>
    %17 = stablehlo.reshape %16 : (tensor<128x1xf32>) -> tensor<128xf32>
    %18 = stablehlo.broadcast_in_dim %17, dims = [0] : (tensor<128xf32>) -> tensor<128x10xf32>
    %19 = stablehlo.subtract %12, %18 : tensor<128x10xf32>
    %20 = stablehlo.broadcast_in_dim %arg5, dims = [0] : (tensor<128xi32>) -> tensor<128x10xi32>
    %21 = stablehlo.iota dim = 1 : tensor<128x10xi32>
    %22 = stablehlo.compare  EQ, %20, %21,  SIGNED : (tensor<128x10xi32>, tensor<128x10xi32>) -> tensor<128x10xi1>
    %23 = stablehlo.convert %22 : (tensor<128x10xi1>) -> tensor<128x10xf32>
    %24 = stablehlo.multiply %19, %23 : tensor<128x10xf32>
    %25 = stablehlo.reduce(%24 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<128x10xf32>, tensor<f32>) -> tensor<128xf32>
    %26 = stablehlo.reduce(%25 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<128xf32>, tensor<f32>) -> tensor<f32>
    %cst_1 = stablehlo.constant dense<1.280000e+02> : tensor<f32>
    %27 = stablehlo.divide %26, %cst_1 : tensor<f32>
    %28 = stablehlo.negate %27 : tensor<f32>
    %cst_2 = stablehlo.constant dense<1.000000e+00> : tensor<f32>
    %29 = stablehlo.negate %cst_2 : tensor<f32>
    %30 = stablehlo.divide %29, %cst_1 : tensor<f32>
    %34 = stablehlo.broadcast_in_dim %30, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %35 = stablehlo.broadcast_in_dim %34, dims = [0] : (tensor<128xf32>) -> tensor<128x10xf32>
    %36 = stablehlo.multiply %35, %23 : tensor<128x10xf32>
    %38 = stablehlo.negate %36 : tensor<128x10xf32>
    %39 = stablehlo.reduce(%38 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<128x10xf32>, tensor<f32>) -> tensor<128xf32>
    %40 = stablehlo.reshape %39 : (tensor<128xf32>) -> tensor<128x1xf32>
    %41 = stablehlo.divide %40, %15 : tensor<128x1xf32>
    %42 = stablehlo.reshape %41 : (tensor<128x1xf32>) -> tensor<128xf32>
    %43 = stablehlo.broadcast_in_dim %42, dims = [0] : (tensor<128xf32>) -> tensor<128x10xf32>
    %44 = stablehlo.multiply %43, %13 : tensor<128x10xf32>
    %45 = stablehlo.add %36, %44 : tensor<128x10xf32>
    %46 = stablehlo.negate %45 : tensor<128x10xf32>
    %47 = stablehlo.reduce(%46 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<128x10xf32>, tensor<f32>) -> tensor<128xf32>
    %48 = stablehlo.reshape %47 : (tensor<128xf32>) -> tensor<128x1xf32>
    %49 = stablehlo.reshape %48 : (tensor<128x1xf32>) -> tensor<128xf32>
    %50 = stablehlo.broadcast_in_dim %8, dims = [0] : (tensor<128xf32>) -> tensor<128x10xf32>
    %51 = stablehlo.compare  EQ, %7, %50,  FLOAT : (tensor<128x10xf32>, tensor<128x10xf32>) -> tensor<128x10xi1>
    %52 = stablehlo.convert %51 : (tensor<128x10xi1>) -> tensor<128x10xf32>
    %53 = stablehlo.reduce(%52 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<128x10xf32>, tensor<f32>) -> tensor<128xf32>
    %54 = stablehlo.broadcast_in_dim %53, dims = [0] : (tensor<128xf32>) -> tensor<128x10xf32>
    %55 = stablehlo.broadcast_in_dim %49, dims = [0] : (tensor<128xf32>) -> tensor<128x10xf32>
    %56 = stablehlo.multiply %55, %52 : tensor<128x10xf32>
    %57 = stablehlo.divide %56, %54 : tensor<128x10xf32>
    %58 = stablehlo.add %45, %57 : tensor<128x10xf32>
    %59 = stablehlo.reduce(%58 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<128x10xf32>, tensor<f32>) -> tensor<10xf32>
    %60 = stablehlo.dot_general %58, %arg2, contracting_dims = [1] x [1], precision = [DEFAULT, DEFAULT] : (tensor<128x10xf32>, tensor<512x10xf32>) -> tensor<128x512xf32>
    %61 = stablehlo.dot_general %4, %58, contracting_dims = [0] x [0], precision = [DEFAULT, DEFAULT] : (tensor<128x512xf32>, tensor<128x10xf32>) -> tensor<512x10xf32>
    %62 = stablehlo.compare  GT, %2, %3,  FLOAT : (tensor<128x512xf32>, tensor<128x512xf32>) -> tensor<128x512xi1>
    %63 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %64 = stablehlo.select %62, %60, %63 : tensor<128x512xi1>, tensor<128x512xf32>
    %67 = stablehlo.reduce(%64 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<128x512xf32>, tensor<f32>) -> tensor<512xf32>
    %69 = stablehlo.dot_general %arg4, %64, contracting_dims = [0] x [0], precision = [DEFAULT, DEFAULT] : (tensor<128x784xf32>, tensor<128x512xf32>) -> tensor<784x512xf32>
    %cst_3 = stablehlo.constant dense<1.000000e-02> : tensor<f32>
    %70 = stablehlo.broadcast_in_dim %cst_3, dims = [] : (tensor<f32>) -> tensor<784x512xf32>
    %71 = stablehlo.multiply %70, %69 : tensor<784x512xf32>
    %72 = stablehlo.subtract %arg0, %71 : tensor<784x512xf32>
    %73 = stablehlo.broadcast_in_dim %cst_3, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %74 = stablehlo.multiply %73, %67 : tensor<512xf32>
    %75 = stablehlo.subtract %arg1, %74 : tensor<512xf32>
    %76 = stablehlo.broadcast_in_dim %cst_3, dims = [] : (tensor<f32>) -> tensor<512x10xf32>
    %77 = stablehlo.multiply %76, %61 : tensor<512x10xf32>
    %78 = stablehlo.subtract %arg2, %77 : tensor<512x10xf32>
    %79 = stablehlo.broadcast_in_dim %cst_3, dims = [] : (tensor<f32>) -> tensor<10xf32>
    %80 = stablehlo.multiply %79, %59 : tensor<10xf32>
    %81 = stablehlo.subtract %arg3, %80 : tensor<10xf32>
    return %28, %72, %75, %78, %81 : tensor<f32>, tensor<784x512xf32>, tensor<512xf32>, tensor<512x10xf32>, tensor<10xf32>
  }
}
