module @jit_gpt2_dp_step attributes {mhlo.num_partitions = 2 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<512x128xbf16>, %arg1: tensor<256x128xbf16>, %arg2: tensor<128xbf16>, %arg3: tensor<128xbf16>, %arg4: tensor<128x384xbf16>, %arg5: tensor<384xbf16>, %arg6: tensor<128x128xbf16>, %arg7: tensor<128xbf16>, %arg8: tensor<128xbf16>, %arg9: tensor<128xbf16>, %arg10: tensor<128x512xbf16>, %arg11: tensor<512xbf16>, %arg12: tensor<512x128xbf16>, %arg13: tensor<128xbf16>, %arg14: tensor<128xbf16>, %arg15: tensor<128xbf16>, %arg16: tensor<512x128xf32>, %arg17: tensor<256x128xf32>, %arg18: tensor<128xf32>, %arg19: tensor<128xf32>, %arg20: tensor<128x384xf32>, %arg21: tensor<384xf32>, %arg22: tensor<128x128xf32>, %arg23: tensor<128xf32>, %arg24: tensor<128xf32>, %arg25: tensor<128xf32>, %arg26: tensor<128x512xf32>, %arg27: tensor<512xf32>, %arg28: tensor<512x128xf32>, %arg29: tensor<128xf32>, %arg30: tensor<128xf32>, %arg31: tensor<128xf32>, %arg32: tensor<512x128xf32>, %arg33: tensor<256x128xf32>, %arg34: tensor<128xf32>, %arg35: tensor<128xf32>, %arg36: tensor<128x384xf32>, %arg37: tensor<384xf32>, %arg38: tensor<128x128xf32>, %arg39: tensor<128xf32>, %arg40: tensor<128xf32>, %arg41: tensor<128xf32>, %arg42: tensor<128x512xf32>, %arg43: tensor<512xf32>, %arg44: tensor<512x128xf32>, %arg45: tensor<128xf32>, %arg46: tensor<128xf32>, %arg47: tensor<128xf32>, %arg48: tensor<4x256xi32>, %arg49: tensor<4x256xi32>, %arg50: tensor<f32>, %arg51: tensor<f32>) -> (tensor<512x128xbf16>, tensor<256x128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128x384xbf16>, tensor<384xbf16>, tensor<128x128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128x512xbf16>, tensor<512xbf16>, tensor<512x128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<512x128xf32>, tensor<256x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x384xf32>, tensor<384xf32>, tensor<128x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x512xf32>, tensor<512xf32>, tensor<512x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<512x128xf32>, tensor<256x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x384xf32>, tensor<384xf32>, tensor<128x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x512xf32>, tensor<512xf32>, tensor<512x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<f32>) {
    %0 = stablehlo.custom_call @Sharding(%arg48) {mhlo.sharding = "{devices=[2,1]<=[2]}"} : (tensor<4x256xi32>) -> tensor<4x256xi32>
    %1 = stablehlo.custom_call @SPMDFullToShardShape(%0) {mhlo.sharding = "{manual}"} : (tensor<4x256xi32>) -> tensor<2x256xi32>
    %2 = stablehlo.custom_call @Sharding(%arg49) {mhlo.sharding = "{devices=[2,1]<=[2]}"} : (tensor<4x256xi32>) -> tensor<4x256xi32>
    %3 = stablehlo.custom_call @SPMDFullToShardShape(%2) {mhlo.sharding = "{manual}"} : (tensor<4x256xi32>) -> tensor<2x256xi32>
    %4 = stablehlo.reshape %1 : (tensor<2x256xi32>) -> tensor<2x256x1xi32>
    %5 = "stablehlo.gather"(%arg0, %4) <{dimension_numbers = #stablehlo.gather<offset_dims = [2], collapsed_slice_dims = [0], start_index_map = [0], index_vector_dim = 2>, indices_are_sorted = false, slice_sizes = array<i64: 1, 128>}> : (tensor<512x128xbf16>, tensor<2x256x1xi32>) -> tensor<2x256x128xbf16>
    %6 = stablehlo.broadcast_in_dim %arg1, dims = [1, 2] : (tensor<256x128xbf16>) -> tensor<2x256x128xbf16>
    %7 = stablehlo.add %5, %6 : tensor<2x256x128xbf16>
    %8 = stablehlo.reshape %7 : (tensor<2x256x128xbf16>) -> tensor<512x128xbf16>
    %9 = stablehlo.convert %8 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %cst = stablehlo.constant dense<0.000000e+00> : tensor<f32>
    %10 = stablehlo.reduce(%9 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %11 = stablehlo.reshape %10 : (tensor<512xf32>) -> tensor<512x1xf32>
    %cst_0 = stablehlo.constant dense<1.280000e+02> : tensor<f32>
    %12 = stablehlo.broadcast_in_dim %cst_0, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %13 = stablehlo.divide %11, %12 : tensor<512x1xf32>
    %14 = stablehlo.reshape %13 : (tensor<512x1xf32>) -> tensor<512xf32>
    %15 = stablehlo.broadcast_in_dim %14, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %16 = stablehlo.subtract %9, %15 : tensor<512x128xf32>
    %17 = stablehlo.multiply %16, %16 : tensor<512x128xf32>
    %18 = stablehlo.reduce(%17 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %19 = stablehlo.reshape %18 : (tensor<512xf32>) -> tensor<512x1xf32>
    %20 = stablehlo.broadcast_in_dim %cst_0, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %21 = stablehlo.divide %19, %20 : tensor<512x1xf32>
    %cst_1 = stablehlo.constant dense<1.000000e-05> : tensor<f32>
    %22 = stablehlo.broadcast_in_dim %cst_1, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %23 = stablehlo.add %21, %22 : tensor<512x1xf32>
    %24 = stablehlo.rsqrt %23 : tensor<512x1xf32>
    %25 = stablehlo.reshape %24 : (tensor<512x1xf32>) -> tensor<512xf32>
    %26 = stablehlo.broadcast_in_dim %25, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %27 = stablehlo.multiply %16, %26 : tensor<512x128xf32>
    %28 = stablehlo.convert %arg2 : (tensor<128xbf16>) -> tensor<128xf32>
    %29 = stablehlo.broadcast_in_dim %28, dims = [1] : (tensor<128xf32>) -> tensor<512x128xf32>
    %30 = stablehlo.multiply %27, %29 : tensor<512x128xf32>
    %31 = stablehlo.convert %arg3 : (tensor<128xbf16>) -> tensor<128xf32>
    %32 = stablehlo.broadcast_in_dim %31, dims = [1] : (tensor<128xf32>) -> tensor<512x128xf32>
    %33 = stablehlo.add %30, %32 : tensor<512x128xf32>
    %34 = stablehlo.convert %33 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %35 = stablehlo.dot_general %34, %arg4, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<128x384xbf16>) -> tensor<512x384xbf16>
    %36 = stablehlo.broadcast_in_dim %arg5, dims = [1] : (tensor<384xbf16>) -> tensor<512x384xbf16>
    %37 = stablehlo.add %35, %36 : tensor<512x384xbf16>
    %38 = stablehlo.slice %37 [0:512, 0:128] : (tensor<512x384xbf16>) -> tensor<512x128xbf16>
    %39 = stablehlo.reshape %38 : (tensor<512x128xbf16>) -> tensor<2x256x2x64xbf16>
    %40 = stablehlo.transpose %39, dims = [0, 2, 1, 3] : (tensor<2x256x2x64xbf16>) -> tensor<2x2x256x64xbf16>
    %41 = stablehlo.slice %37 [0:512, 128:256] : (tensor<512x384xbf16>) -> tensor<512x128xbf16>
    %42 = stablehlo.reshape %41 : (tensor<512x128xbf16>) -> tensor<2x256x2x64xbf16>
    %43 = stablehlo.transpose %42, dims = [0, 2, 1, 3] : (tensor<2x256x2x64xbf16>) -> tensor<2x2x256x64xbf16>
    %44 = stablehlo.slice %37 [0:512, 256:384] : (tensor<512x384xbf16>) -> tensor<512x128xbf16>
    %45 = stablehlo.reshape %44 : (tensor<512x128xbf16>) -> tensor<2x256x2x64xbf16>
    %46 = stablehlo.transpose %45, dims = [0, 2, 1, 3] : (tensor<2x256x2x64xbf16>) -> tensor<2x2x256x64xbf16>
    %47 = stablehlo.dot_general %40, %43, batching_dims = [0, 1] x [0, 1], contracting_dims = [3] x [3], precision = [DEFAULT, DEFAULT] : (tensor<2x2x256x64xbf16>, tensor<2x2x256x64xbf16>) -> tensor<2x2x256x256xf32>
    %cst_2 = stablehlo.constant dense<1.250000e-01> : tensor<f32>
    %48 = stablehlo.broadcast_in_dim %cst_2, dims = [] : (tensor<f32>) -> tensor<2x2x256x256xf32>
    %49 = stablehlo.multiply %47, %48 : tensor<2x2x256x256xf32>
    %50 = stablehlo.iota dim = 0 : tensor<256x256xi32>
    %51 = stablehlo.iota dim = 1 : tensor<256x256xi32>
    %52 = stablehlo.compare  GE, %50, %51,  SIGNED : (tensor<256x256xi32>, tensor<256x256xi32>) -> tensor<256x256xi1>
    %53 = stablehlo.broadcast_in_dim %52, dims = [2, 3] : (tensor<256x256xi1>) -> tensor<2x2x256x256xi1>
    %cst_3 = stablehlo.constant dense<0xFF800000> : tensor<f32>
    %54 = stablehlo.broadcast_in_dim %cst_3, dims = [] : (tensor<f32>) -> tensor<2x2x256x256xf32>
    %55 = stablehlo.select %53, %49, %54 : tensor<2x2x256x256xi1>, tensor<2x2x256x256xf32>
    %56 = stablehlo.reduce(%55 init: %cst_3) applies stablehlo.maximum across dimensions = [3] : (tensor<2x2x256x256xf32>, tensor<f32>) -> tensor<2x2x256xf32>
    %57 = stablehlo.reshape %56 : (tensor<2x2x256xf32>) -> tensor<2x2x256x1xf32>
    %58 = stablehlo.reshape %57 : (tensor<2x2x256x1xf32>) -> tensor<2x2x256xf32>
    %59 = stablehlo.broadcast_in_dim %58, dims = [0, 1, 2] : (tensor<2x2x256xf32>) -> tensor<2x2x256x256xf32>
    %60 = stablehlo.subtract %55, %59 : tensor<2x2x256x256xf32>
    %61 = stablehlo.exponential %60 : tensor<2x2x256x256xf32>
    %62 = stablehlo.reduce(%61 init: %cst) applies stablehlo.add across dimensions = [3] : (tensor<2x2x256x256xf32>, tensor<f32>) -> tensor<2x2x256xf32>
    %63 = stablehlo.reshape %62 : (tensor<2x2x256xf32>) -> tensor<2x2x256x1xf32>
    %64 = stablehlo.reshape %63 : (tensor<2x2x256x1xf32>) -> tensor<2x2x256xf32>
    %65 = stablehlo.broadcast_in_dim %64, dims = [0, 1, 2] : (tensor<2x2x256xf32>) -> tensor<2x2x256x256xf32>
    %66 = stablehlo.divide %61, %65 : tensor<2x2x256x256xf32>
    %67 = stablehlo.convert %66 : (tensor<2x2x256x256xf32>) -> tensor<2x2x256x256xbf16>
    %68 = stablehlo.dot_general %67, %46, batching_dims = [0, 1] x [0, 1], contracting_dims = [3] x [2], precision = [DEFAULT, DEFAULT] : (tensor<2x2x256x256xbf16>, tensor<2x2x256x64xbf16>) -> tensor<2x2x256x64xbf16>
    %69 = stablehlo.transpose %68, dims = [0, 2, 1, 3] : (tensor<2x2x256x64xbf16>) -> tensor<2x256x2x64xbf16>
    %70 = stablehlo.reshape %69 : (tensor<2x256x2x64xbf16>) -> tensor<512x128xbf16>
    %71 = stablehlo.dot_general %70, %arg6, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<128x128xbf16>) -> tensor<512x128xbf16>
    %72 = stablehlo.broadcast_in_dim %arg7, dims = [1] : (tensor<128xbf16>) -> tensor<512x128xbf16>
    %73 = stablehlo.add %71, %72 : tensor<512x128xbf16>
    %74 = stablehlo.add %8, %73 : tensor<512x128xbf16>
    %75 = stablehlo.convert %74 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %76 = stablehlo.reduce(%75 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %77 = stablehlo.reshape %76 : (tensor<512xf32>) -> tensor<512x1xf32>
    %78 = stablehlo.broadcast_in_dim %cst_0, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %79 = stablehlo.divide %77, %78 : tensor<512x1xf32>
    %80 = stablehlo.reshape %79 : (tensor<512x1xf32>) -> tensor<512xf32>
    %81 = stablehlo.broadcast_in_dim %80, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %82 = stablehlo.subtract %75, %81 : tensor<512x128xf32>
    %83 = stablehlo.multiply %82, %82 : tensor<512x128xf32>
    %84 = stablehlo.reduce(%83 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %85 = stablehlo.reshape %84 : (tensor<512xf32>) -> tensor<512x1xf32>
    %86 = stablehlo.broadcast_in_dim %cst_0, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %87 = stablehlo.divide %85, %86 : tensor<512x1xf32>
    %88 = stablehlo.broadcast_in_dim %cst_1, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %89 = stablehlo.add %87, %88 : tensor<512x1xf32>
    %90 = stablehlo.rsqrt %89 : tensor<512x1xf32>
    %91 = stablehlo.reshape %90 : (tensor<512x1xf32>) -> tensor<512xf32>
    %92 = stablehlo.broadcast_in_dim %91, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %93 = stablehlo.multiply %82, %92 : tensor<512x128xf32>
    %94 = stablehlo.convert %arg8 : (tensor<128xbf16>) -> tensor<128xf32>
    %95 = stablehlo.broadcast_in_dim %94, dims = [1] : (tensor<128xf32>) -> tensor<512x128xf32>
    %96 = stablehlo.multiply %93, %95 : tensor<512x128xf32>
    %97 = stablehlo.convert %arg9 : (tensor<128xbf16>) -> tensor<128xf32>
    %98 = stablehlo.broadcast_in_dim %97, dims = [1] : (tensor<128xf32>) -> tensor<512x128xf32>
    %99 = stablehlo.add %96, %98 : tensor<512x128xf32>
    %100 = stablehlo.convert %99 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %101 = stablehlo.dot_general %100, %arg10, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<128x512xbf16>) -> tensor<512x512xbf16>
    %102 = stablehlo.broadcast_in_dim %arg11, dims = [1] : (tensor<512xbf16>) -> tensor<512x512xbf16>
    %103 = stablehlo.add %101, %102 : tensor<512x512xbf16>
    %104 = stablehlo.convert %103 : (tensor<512x512xbf16>) -> tensor<512x512xf32>
    %105 = stablehlo.multiply %104, %104 : tensor<512x512xf32>
    %106 = stablehlo.multiply %105, %104 : tensor<512x512xf32>
    %cst_4 = stablehlo.constant dense<4.471500e-02> : tensor<f32>
    %107 = stablehlo.broadcast_in_dim %cst_4, dims = [] : (tensor<f32>) -> tensor<512x512xf32>
    %108 = stablehlo.multiply %107, %106 : tensor<512x512xf32>
    %109 = stablehlo.add %104, %108 : tensor<512x512xf32>
    %cst_5 = stablehlo.constant dense<7.978846e-01> : tensor<f32>
    %110 = stablehlo.broadcast_in_dim %cst_5, dims = [] : (tensor<f32>) -> tensor<512x512xf32>
    %111 = stablehlo.multiply %109, %110 : tensor<512x512xf32>
    %cst_6 = stablehlo.constant dense<5.000000e-01> : tensor<f32>
    %112 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<512x512xf32>
    %113 = stablehlo.multiply %112, %104 : tensor<512x512xf32>
    %114 = stablehlo.tanh %111 : tensor<512x512xf32>
    %cst_7 = stablehlo.constant dense<1.000000e+00> : tensor<f32>
    %115 = stablehlo.broadcast_in_dim %cst_7, dims = [] : (tensor<f32>) -> tensor<512x512xf32>
    %116 = stablehlo.add %115, %114 : tensor<512x512xf32>
    %117 = stablehlo.multiply %113, %116 : tensor<512x512xf32>
    %118 = stablehlo.convert %117 : (tensor<512x512xf32>) -> tensor<512x512xbf16>
    %119 = stablehlo.dot_general %118, %arg12, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x512xbf16>, tensor<512x128xbf16>) -> tensor<512x128xbf16>
    %120 = stablehlo.broadcast_in_dim %arg13, dims = [1] : (tensor<128xbf16>) -> tensor<512x128xbf16>
    %121 = stablehlo.add %119, %120 : tensor<512x128xbf16>
    %122 = stablehlo.add %74, %121 : tensor<512x128xbf16>
    %123 = stablehlo.convert %122 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %124 = stablehlo.reduce(%123 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %125 = stablehlo.reshape %124 : (tensor<512xf32>) -> tensor<512x1xf32>
    %126 = stablehlo.broadcast_in_dim %cst_0, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %127 = stablehlo.divide %125, %126 : tensor<512x1xf32>
    %128 = stablehlo.reshape %127 : (tensor<512x1xf32>) -> tensor<512xf32>
    %129 = stablehlo.broadcast_in_dim %128, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %130 = stablehlo.subtract %123, %129 : tensor<512x128xf32>
    %131 = stablehlo.multiply %130, %130 : tensor<512x128xf32>
    %132 = stablehlo.reduce(%131 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %133 = stablehlo.reshape %132 : (tensor<512xf32>) -> tensor<512x1xf32>
    %134 = stablehlo.broadcast_in_dim %cst_0, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %135 = stablehlo.divide %133, %134 : tensor<512x1xf32>
    %136 = stablehlo.broadcast_in_dim %cst_1, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %137 = stablehlo.add %135, %136 : tensor<512x1xf32>
    %138 = stablehlo.rsqrt %137 : tensor<512x1xf32>
    %139 = stablehlo.reshape %138 : (tensor<512x1xf32>) -> tensor<512xf32>
    %140 = stablehlo.broadcast_in_dim %139, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %141 = stablehlo.multiply %130, %140 : tensor<512x128xf32>
    %142 = stablehlo.convert %arg14 : (tensor<128xbf16>) -> tensor<128xf32>
    %143 = stablehlo.broadcast_in_dim %142, dims = [1] : (tensor<128xf32>) -> tensor<512x128xf32>
    %144 = stablehlo.multiply %141, %143 : tensor<512x128xf32>
    %145 = stablehlo.convert %arg15 : (tensor<128xbf16>) -> tensor<128xf32>
    %146 = stablehlo.broadcast_in_dim %145, dims = [1] : (tensor<128xf32>) -> tensor<512x128xf32>
    %147 = stablehlo.add %144, %146 : tensor<512x128xf32>
    %148 = stablehlo.convert %147 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %149 = stablehlo.dot_general %148, %arg0, contracting_dims = [1] x [1], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<512x128xbf16>) -> tensor<512x512xf32>
    %150 = stablehlo.reduce(%149 init: %cst_3) applies stablehlo.maximum across dimensions = [1] : (tensor<512x512xf32>, tensor<f32>) -> tensor<512xf32>
    %151 = stablehlo.reshape %150 : (tensor<512xf32>) -> tensor<512x1xf32>
    %152 = stablehlo.reshape %151 : (tensor<512x1xf32>) -> tensor<512xf32>
    %153 = stablehlo.broadcast_in_dim %152, dims = [0] : (tensor<512xf32>) -> tensor<512x512xf32>
    %154 = stablehlo.subtract %149, %153 : tensor<512x512xf32>
    %155 = stablehlo.exponential %154 : tensor<512x512xf32>
    %156 = stablehlo.reduce(%155 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x512xf32>, tensor<f32>) -> tensor<512xf32>
    %157 = stablehlo.reshape %156 : (tensor<512xf32>) -> tensor<512x1xf32>
    %158 = stablehlo.log %157 : tensor<512x1xf32>
    %159 = stablehlo.reshape %3 : (tensor<2x256xi32>) -> tensor<512xi32>
    %160 = stablehlo.broadcast_in_dim %159, dims = [0] : (tensor<512xi32>) -> tensor<512x512xi32>
    %161 = stablehlo.iota dim = 1 : tensor<512x512xi32>
    %162 = stablehlo.compare  EQ, %160, %161,  SIGNED : (tensor<512x512xi32>, tensor<512x512xi32>) -> tensor<512x512xi1>
    %163 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<512x512xf32>
    %164 = stablehlo.select %162, %154, %163 : tensor<512x512xi1>, tensor<512x512xf32>
    %165 = stablehlo.reduce(%164 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x512xf32>, tensor<f32>) -> tensor<512xf32>
    %166 = stablehlo.reshape %165 : (tensor<512xf32>) -> tensor<512x1xf32>
    %167 = stablehlo.subtract %158, %166 : tensor<512x1xf32>
    %168 = stablehlo.reduce(%167 init: %cst) applies stablehlo.add across dimensions = [0, 1] : (tensor<512x1xf32>, tensor<f32>) -> tensor<f32>
    %cst_8 = stablehlo.constant dense<5.120000e+02> : tensor<f32>
    %169 = stablehlo.divide %168, %cst_8 : tensor<f32>
    %170 = stablehlo.divide %cst_7, %cst_8 : tensor<f32>
    %174 = stablehlo.broadcast_in_dim %170, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %175 = stablehlo.negate %174 : tensor<512x1xf32>
    %176 = stablehlo.reshape %175 : (tensor<512x1xf32>) -> tensor<512xf32>
    %177 = stablehlo.broadcast_in_dim %176, dims = [0] : (tensor<512xf32>) -> tensor<512x512xf32>
    %178 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<512x512xf32>
    %179 = stablehlo.select %162, %177, %178 : tensor<512x512xi1>, tensor<512x512xf32>
    %182 = stablehlo.divide %174, %157 : tensor<512x1xf32>
    %183 = stablehlo.reshape %182 : (tensor<512x1xf32>) -> tensor<512xf32>
    %184 = stablehlo.broadcast_in_dim %183, dims = [0] : (tensor<512xf32>) -> tensor<512x512xf32>
    %185 = stablehlo.multiply %184, %155 : tensor<512x512xf32>
    %186 = stablehlo.add %179, %185 : tensor<512x512xf32>
    %190 = stablehlo.dot_general %186, %arg0, contracting_dims = [1] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x512xf32>, tensor<512x128xbf16>) -> tensor<512x128xbf16>
    %191 = stablehlo.dot_general %148, %186, contracting_dims = [0] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<512x512xf32>) -> tensor<128x512xbf16>
    %192 = stablehlo.transpose %191, dims = [1, 0] : (tensor<128x512xbf16>) -> tensor<512x128xbf16>
    %193 = stablehlo.convert %190 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %194 = stablehlo.reduce(%193 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<512x128xf32>, tensor<f32>) -> tensor<128xf32>
    %195 = stablehlo.convert %194 : (tensor<128xf32>) -> tensor<128xbf16>
    %196 = stablehlo.multiply %193, %143 : tensor<512x128xf32>
    %197 = stablehlo.multiply %193, %141 : tensor<512x128xf32>
    %198 = stablehlo.reduce(%197 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<512x128xf32>, tensor<f32>) -> tensor<128xf32>
    %199 = stablehlo.convert %198 : (tensor<128xf32>) -> tensor<128xbf16>
    %200 = stablehlo.multiply %196, %140 : tensor<512x128xf32>
    %201 = stablehlo.multiply %196, %130 : tensor<512x128xf32>
    %202 = stablehlo.reduce(%201 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %203 = stablehlo.reshape %202 : (tensor<512xf32>) -> tensor<512x1xf32>
    %cst_9 = stablehlo.constant dense<-5.000000e-01> : tensor<f32>
    %204 = stablehlo.broadcast_in_dim %cst_9, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %205 = stablehlo.multiply %203, %204 : tensor<512x1xf32>
    %206 = stablehlo.multiply %205, %138 : tensor<512x1xf32>
    %207 = stablehlo.divide %206, %137 : tensor<512x1xf32>
    %209 = stablehlo.divide %207, %134 : tensor<512x1xf32>
    %214 = stablehlo.reshape %209 : (tensor<512x1xf32>) -> tensor<512xf32>
    %215 = stablehlo.broadcast_in_dim %214, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %216 = stablehlo.multiply %215, %130 : tensor<512x128xf32>
    %217 = stablehlo.add %200, %216 : tensor<512x128xf32>
    %218 = stablehlo.multiply %215, %130 : tensor<512x128xf32>
    %219 = stablehlo.add %217, %218 : tensor<512x128xf32>
    %220 = stablehlo.negate %219 : tensor<512x128xf32>
    %221 = stablehlo.reduce(%220 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %222 = stablehlo.reshape %221 : (tensor<512xf32>) -> tensor<512x1xf32>
    %223 = stablehlo.divide %222, %126 : tensor<512x1xf32>
    %228 = stablehlo.reshape %223 : (tensor<512x1xf32>) -> tensor<512xf32>
    %229 = stablehlo.broadcast_in_dim %228, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %230 = stablehlo.add %219, %229 : tensor<512x128xf32>
    %231 = stablehlo.convert %230 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %cst_10 = stablehlo.constant dense<0.000000e+00> : tensor<bf16>
    %232 = stablehlo.reduce(%231 init: %cst_10) applies stablehlo.add across dimensions = [0] : (tensor<512x128xbf16>, tensor<bf16>) -> tensor<128xbf16>
    %233 = stablehlo.dot_general %231, %arg12, contracting_dims = [1] x [1], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<512x128xbf16>) -> tensor<512x512xbf16>
    %234 = stablehlo.dot_general %118, %231, contracting_dims = [0] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x512xbf16>, tensor<512x128xbf16>) -> tensor<512x128xbf16>
    %235 = stablehlo.convert %233 : (tensor<512x512xbf16>) -> tensor<512x512xf32>
    %236 = stablehlo.multiply %235, %116 : tensor<512x512xf32>
    %237 = stablehlo.multiply %235, %113 : tensor<512x512xf32>
    %239 = stablehlo.multiply %114, %114 : tensor<512x512xf32>
    %240 = stablehlo.broadcast_in_dim %cst_7, dims = [] : (tensor<f32>) -> tensor<512x512xf32>
    %241 = stablehlo.subtract %240, %239 : tensor<512x512xf32>
    %242 = stablehlo.multiply %237, %241 : tensor<512x512xf32>
    %244 = stablehlo.multiply %236, %112 : tensor<512x512xf32>
    %246 = stablehlo.multiply %242, %110 : tensor<512x512xf32>
    %249 = stablehlo.add %244, %246 : tensor<512x512xf32>
    %251 = stablehlo.multiply %246, %107 : tensor<512x512xf32>
    %253 = stablehlo.multiply %251, %104 : tensor<512x512xf32>
    %254 = stablehlo.multiply %251, %105 : tensor<512x512xf32>
    %255 = stablehlo.add %249, %254 : tensor<512x512xf32>
    %256 = stablehlo.multiply %253, %104 : tensor<512x512xf32>
    %257 = stablehlo.add %255, %256 : tensor<512x512xf32>
    %258 = stablehlo.multiply %253, %104 : tensor<512x512xf32>
    %259 = stablehlo.add %257, %258 : tensor<512x512xf32>
    %260 = stablehlo.convert %259 : (tensor<512x512xf32>) -> tensor<512x512xbf16>
    %261 = stablehlo.reduce(%260 init: %cst_10) applies stablehlo.add across dimensions = [0] : (tensor<512x512xbf16>, tensor<bf16>) -> tensor<512xbf16>
    %262 = stablehlo.dot_general %260, %arg10, contracting_dims = [1] x [1], precision = [DEFAULT, DEFAULT] : (tensor<512x512xbf16>, tensor<128x512xbf16>) -> tensor<512x128xbf16>
    %263 = stablehlo.dot_general %100, %260, contracting_dims = [0] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<512x512xbf16>) -> tensor<128x512xbf16>
    %264 = stablehlo.convert %262 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %265 = stablehlo.reduce(%264 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<512x128xf32>, tensor<f32>) -> tensor<128xf32>
    %266 = stablehlo.convert %265 : (tensor<128xf32>) -> tensor<128xbf16>
    %267 = stablehlo.multiply %264, %95 : tensor<512x128xf32>
    %268 = stablehlo.multiply %264, %93 : tensor<512x128xf32>
    %269 = stablehlo.reduce(%268 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<512x128xf32>, tensor<f32>) -> tensor<128xf32>
    %270 = stablehlo.convert %269 : (tensor<128xf32>) -> tensor<128xbf16>
    %271 = stablehlo.multiply %267, %92 : tensor<512x128xf32>
    %272 = stablehlo.multiply %267, %82 : tensor<512x128xf32>
    %273 = stablehlo.reduce(%272 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %274 = stablehlo.reshape %273 : (tensor<512xf32>) -> tensor<512x1xf32>
    %275 = stablehlo.broadcast_in_dim %cst_9, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %276 = stablehlo.multiply %274, %275 : tensor<512x1xf32>
    %277 = stablehlo.multiply %276, %90 : tensor<512x1xf32>
    %278 = stablehlo.divide %277, %89 : tensor<512x1xf32>
    %280 = stablehlo.divide %278, %86 : tensor<512x1xf32>
    %285 = stablehlo.reshape %280 : (tensor<512x1xf32>) -> tensor<512xf32>
    %286 = stablehlo.broadcast_in_dim %285, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %287 = stablehlo.multiply %286, %82 : tensor<512x128xf32>
    %288 = stablehlo.add %271, %287 : tensor<512x128xf32>
    %289 = stablehlo.multiply %286, %82 : tensor<512x128xf32>
    %290 = stablehlo.add %288, %289 : tensor<512x128xf32>
    %291 = stablehlo.negate %290 : tensor<512x128xf32>
    %292 = stablehlo.reduce(%291 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %293 = stablehlo.reshape %292 : (tensor<512xf32>) -> tensor<512x1xf32>
    %294 = stablehlo.divide %293, %78 : tensor<512x1xf32>
    %299 = stablehlo.reshape %294 : (tensor<512x1xf32>) -> tensor<512xf32>
    %300 = stablehlo.broadcast_in_dim %299, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %301 = stablehlo.add %290, %300 : tensor<512x128xf32>
    %302 = stablehlo.convert %301 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %303 = stablehlo.add %231, %302 : tensor<512x128xbf16>
    %304 = stablehlo.reduce(%303 init: %cst_10) applies stablehlo.add across dimensions = [0] : (tensor<512x128xbf16>, tensor<bf16>) -> tensor<128xbf16>
    %305 = stablehlo.dot_general %303, %arg6, contracting_dims = [1] x [1], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<128x128xbf16>) -> tensor<512x128xbf16>
    %306 = stablehlo.dot_general %70, %303, contracting_dims = [0] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<512x128xbf16>) -> tensor<128x128xbf16>
    %307 = stablehlo.reshape %305 : (tensor<512x128xbf16>) -> tensor<2x256x2x64xbf16>
    %308 = stablehlo.transpose %307, dims = [0, 2, 1, 3] : (tensor<2x256x2x64xbf16>) -> tensor<2x2x256x64xbf16>
    %309 = stablehlo.dot_general %308, %46, batching_dims = [0, 1] x [0, 1], contracting_dims = [3] x [3], precision = [DEFAULT, DEFAULT] : (tensor<2x2x256x64xbf16>, tensor<2x2x256x64xbf16>) -> tensor<2x2x256x256xbf16>
    %310 = stablehlo.dot_general %67, %308, batching_dims = [0, 1] x [0, 1], contracting_dims = [2] x [2], precision = [DEFAULT, DEFAULT] : (tensor<2x2x256x256xbf16>, tensor<2x2x256x64xbf16>) -> tensor<2x2x256x64xbf16>
    %311 = stablehlo.convert %309 : (tensor<2x2x256x256xbf16>) -> tensor<2x2x256x256xf32>
    %312 = stablehlo.divide %311, %65 : tensor<2x2x256x256xf32>
    %313 = stablehlo.multiply %311, %66 : tensor<2x2x256x256xf32>
    %314 = stablehlo.negate %313 : tensor<2x2x256x256xf32>
    %315 = stablehlo.divide %314, %65 : tensor<2x2x256x256xf32>
    %316 = stablehlo.reduce(%315 init: %cst) applies stablehlo.add across dimensions = [3] : (tensor<2x2x256x256xf32>, tensor<f32>) -> tensor<2x2x256xf32>
    %317 = stablehlo.reshape %316 : (tensor<2x2x256xf32>) -> tensor<2x2x256x1xf32>
    %318 = stablehlo.reshape %317 : (tensor<2x2x256x1xf32>) -> tensor<2x2x256xf32>
    %319 = stablehlo.broadcast_in_dim %318, dims = [0, 1, 2] : (tensor<2x2x256xf32>) -> tensor<2x2x256x256xf32>
    %320 = stablehlo.add %312, %319 : tensor<2x2x256x256xf32>
    %321 = stablehlo.multiply %320, %61 : tensor<2x2x256x256xf32>
    %325 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<2x2x256x256xf32>
    %326 = stablehlo.select %53, %321, %325 : tensor<2x2x256x256xi1>, tensor<2x2x256x256xf32>
    %329 = stablehlo.multiply %326, %48 : tensor<2x2x256x256xf32>
    %332 = stablehlo.dot_general %329, %43, batching_dims = [0, 1] x [0, 1], contracting_dims = [3] x [2], precision = [DEFAULT, DEFAULT] : (tensor<2x2x256x256xf32>, tensor<2x2x256x64xbf16>) -> tensor<2x2x256x64xbf16>
    %333 = stablehlo.dot_general %40, %329, batching_dims = [0, 1] x [0, 1], contracting_dims = [2] x [2], precision = [DEFAULT, DEFAULT] : (tensor<2x2x256x64xbf16>, tensor<2x2x256x256xf32>) -> tensor<2x2x64x256xbf16>
    %334 = stablehlo.transpose %333, dims = [0, 1, 3, 2] : (tensor<2x2x64x256xbf16>) -> tensor<2x2x256x64xbf16>
    %335 = stablehlo.transpose %310, dims = [0, 2, 1, 3] : (tensor<2x2x256x64xbf16>) -> tensor<2x256x2x64xbf16>
    %336 = stablehlo.reshape %335 : (tensor<2x256x2x64xbf16>) -> tensor<512x128xbf16>
    %337 = stablehlo.pad %336, %cst_10, low = [0, 256], high = [0, 0], interior = [0, 0] : (tensor<512x128xbf16>, tensor<bf16>) -> tensor<512x384xbf16>
    %338 = stablehlo.transpose %334, dims = [0, 2, 1, 3] : (tensor<2x2x256x64xbf16>) -> tensor<2x256x2x64xbf16>
    %339 = stablehlo.reshape %338 : (tensor<2x256x2x64xbf16>) -> tensor<512x128xbf16>
    %340 = stablehlo.pad %339, %cst_10, low = [0, 128], high = [0, 128], interior = [0, 0] : (tensor<512x128xbf16>, tensor<bf16>) -> tensor<512x384xbf16>
    %341 = stablehlo.add %337, %340 : tensor<512x384xbf16>
    %342 = stablehlo.transpose %332, dims = [0, 2, 1, 3] : (tensor<2x2x256x64xbf16>) -> tensor<2x256x2x64xbf16>
    %343 = stablehlo.reshape %342 : (tensor<2x256x2x64xbf16>) -> tensor<512x128xbf16>
    %344 = stablehlo.pad %343, %cst_10, low = [0, 0], high = [0, 256], interior = [0, 0] : (tensor<512x128xbf16>, tensor<bf16>) -> tensor<512x384xbf16>
    %345 = stablehlo.add %341, %344 : tensor<512x384xbf16>
    %346 = stablehlo.reduce(%345 init: %cst_10) applies stablehlo.add across dimensions = [0] : (tensor<512x384xbf16>, tensor<bf16>) -> tensor<384xbf16>
    %347 = stablehlo.dot_general %345, %arg4, contracting_dims = [1] x [1], precision = [DEFAULT, DEFAULT] : (tensor<512x384xbf16>, tensor<128x384xbf16>) -> tensor<512x128xbf16>
    %348 = stablehlo.dot_general %34, %345, contracting_dims = [0] x [0], precision = [DEFAULT, DEFAULT] : (tensor<512x128xbf16>, tensor<512x384xbf16>) -> tensor<128x384xbf16>
    %349 = stablehlo.convert %347 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %350 = stablehlo.reduce(%349 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<512x128xf32>, tensor<f32>) -> tensor<128xf32>
    %351 = stablehlo.convert %350 : (tensor<128xf32>) -> tensor<128xbf16>
    %352 = stablehlo.multiply %349, %29 : tensor<512x128xf32>
    %353 = stablehlo.multiply %349, %27 : tensor<512x128xf32>
    %354 = stablehlo.reduce(%353 init: %cst) applies stablehlo.add across dimensions = [0] : (tensor<512x128xf32>, tensor<f32>) -> tensor<128xf32>
    %355 = stablehlo.convert %354 : (tensor<128xf32>) -> tensor<128xbf16>
    %356 = stablehlo.multiply %352, %26 : tensor<512x128xf32>
    %357 = stablehlo.multiply %352, %16 : tensor<512x128xf32>
    %358 = stablehlo.reduce(%357 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %359 = stablehlo.reshape %358 : (tensor<512xf32>) -> tensor<512x1xf32>
    %360 = stablehlo.broadcast_in_dim %cst_9, dims = [] : (tensor<f32>) -> tensor<512x1xf32>
    %361 = stablehlo.multiply %359, %360 : tensor<512x1xf32>
    %362 = stablehlo.multiply %361, %24 : tensor<512x1xf32>
    %363 = stablehlo.divide %362, %23 : tensor<512x1xf32>
    %365 = stablehlo.divide %363, %20 : tensor<512x1xf32>
    %370 = stablehlo.reshape %365 : (tensor<512x1xf32>) -> tensor<512xf32>
    %371 = stablehlo.broadcast_in_dim %370, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %372 = stablehlo.multiply %371, %16 : tensor<512x128xf32>
    %373 = stablehlo.add %356, %372 : tensor<512x128xf32>
    %374 = stablehlo.multiply %371, %16 : tensor<512x128xf32>
    %375 = stablehlo.add %373, %374 : tensor<512x128xf32>
    %376 = stablehlo.negate %375 : tensor<512x128xf32>
    %377 = stablehlo.reduce(%376 init: %cst) applies stablehlo.add across dimensions = [1] : (tensor<512x128xf32>, tensor<f32>) -> tensor<512xf32>
    %378 = stablehlo.reshape %377 : (tensor<512xf32>) -> tensor<512x1xf32>
    %379 = stablehlo.divide %378, %12 : tensor<512x1xf32>
    %384 = stablehlo.reshape %379 : (tensor<512x1xf32>) -> tensor<512xf32>
    %385 = stablehlo.broadcast_in_dim %384, dims = [0] : (tensor<512xf32>) -> tensor<512x128xf32>
    %386 = stablehlo.add %375, %385 : tensor<512x128xf32>
    %387 = stablehlo.convert %386 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %388 = stablehlo.add %303, %387 : tensor<512x128xbf16>
    %389 = stablehlo.reshape %388 : (tensor<512x128xbf16>) -> tensor<2x256x128xbf16>
    %390 = stablehlo.reduce(%389 init: %cst_10) applies stablehlo.add across dimensions = [0] : (tensor<2x256x128xbf16>, tensor<bf16>) -> tensor<256x128xbf16>
    %391 = stablehlo.broadcast_in_dim %cst_10, dims = [] : (tensor<bf16>) -> tensor<512x128xbf16>
    %392 = stablehlo.reshape %4 : (tensor<2x256x1xi32>) -> tensor<2x256xi32>
    %393 = stablehlo.reshape %392 : (tensor<2x256xi32>) -> tensor<2x256x1xi32>
    %394 = "stablehlo.scatter"(%391, %393, %389) <{indices_are_sorted = false, scatter_dimension_numbers = #stablehlo.scatter<update_window_dims = [2], inserted_window_dims = [0], scatter_dims_to_operand_dims = [0], index_vector_dim = 2>, unique_indices = false}> ({
      ^bb0(%a0: tensor<bf16>, %a1: tensor<bf16>):
        %s0 = stablehlo.add %a0, %a1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<512x128xbf16>, tensor<2x256x1xi32>, tensor<2x256x128xbf16>) -> tensor<512x128xbf16>
    %395 = stablehlo.add %192, %394 : tensor<512x128xbf16>
    %396 = "stablehlo.all_reduce"(%395) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<512x128xbf16>) -> tensor<512x128xbf16>
    %397 = stablehlo.convert %396 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %398 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %399 = stablehlo.multiply %397, %398 : tensor<512x128xf32>
    %cst_11 = stablehlo.constant dense<9.000000e-01> : tensor<f32>
    %400 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %401 = stablehlo.multiply %400, %arg16 : tensor<512x128xf32>
    %cst_12 = stablehlo.constant dense<1.000000e-01> : tensor<f32>
    %402 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %403 = stablehlo.multiply %402, %399 : tensor<512x128xf32>
    %404 = stablehlo.add %401, %403 : tensor<512x128xf32>
    %cst_13 = stablehlo.constant dense<9.500000e-01> : tensor<f32>
    %405 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %406 = stablehlo.multiply %405, %arg32 : tensor<512x128xf32>
    %407 = stablehlo.multiply %399, %399 : tensor<512x128xf32>
    %cst_14 = stablehlo.constant dense<5.000000e-02> : tensor<f32>
    %408 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %409 = stablehlo.multiply %408, %407 : tensor<512x128xf32>
    %410 = stablehlo.add %406, %409 : tensor<512x128xf32>
    %411 = stablehlo.convert %arg0 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %412 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %413 = stablehlo.divide %404, %412 : tensor<512x128xf32>
    %414 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %415 = stablehlo.divide %410, %414 : tensor<512x128xf32>
    %416 = stablehlo.sqrt %415 : tensor<512x128xf32>
    %cst_15 = stablehlo.constant dense<1.000000e-08> : tensor<f32>
    %417 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %418 = stablehlo.add %416, %417 : tensor<512x128xf32>
    %419 = stablehlo.divide %413, %418 : tensor<512x128xf32>
    %cst_16 = stablehlo.constant dense<1.000000e-01> : tensor<f32>
    %420 = stablehlo.broadcast_in_dim %cst_16, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %421 = stablehlo.multiply %420, %411 : tensor<512x128xf32>
    %422 = stablehlo.add %419, %421 : tensor<512x128xf32>
    %cst_17 = stablehlo.constant dense<3.000000e-04> : tensor<f32>
    %423 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %424 = stablehlo.multiply %423, %422 : tensor<512x128xf32>
    %425 = stablehlo.subtract %411, %424 : tensor<512x128xf32>
    %426 = stablehlo.convert %425 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %427 = "stablehlo.all_reduce"(%390) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<256x128xbf16>) -> tensor<256x128xbf16>
    %428 = stablehlo.convert %427 : (tensor<256x128xbf16>) -> tensor<256x128xf32>
    %429 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %430 = stablehlo.multiply %428, %429 : tensor<256x128xf32>
    %431 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %432 = stablehlo.multiply %431, %arg17 : tensor<256x128xf32>
    %433 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %434 = stablehlo.multiply %433, %430 : tensor<256x128xf32>
    %435 = stablehlo.add %432, %434 : tensor<256x128xf32>
    %436 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %437 = stablehlo.multiply %436, %arg33 : tensor<256x128xf32>
    %438 = stablehlo.multiply %430, %430 : tensor<256x128xf32>
    %439 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %440 = stablehlo.multiply %439, %438 : tensor<256x128xf32>
    %441 = stablehlo.add %437, %440 : tensor<256x128xf32>
    %442 = stablehlo.convert %arg1 : (tensor<256x128xbf16>) -> tensor<256x128xf32>
    %443 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %444 = stablehlo.divide %435, %443 : tensor<256x128xf32>
    %445 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %446 = stablehlo.divide %441, %445 : tensor<256x128xf32>
    %447 = stablehlo.sqrt %446 : tensor<256x128xf32>
    %448 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %449 = stablehlo.add %447, %448 : tensor<256x128xf32>
    %450 = stablehlo.divide %444, %449 : tensor<256x128xf32>
    %451 = stablehlo.broadcast_in_dim %cst_16, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %452 = stablehlo.multiply %451, %442 : tensor<256x128xf32>
    %453 = stablehlo.add %450, %452 : tensor<256x128xf32>
    %454 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<256x128xf32>
    %455 = stablehlo.multiply %454, %453 : tensor<256x128xf32>
    %456 = stablehlo.subtract %442, %455 : tensor<256x128xf32>
    %457 = stablehlo.convert %456 : (tensor<256x128xf32>) -> tensor<256x128xbf16>
    %458 = "stablehlo.all_reduce"(%355) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %459 = stablehlo.convert %458 : (tensor<128xbf16>) -> tensor<128xf32>
    %460 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %461 = stablehlo.multiply %459, %460 : tensor<128xf32>
    %462 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %463 = stablehlo.multiply %462, %arg18 : tensor<128xf32>
    %464 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %465 = stablehlo.multiply %464, %461 : tensor<128xf32>
    %466 = stablehlo.add %463, %465 : tensor<128xf32>
    %467 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %468 = stablehlo.multiply %467, %arg34 : tensor<128xf32>
    %469 = stablehlo.multiply %461, %461 : tensor<128xf32>
    %470 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %471 = stablehlo.multiply %470, %469 : tensor<128xf32>
    %472 = stablehlo.add %468, %471 : tensor<128xf32>
    %473 = stablehlo.convert %arg2 : (tensor<128xbf16>) -> tensor<128xf32>
    %474 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %475 = stablehlo.divide %466, %474 : tensor<128xf32>
    %476 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %477 = stablehlo.divide %472, %476 : tensor<128xf32>
    %478 = stablehlo.sqrt %477 : tensor<128xf32>
    %479 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %480 = stablehlo.add %478, %479 : tensor<128xf32>
    %481 = stablehlo.divide %475, %480 : tensor<128xf32>
    %482 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %483 = stablehlo.add %481, %482 : tensor<128xf32>
    %484 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %485 = stablehlo.multiply %484, %483 : tensor<128xf32>
    %486 = stablehlo.subtract %473, %485 : tensor<128xf32>
    %487 = stablehlo.convert %486 : (tensor<128xf32>) -> tensor<128xbf16>
    %488 = "stablehlo.all_reduce"(%351) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %489 = stablehlo.convert %488 : (tensor<128xbf16>) -> tensor<128xf32>
    %490 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %491 = stablehlo.multiply %489, %490 : tensor<128xf32>
    %492 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %493 = stablehlo.multiply %492, %arg19 : tensor<128xf32>
    %494 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %495 = stablehlo.multiply %494, %491 : tensor<128xf32>
    %496 = stablehlo.add %493, %495 : tensor<128xf32>
    %497 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %498 = stablehlo.multiply %497, %arg35 : tensor<128xf32>
    %499 = stablehlo.multiply %491, %491 : tensor<128xf32>
    %500 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %501 = stablehlo.multiply %500, %499 : tensor<128xf32>
    %502 = stablehlo.add %498, %501 : tensor<128xf32>
    %503 = stablehlo.convert %arg3 : (tensor<128xbf16>) -> tensor<128xf32>
    %504 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %505 = stablehlo.divide %496, %504 : tensor<128xf32>
    %506 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %507 = stablehlo.divide %502, %506 : tensor<128xf32>
    %508 = stablehlo.sqrt %507 : tensor<128xf32>
    %509 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %510 = stablehlo.add %508, %509 : tensor<128xf32>
    %511 = stablehlo.divide %505, %510 : tensor<128xf32>
    %512 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %513 = stablehlo.add %511, %512 : tensor<128xf32>
    %514 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %515 = stablehlo.multiply %514, %513 : tensor<128xf32>
    %516 = stablehlo.subtract %503, %515 : tensor<128xf32>
    %517 = stablehlo.convert %516 : (tensor<128xf32>) -> tensor<128xbf16>
    %518 = "stablehlo.all_reduce"(%348) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128x384xbf16>) -> tensor<128x384xbf16>
    %519 = stablehlo.convert %518 : (tensor<128x384xbf16>) -> tensor<128x384xf32>
    %520 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %521 = stablehlo.multiply %519, %520 : tensor<128x384xf32>
    %522 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %523 = stablehlo.multiply %522, %arg20 : tensor<128x384xf32>
    %524 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %525 = stablehlo.multiply %524, %521 : tensor<128x384xf32>
    %526 = stablehlo.add %523, %525 : tensor<128x384xf32>
    %527 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %528 = stablehlo.multiply %527, %arg36 : tensor<128x384xf32>
    %529 = stablehlo.multiply %521, %521 : tensor<128x384xf32>
    %530 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %531 = stablehlo.multiply %530, %529 : tensor<128x384xf32>
    %532 = stablehlo.add %528, %531 : tensor<128x384xf32>
    %533 = stablehlo.convert %arg4 : (tensor<128x384xbf16>) -> tensor<128x384xf32>
    %534 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %535 = stablehlo.divide %526, %534 : tensor<128x384xf32>
    %536 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %537 = stablehlo.divide %532, %536 : tensor<128x384xf32>
    %538 = stablehlo.sqrt %537 : tensor<128x384xf32>
    %539 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %540 = stablehlo.add %538, %539 : tensor<128x384xf32>
    %541 = stablehlo.divide %535, %540 : tensor<128x384xf32>
    %542 = stablehlo.broadcast_in_dim %cst_16, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %543 = stablehlo.multiply %542, %533 : tensor<128x384xf32>
    %544 = stablehlo.add %541, %543 : tensor<128x384xf32>
    %545 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128x384xf32>
    %546 = stablehlo.multiply %545, %544 : tensor<128x384xf32>
    %547 = stablehlo.subtract %533, %546 : tensor<128x384xf32>
    %548 = stablehlo.convert %547 : (tensor<128x384xf32>) -> tensor<128x384xbf16>
    %549 = "stablehlo.all_reduce"(%346) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<384xbf16>) -> tensor<384xbf16>
    %550 = stablehlo.convert %549 : (tensor<384xbf16>) -> tensor<384xf32>
    %551 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %552 = stablehlo.multiply %550, %551 : tensor<384xf32>
    %553 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %554 = stablehlo.multiply %553, %arg21 : tensor<384xf32>
    %555 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %556 = stablehlo.multiply %555, %552 : tensor<384xf32>
    %557 = stablehlo.add %554, %556 : tensor<384xf32>
    %558 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %559 = stablehlo.multiply %558, %arg37 : tensor<384xf32>
    %560 = stablehlo.multiply %552, %552 : tensor<384xf32>
    %561 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %562 = stablehlo.multiply %561, %560 : tensor<384xf32>
    %563 = stablehlo.add %559, %562 : tensor<384xf32>
    %564 = stablehlo.convert %arg5 : (tensor<384xbf16>) -> tensor<384xf32>
    %565 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %566 = stablehlo.divide %557, %565 : tensor<384xf32>
    %567 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %568 = stablehlo.divide %563, %567 : tensor<384xf32>
    %569 = stablehlo.sqrt %568 : tensor<384xf32>
    %570 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %571 = stablehlo.add %569, %570 : tensor<384xf32>
    %572 = stablehlo.divide %566, %571 : tensor<384xf32>
    %573 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %574 = stablehlo.add %572, %573 : tensor<384xf32>
    %575 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<384xf32>
    %576 = stablehlo.multiply %575, %574 : tensor<384xf32>
    %577 = stablehlo.subtract %564, %576 : tensor<384xf32>
    %578 = stablehlo.convert %577 : (tensor<384xf32>) -> tensor<384xbf16>
    %579 = "stablehlo.all_reduce"(%306) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128x128xbf16>) -> tensor<128x128xbf16>
    %580 = stablehlo.convert %579 : (tensor<128x128xbf16>) -> tensor<128x128xf32>
    %581 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %582 = stablehlo.multiply %580, %581 : tensor<128x128xf32>
    %583 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %584 = stablehlo.multiply %583, %arg22 : tensor<128x128xf32>
    %585 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %586 = stablehlo.multiply %585, %582 : tensor<128x128xf32>
    %587 = stablehlo.add %584, %586 : tensor<128x128xf32>
    %588 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %589 = stablehlo.multiply %588, %arg38 : tensor<128x128xf32>
    %590 = stablehlo.multiply %582, %582 : tensor<128x128xf32>
    %591 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %592 = stablehlo.multiply %591, %590 : tensor<128x128xf32>
    %593 = stablehlo.add %589, %592 : tensor<128x128xf32>
    %594 = stablehlo.convert %arg6 : (tensor<128x128xbf16>) -> tensor<128x128xf32>
    %595 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %596 = stablehlo.divide %587, %595 : tensor<128x128xf32>
    %597 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %598 = stablehlo.divide %593, %597 : tensor<128x128xf32>
    %599 = stablehlo.sqrt %598 : tensor<128x128xf32>
    %600 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %601 = stablehlo.add %599, %600 : tensor<128x128xf32>
    %602 = stablehlo.divide %596, %601 : tensor<128x128xf32>
    %603 = stablehlo.broadcast_in_dim %cst_16, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %604 = stablehlo.multiply %603, %594 : tensor<128x128xf32>
    %605 = stablehlo.add %602, %604 : tensor<128x128xf32>
    %606 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128x128xf32>
    %607 = stablehlo.multiply %606, %605 : tensor<128x128xf32>
    %608 = stablehlo.subtract %594, %607 : tensor<128x128xf32>
    %609 = stablehlo.convert %608 : (tensor<128x128xf32>) -> tensor<128x128xbf16>
    %610 = "stablehlo.all_reduce"(%304) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %611 = stablehlo.convert %610 : (tensor<128xbf16>) -> tensor<128xf32>
    %612 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %613 = stablehlo.multiply %611, %612 : tensor<128xf32>
    %614 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %615 = stablehlo.multiply %614, %arg23 : tensor<128xf32>
    %616 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %617 = stablehlo.multiply %616, %613 : tensor<128xf32>
    %618 = stablehlo.add %615, %617 : tensor<128xf32>
    %619 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %620 = stablehlo.multiply %619, %arg39 : tensor<128xf32>
    %621 = stablehlo.multiply %613, %613 : tensor<128xf32>
    %622 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %623 = stablehlo.multiply %622, %621 : tensor<128xf32>
    %624 = stablehlo.add %620, %623 : tensor<128xf32>
    %625 = stablehlo.convert %arg7 : (tensor<128xbf16>) -> tensor<128xf32>
    %626 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %627 = stablehlo.divide %618, %626 : tensor<128xf32>
    %628 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %629 = stablehlo.divide %624, %628 : tensor<128xf32>
    %630 = stablehlo.sqrt %629 : tensor<128xf32>
    %631 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %632 = stablehlo.add %630, %631 : tensor<128xf32>
    %633 = stablehlo.divide %627, %632 : tensor<128xf32>
    %634 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %635 = stablehlo.add %633, %634 : tensor<128xf32>
    %636 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %637 = stablehlo.multiply %636, %635 : tensor<128xf32>
    %638 = stablehlo.subtract %625, %637 : tensor<128xf32>
    %639 = stablehlo.convert %638 : (tensor<128xf32>) -> tensor<128xbf16>
    %640 = "stablehlo.all_reduce"(%270) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %641 = stablehlo.convert %640 : (tensor<128xbf16>) -> tensor<128xf32>
    %642 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %643 = stablehlo.multiply %641, %642 : tensor<128xf32>
    %644 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %645 = stablehlo.multiply %644, %arg24 : tensor<128xf32>
    %646 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %647 = stablehlo.multiply %646, %643 : tensor<128xf32>
    %648 = stablehlo.add %645, %647 : tensor<128xf32>
    %649 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %650 = stablehlo.multiply %649, %arg40 : tensor<128xf32>
    %651 = stablehlo.multiply %643, %643 : tensor<128xf32>
    %652 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %653 = stablehlo.multiply %652, %651 : tensor<128xf32>
    %654 = stablehlo.add %650, %653 : tensor<128xf32>
    %655 = stablehlo.convert %arg8 : (tensor<128xbf16>) -> tensor<128xf32>
    %656 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %657 = stablehlo.divide %648, %656 : tensor<128xf32>
    %658 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %659 = stablehlo.divide %654, %658 : tensor<128xf32>
    %660 = stablehlo.sqrt %659 : tensor<128xf32>
    %661 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %662 = stablehlo.add %660, %661 : tensor<128xf32>
    %663 = stablehlo.divide %657, %662 : tensor<128xf32>
    %664 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %665 = stablehlo.add %663, %664 : tensor<128xf32>
    %666 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %667 = stablehlo.multiply %666, %665 : tensor<128xf32>
    %668 = stablehlo.subtract %655, %667 : tensor<128xf32>
    %669 = stablehlo.convert %668 : (tensor<128xf32>) -> tensor<128xbf16>
    %670 = "stablehlo.all_reduce"(%266) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %671 = stablehlo.convert %670 : (tensor<128xbf16>) -> tensor<128xf32>
    %672 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %673 = stablehlo.multiply %671, %672 : tensor<128xf32>
    %674 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %675 = stablehlo.multiply %674, %arg25 : tensor<128xf32>
    %676 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %677 = stablehlo.multiply %676, %673 : tensor<128xf32>
    %678 = stablehlo.add %675, %677 : tensor<128xf32>
    %679 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %680 = stablehlo.multiply %679, %arg41 : tensor<128xf32>
    %681 = stablehlo.multiply %673, %673 : tensor<128xf32>
    %682 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %683 = stablehlo.multiply %682, %681 : tensor<128xf32>
    %684 = stablehlo.add %680, %683 : tensor<128xf32>
    %685 = stablehlo.convert %arg9 : (tensor<128xbf16>) -> tensor<128xf32>
    %686 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %687 = stablehlo.divide %678, %686 : tensor<128xf32>
    %688 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %689 = stablehlo.divide %684, %688 : tensor<128xf32>
    %690 = stablehlo.sqrt %689 : tensor<128xf32>
    %691 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %692 = stablehlo.add %690, %691 : tensor<128xf32>
    %693 = stablehlo.divide %687, %692 : tensor<128xf32>
    %694 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %695 = stablehlo.add %693, %694 : tensor<128xf32>
    %696 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %697 = stablehlo.multiply %696, %695 : tensor<128xf32>
    %698 = stablehlo.subtract %685, %697 : tensor<128xf32>
    %699 = stablehlo.convert %698 : (tensor<128xf32>) -> tensor<128xbf16>
    %700 = "stablehlo.all_reduce"(%263) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128x512xbf16>) -> tensor<128x512xbf16>
    %701 = stablehlo.convert %700 : (tensor<128x512xbf16>) -> tensor<128x512xf32>
    %702 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %703 = stablehlo.multiply %701, %702 : tensor<128x512xf32>
    %704 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %705 = stablehlo.multiply %704, %arg26 : tensor<128x512xf32>
    %706 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %707 = stablehlo.multiply %706, %703 : tensor<128x512xf32>
    %708 = stablehlo.add %705, %707 : tensor<128x512xf32>
    %709 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %710 = stablehlo.multiply %709, %arg42 : tensor<128x512xf32>
    %711 = stablehlo.multiply %703, %703 : tensor<128x512xf32>
    %712 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %713 = stablehlo.multiply %712, %711 : tensor<128x512xf32>
    %714 = stablehlo.add %710, %713 : tensor<128x512xf32>
    %715 = stablehlo.convert %arg10 : (tensor<128x512xbf16>) -> tensor<128x512xf32>
    %716 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %717 = stablehlo.divide %708, %716 : tensor<128x512xf32>
    %718 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %719 = stablehlo.divide %714, %718 : tensor<128x512xf32>
    %720 = stablehlo.sqrt %719 : tensor<128x512xf32>
    %721 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %722 = stablehlo.add %720, %721 : tensor<128x512xf32>
    %723 = stablehlo.divide %717, %722 : tensor<128x512xf32>
    %724 = stablehlo.broadcast_in_dim %cst_16, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %725 = stablehlo.multiply %724, %715 : tensor<128x512xf32>
    %726 = stablehlo.add %723, %725 : tensor<128x512xf32>
    %727 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128x512xf32>
    %728 = stablehlo.multiply %727, %726 : tensor<128x512xf32>
    %729 = stablehlo.subtract %715, %728 : tensor<128x512xf32>
    %730 = stablehlo.convert %729 : (tensor<128x512xf32>) -> tensor<128x512xbf16>
    %731 = "stablehlo.all_reduce"(%261) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<512xbf16>) -> tensor<512xbf16>
    %732 = stablehlo.convert %731 : (tensor<512xbf16>) -> tensor<512xf32>
    %733 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %734 = stablehlo.multiply %732, %733 : tensor<512xf32>
    %735 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %736 = stablehlo.multiply %735, %arg27 : tensor<512xf32>
    %737 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %738 = stablehlo.multiply %737, %734 : tensor<512xf32>
    %739 = stablehlo.add %736, %738 : tensor<512xf32>
    %740 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %741 = stablehlo.multiply %740, %arg43 : tensor<512xf32>
    %742 = stablehlo.multiply %734, %734 : tensor<512xf32>
    %743 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %744 = stablehlo.multiply %743, %742 : tensor<512xf32>
    %745 = stablehlo.add %741, %744 : tensor<512xf32>
    %746 = stablehlo.convert %arg11 : (tensor<512xbf16>) -> tensor<512xf32>
    %747 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %748 = stablehlo.divide %739, %747 : tensor<512xf32>
    %749 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %750 = stablehlo.divide %745, %749 : tensor<512xf32>
    %751 = stablehlo.sqrt %750 : tensor<512xf32>
    %752 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %753 = stablehlo.add %751, %752 : tensor<512xf32>
    %754 = stablehlo.divide %748, %753 : tensor<512xf32>
    %755 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %756 = stablehlo.add %754, %755 : tensor<512xf32>
    %757 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<512xf32>
    %758 = stablehlo.multiply %757, %756 : tensor<512xf32>
    %759 = stablehlo.subtract %746, %758 : tensor<512xf32>
    %760 = stablehlo.convert %759 : (tensor<512xf32>) -> tensor<512xbf16>
    %761 = "stablehlo.all_reduce"(%234) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<512x128xbf16>) -> tensor<512x128xbf16>
    %762 = stablehlo.convert %761 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %763 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %764 = stablehlo.multiply %762, %763 : tensor<512x128xf32>
    %765 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %766 = stablehlo.multiply %765, %arg28 : tensor<512x128xf32>
    %767 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %768 = stablehlo.multiply %767, %764 : tensor<512x128xf32>
    %769 = stablehlo.add %766, %768 : tensor<512x128xf32>
    %770 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %771 = stablehlo.multiply %770, %arg44 : tensor<512x128xf32>
    %772 = stablehlo.multiply %764, %764 : tensor<512x128xf32>
    %773 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %774 = stablehlo.multiply %773, %772 : tensor<512x128xf32>
    %775 = stablehlo.add %771, %774 : tensor<512x128xf32>
    %776 = stablehlo.convert %arg12 : (tensor<512x128xbf16>) -> tensor<512x128xf32>
    %777 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %778 = stablehlo.divide %769, %777 : tensor<512x128xf32>
    %779 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %780 = stablehlo.divide %775, %779 : tensor<512x128xf32>
    %781 = stablehlo.sqrt %780 : tensor<512x128xf32>
    %782 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %783 = stablehlo.add %781, %782 : tensor<512x128xf32>
    %784 = stablehlo.divide %778, %783 : tensor<512x128xf32>
    %785 = stablehlo.broadcast_in_dim %cst_16, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %786 = stablehlo.multiply %785, %776 : tensor<512x128xf32>
    %787 = stablehlo.add %784, %786 : tensor<512x128xf32>
    %788 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<512x128xf32>
    %789 = stablehlo.multiply %788, %787 : tensor<512x128xf32>
    %790 = stablehlo.subtract %776, %789 : tensor<512x128xf32>
    %791 = stablehlo.convert %790 : (tensor<512x128xf32>) -> tensor<512x128xbf16>
    %792 = "stablehlo.all_reduce"(%232) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %793 = stablehlo.convert %792 : (tensor<128xbf16>) -> tensor<128xf32>
    %794 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %795 = stablehlo.multiply %793, %794 : tensor<128xf32>
    %796 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %797 = stablehlo.multiply %796, %arg29 : tensor<128xf32>
    %798 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %799 = stablehlo.multiply %798, %795 : tensor<128xf32>
    %800 = stablehlo.add %797, %799 : tensor<128xf32>
    %801 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %802 = stablehlo.multiply %801, %arg45 : tensor<128xf32>
    %803 = stablehlo.multiply %795, %795 : tensor<128xf32>
    %804 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %805 = stablehlo.multiply %804, %803 : tensor<128xf32>
    %806 = stablehlo.add %802, %805 : tensor<128xf32>
    %807 = stablehlo.convert %arg13 : (tensor<128xbf16>) -> tensor<128xf32>
    %808 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %809 = stablehlo.divide %800, %808 : tensor<128xf32>
    %810 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %811 = stablehlo.divide %806, %810 : tensor<128xf32>
    %812 = stablehlo.sqrt %811 : tensor<128xf32>
    %813 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %814 = stablehlo.add %812, %813 : tensor<128xf32>
    %815 = stablehlo.divide %809, %814 : tensor<128xf32>
    %816 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %817 = stablehlo.add %815, %816 : tensor<128xf32>
    %818 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %819 = stablehlo.multiply %818, %817 : tensor<128xf32>
    %820 = stablehlo.subtract %807, %819 : tensor<128xf32>
    %821 = stablehlo.convert %820 : (tensor<128xf32>) -> tensor<128xbf16>
    %822 = "stablehlo.all_reduce"(%199) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %823 = stablehlo.convert %822 : (tensor<128xbf16>) -> tensor<128xf32>
    %824 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %825 = stablehlo.multiply %823, %824 : tensor<128xf32>
    %826 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %827 = stablehlo.multiply %826, %arg30 : tensor<128xf32>
    %828 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %829 = stablehlo.multiply %828, %825 : tensor<128xf32>
    %830 = stablehlo.add %827, %829 : tensor<128xf32>
    %831 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %832 = stablehlo.multiply %831, %arg46 : tensor<128xf32>
    %833 = stablehlo.multiply %825, %825 : tensor<128xf32>
    %834 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %835 = stablehlo.multiply %834, %833 : tensor<128xf32>
    %836 = stablehlo.add %832, %835 : tensor<128xf32>
    %837 = stablehlo.convert %arg14 : (tensor<128xbf16>) -> tensor<128xf32>
    %838 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %839 = stablehlo.divide %830, %838 : tensor<128xf32>
    %840 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %841 = stablehlo.divide %836, %840 : tensor<128xf32>
    %842 = stablehlo.sqrt %841 : tensor<128xf32>
    %843 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %844 = stablehlo.add %842, %843 : tensor<128xf32>
    %845 = stablehlo.divide %839, %844 : tensor<128xf32>
    %846 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %847 = stablehlo.add %845, %846 : tensor<128xf32>
    %848 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %849 = stablehlo.multiply %848, %847 : tensor<128xf32>
    %850 = stablehlo.subtract %837, %849 : tensor<128xf32>
    %851 = stablehlo.convert %850 : (tensor<128xf32>) -> tensor<128xbf16>
    %852 = "stablehlo.all_reduce"(%195) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<bf16>, %r1: tensor<bf16>):
        %s0 = stablehlo.add %r0, %r1 : tensor<bf16>
        stablehlo.return %s0 : tensor<bf16>
      }) : (tensor<128xbf16>) -> tensor<128xbf16>
    %853 = stablehlo.convert %852 : (tensor<128xbf16>) -> tensor<128xf32>
    %854 = stablehlo.broadcast_in_dim %cst_6, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %855 = stablehlo.multiply %853, %854 : tensor<128xf32>
    %856 = stablehlo.broadcast_in_dim %cst_11, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %857 = stablehlo.multiply %856, %arg31 : tensor<128xf32>
    %858 = stablehlo.broadcast_in_dim %cst_12, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %859 = stablehlo.multiply %858, %855 : tensor<128xf32>
    %860 = stablehlo.add %857, %859 : tensor<128xf32>
    %861 = stablehlo.broadcast_in_dim %cst_13, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %862 = stablehlo.multiply %861, %arg47 : tensor<128xf32>
    %863 = stablehlo.multiply %855, %855 : tensor<128xf32>
    %864 = stablehlo.broadcast_in_dim %cst_14, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %865 = stablehlo.multiply %864, %863 : tensor<128xf32>
    %866 = stablehlo.add %862, %865 : tensor<128xf32>
    %867 = stablehlo.convert %arg15 : (tensor<128xbf16>) -> tensor<128xf32>
    %868 = stablehlo.broadcast_in_dim %arg50, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %869 = stablehlo.divide %860, %868 : tensor<128xf32>
    %870 = stablehlo.broadcast_in_dim %arg51, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %871 = stablehlo.divide %866, %870 : tensor<128xf32>
    %872 = stablehlo.sqrt %871 : tensor<128xf32>
    %873 = stablehlo.broadcast_in_dim %cst_15, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %874 = stablehlo.add %872, %873 : tensor<128xf32>
    %875 = stablehlo.divide %869, %874 : tensor<128xf32>
    %876 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %877 = stablehlo.add %875, %876 : tensor<128xf32>
    %878 = stablehlo.broadcast_in_dim %cst_17, dims = [] : (tensor<f32>) -> tensor<128xf32>
    %879 = stablehlo.multiply %878, %877 : tensor<128xf32>
    %880 = stablehlo.subtract %867, %879 : tensor<128xf32>
    %881 = stablehlo.convert %880 : (tensor<128xf32>) -> tensor<128xbf16>
    %882 = "stablehlo.all_reduce"(%169) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<f32>, %r1: tensor<f32>):
        %s0 = stablehlo.add %r0, %r1 : tensor<f32>
        stablehlo.return %s0 : tensor<f32>
      }) : (tensor<f32>) -> tensor<f32>
    %883 = stablehlo.multiply %882, %cst_6 : tensor<f32>
    return %426, %457, %487, %517, %548, %578, %609, %639, %669, %699, %730, %760, %791, %821, %851, %881, %404, %435, %466, %496, %526, %557, %587, %618, %648, %678, %708, %739, %769, %800, %830, %860, %410, %441, %472, %502, %532, %563, %593, %624, %654, %684, %714, %745, %775, %806, %836, %866, %883 : tensor<512x128xbf16>, tensor<256x128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128x384xbf16>, tensor<384xbf16>, tensor<128x128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128x512xbf16>, tensor<512xbf16>, tensor<512x128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<128xbf16>, tensor<512x128xf32>, tensor<256x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x384xf32>, tensor<384xf32>, tensor<128x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x512xf32>, tensor<512xf32>, tensor<512x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<512x128xf32>, tensor<256x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x384xf32>, tensor<384xf32>, tensor<128x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128x512xf32>, tensor<512xf32>, tensor<512x128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<128xf32>, tensor<f32>
  }
}
