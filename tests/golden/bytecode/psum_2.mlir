module @jit_psum attributes {mhlo.num_partitions = 2 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<2048xf32>) -> (tensor<2048xf32>) {
    %0 = stablehlo.custom_call @Sharding(%arg0) {mhlo.sharding = "{devices=[2,1]<=[2]}"} : (tensor<2048xf32>) -> tensor<2048xf32>
    %1 = stablehlo.custom_call @SPMDFullToShardShape(%0) {mhlo.sharding = "{manual}"} : (tensor<2048xf32>) -> tensor<1024xf32>
    %2 = "stablehlo.all_reduce"(%1) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, use_global_device_ids}> ({
      ^bb0(%r0: tensor<f32>, %r1: tensor<f32>):
        %s0 = stablehlo.add %r0, %r1 : tensor<f32>
        stablehlo.return %s0 : tensor<f32>
      }) : (tensor<1024xf32>) -> tensor<1024xf32>
    %3 = stablehlo.custom_call @Sharding(%2) {mhlo.sharding = "{manual}"} : (tensor<1024xf32>) -> tensor<1024xf32>
    %4 = stablehlo.custom_call @SPMDShardToFullShape(%3) {mhlo.sharding = "{replicated}"} : (tensor<1024xf32>) -> tensor<2048xf32>
    return %4 : tensor<2048xf32>
  }
}
