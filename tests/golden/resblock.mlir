module {
  func.func @forward(%arg0: tensor<2x8x12x12xf32>, %arg1: tensor<16x8x3x3xf32>, %arg2: tensor<16xf32>, %arg3: tensor<16x16x3x3xf32>, %arg4: tensor<16xf32>, %arg5: tensor<16x8x1x1xf32>, %arg6: tensor<16xf32>) -> (tensor<2x16x6x6xf32>, tensor<2x16x1x1xf32>) attributes {gawee.onnx_source = "golden:resblock"} {
    %0 = "gawee.max_pool"(%arg0) <{ceilMode = false, dilation = array<i64: 1, 1>, kernelSize = array<i64: 3, 3>, padding = array<i64: 1, 1>, strides = array<i64: 1, 1>}> : (tensor<2x8x12x12xf32>) -> tensor<2x8x12x12xf32>
    %1 = "gawee.conv"(%0, %arg1, %arg2) <{dilation = array<i64: 1, 1>, padding = array<i64: 1, 1>, strides = array<i64: 2, 2>}> : (tensor<2x8x12x12xf32>, tensor<16x8x3x3xf32>, tensor<16xf32>) -> tensor<2x16x6x6xf32>
    %2 = "gawee.relu"(%1) : (tensor<2x16x6x6xf32>) -> tensor<2x16x6x6xf32>
    %3 = "gawee.conv"(%2, %arg3, %arg4) <{dilation = array<i64: 1, 1>, padding = array<i64: 1, 1>, strides = array<i64: 1, 1>}> : (tensor<2x16x6x6xf32>, tensor<16x16x3x3xf32>, tensor<16xf32>) -> tensor<2x16x6x6xf32>
    %4 = "gawee.conv"(%0, %arg5, %arg6) <{dilation = array<i64: 1, 1>, padding = array<i64: 0, 0>, strides = array<i64: 2, 2>}> : (tensor<2x8x12x12xf32>, tensor<16x8x1x1xf32>, tensor<16xf32>) -> tensor<2x16x6x6xf32>
    %5 = "gawee.add"(%3, %4) : (tensor<2x16x6x6xf32>, tensor<2x16x6x6xf32>) -> tensor<2x16x6x6xf32>
    %6 = "gawee.relu"(%5) : (tensor<2x16x6x6xf32>) -> tensor<2x16x6x6xf32>
    %7 = "gawee.global_average_pool"(%6) : (tensor<2x16x6x6xf32>) -> tensor<2x16x1x1xf32>
    return %6, %7 : tensor<2x16x6x6xf32>, tensor<2x16x1x1xf32>
  }
}
