module {
  func.func @forward(%arg0: tensor<2x3xf32>, %arg1: tensor<2x3xf32>, %arg2: tensor<1x3x32x32xf32>, %arg3: tensor<16x3x3x3xf32>, %arg4: tensor<16xf32>) -> (tensor<2x3xf32>, tensor<2x3xf32>, tensor<1x16x30x30xf32>) attributes {gawee.onnx_source = "golden:simple"} {
    %0 = "gawee.conv"(%arg2, %arg3, %arg4) <{dilation = array<i64: 1, 1>, padding = array<i64: 0, 0>, strides = array<i64: 1, 1>}> : (tensor<1x3x32x32xf32>, tensor<16x3x3x3xf32>, tensor<16xf32>) -> tensor<1x16x30x30xf32>
    %1 = "gawee.add"(%arg0, %arg1) : (tensor<2x3xf32>, tensor<2x3xf32>) -> tensor<2x3xf32>
    %2 = "gawee.relu"(%arg0) : (tensor<2x3xf32>) -> tensor<2x3xf32>
    return %1, %2, %0 : tensor<2x3xf32>, tensor<2x3xf32>, tensor<1x16x30x30xf32>
  }
}
