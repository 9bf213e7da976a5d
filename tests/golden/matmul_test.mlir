module {
  func.func @forward(%arg0: tensor<2x4xf32>, %arg1: tensor<4x3xf32>, %arg2: tensor<1x2x3x4xf32>, %arg3: tensor<1x2x4x5xf32>) -> (tensor<2x3xf32>, tensor<1x2x3x5xf32>) attributes {gawee.onnx_source = "golden:matmul"} {
    %0 = "gawee.matmul"(%arg0, %arg1) : (tensor<2x4xf32>, tensor<4x3xf32>) -> tensor<2x3xf32>
    %1 = "gawee.matmul"(%arg2, %arg3) : (tensor<1x2x3x4xf32>, tensor<1x2x4x5xf32>) -> tensor<1x2x3x5xf32>
    return %0, %1 : tensor<2x3xf32>, tensor<1x2x3x5xf32>
  }
}
