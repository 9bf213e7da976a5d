#map = affine_map<(d0, d1, d2) -> (d0, d1, d2)>
#map1 = affine_map<(d0, d1) -> (d0, d1)>
module {
  func.func @forward(%arg0: tensor<2x6xi64>, %arg1: tensor<40x8xf32>) -> tensor<2x6x8xf32> attributes {gawee.onnx_source = "golden:rope"} {
    %0 = "gawee.gather"(%arg1, %arg0) <{axis = 0 : i64}> : (tensor<40x8xf32>, tensor<2x6xi64>) -> tensor<2x6x8xf32>
    %cst = arith.constant dense<0> : tensor<i64>
    %cst_0 = arith.constant dense<6> : tensor<i64>
    %cst_1 = arith.constant dense<1> : tensor<i64>
    %1 = "gawee.range"(%cst, %cst_0, %cst_1) : (tensor<i64>, tensor<i64>, tensor<i64>) -> tensor<6xi64>
    %2 = "gawee.unsqueeze"(%1) <{axes = array<i64: 1>}> : (tensor<6xi64>) -> tensor<6x1xi64>
    %3 = "gawee.cast"(%2) <{toType = 1 : i64}> : (tensor<6x1xi64>) -> tensor<6x1xf32>
    %cst_2 = arith.constant dense<7.000000e-01> : tensor<1x8xf32>
    %4 = "gawee.mul"(%3, %cst_2) : (tensor<6x1xf32>, tensor<1x8xf32>) -> tensor<6x8xf32>
    %cst_3 = arith.constant dense<0> : tensor<1xi64>
    %cst_4 = arith.constant dense<4> : tensor<1xi64>
    %cst_5 = arith.constant dense<2> : tensor<1xi64>
    %cst_6 = arith.constant dense<1> : tensor<1xi64>
    %5 = "gawee.slice"(%0, %cst_3, %cst_4, %cst_5, %cst_6) : (tensor<2x6x8xf32>, tensor<1xi64>, tensor<1xi64>, tensor<1xi64>, tensor<1xi64>) -> tensor<2x6x4xf32>
    %cst_7 = arith.constant dense<4> : tensor<1xi64>
    %cst_8 = arith.constant dense<8> : tensor<1xi64>
    %cst_9 = arith.constant dense<2> : tensor<1xi64>
    %cst_10 = arith.constant dense<1> : tensor<1xi64>
    %6 = "gawee.slice"(%0, %cst_7, %cst_8, %cst_9, %cst_10) : (tensor<2x6x8xf32>, tensor<1xi64>, tensor<1xi64>, tensor<1xi64>, tensor<1xi64>) -> tensor<2x6x4xf32>
    %7 = tensor.empty() : tensor<2x6x4xf32>
    %8 = linalg.generic {indexing_maps = [#map, #map], iterator_types = ["parallel", "parallel", "parallel"]} ins(%6 : tensor<2x6x4xf32>) outs(%7 : tensor<2x6x4xf32>) {
    ^bb0(%in: f32, %out: f32):
      %r = arith.negf %in : f32
      linalg.yield %r : f32
    } -> tensor<2x6x4xf32>
    %9 = "gawee.cat"(%8, %5) <{axis = 2 : i64}> : (tensor<2x6x4xf32>, tensor<2x6x4xf32>) -> tensor<2x6x8xf32>
    %10 = tensor.empty() : tensor<6x8xf32>
    %11 = linalg.generic {indexing_maps = [#map1, #map1], iterator_types = ["parallel", "parallel"]} ins(%4 : tensor<6x8xf32>) outs(%10 : tensor<6x8xf32>) {
    ^bb0(%in: f32, %out: f32):
      %r = math.cos %in : f32
      linalg.yield %r : f32
    } -> tensor<6x8xf32>
    %12 = "gawee.mul"(%0, %11) : (tensor<2x6x8xf32>, tensor<6x8xf32>) -> tensor<2x6x8xf32>
    %13 = tensor.empty() : tensor<6x8xf32>
    %14 = linalg.generic {indexing_maps = [#map1, #map1], iterator_types = ["parallel", "parallel"]} ins(%4 : tensor<6x8xf32>) outs(%13 : tensor<6x8xf32>) {
    ^bb0(%in: f32, %out: f32):
      %r = math.sin %in : f32
      linalg.yield %r : f32
    } -> tensor<6x8xf32>
    %15 = "gawee.mul"(%9, %14) : (tensor<2x6x8xf32>, tensor<6x8xf32>) -> tensor<2x6x8xf32>
    %16 = "gawee.add"(%12, %15) : (tensor<2x6x8xf32>, tensor<2x6x8xf32>) -> tensor<2x6x8xf32>
    return %16 : tensor<2x6x8xf32>
  }
}
