#map = affine_map<(d0, d1, d2) -> (d0, d1, d2)>
#map1 = affine_map<(d0, d1, d2) -> ()>
#map2 = affine_map<(d0, d1) -> (0, d1)>
#map3 = affine_map<(d0, d1) -> (d0, 0)>
#map4 = affine_map<(d0, d1) -> (d0, d1)>
module {
  func.func @forward(%arg0: tensor<1x16x32xf32>, %arg1: tensor<32x32xf32>, %arg2: tensor<32x32xf32>, %arg3: tensor<32x32xf32>) -> (tensor<1x16x32xf32>, tensor<1x16x32xf32>) attributes {gawee.onnx_source = "golden:attention"} {
    %0 = "gawee.reduce_mean"(%arg0) <{axes = array<i64: -1>, keepDims = true}> : (tensor<1x16x32xf32>) -> tensor<1x16x1xf32>
    %1 = "gawee.sub"(%arg0, %0) : (tensor<1x16x32xf32>, tensor<1x16x1xf32>) -> tensor<1x16x32xf32>
    %cst = arith.constant dense<2.000000e+00> : tensor<f32>
    %2 = tensor.empty() : tensor<1x16x32xf32>
    %3 = linalg.generic {indexing_maps = [#map, #map1, #map], iterator_types = ["parallel", "parallel", "parallel"]} ins(%1, %cst : tensor<1x16x32xf32>, tensor<f32>) outs(%2 : tensor<1x16x32xf32>) {
    ^bb0(%in: f32, %in_0: f32, %out: f32):
      %r = math.powf %in, %in_0 : f32
      linalg.yield %r : f32
    } -> tensor<1x16x32xf32>
    %4 = "gawee.reduce_mean"(%3) <{axes = array<i64: -1>, keepDims = true}> : (tensor<1x16x32xf32>) -> tensor<1x16x1xf32>
    %cst_0 = arith.constant dense<1.000000e-12> : tensor<f32>
    %5 = "gawee.add"(%4, %cst_0) : (tensor<1x16x1xf32>, tensor<f32>) -> tensor<1x16x1xf32>
    %6 = "gawee.sqrt"(%5) : (tensor<1x16x1xf32>) -> tensor<1x16x1xf32>
    %7 = "gawee.div"(%1, %6) : (tensor<1x16x32xf32>, tensor<1x16x1xf32>) -> tensor<1x16x32xf32>
    %8 = "gawee.matmul"(%7, %arg1) : (tensor<1x16x32xf32>, tensor<32x32xf32>) -> tensor<1x16x32xf32>
    %cst_1 = arith.constant dense<[1, 16, 2, 16]> : tensor<4xi64>
    %9 = "gawee.reshape"(%8, %cst_1) : (tensor<1x16x32xf32>, tensor<4xi64>) -> tensor<1x16x2x16xf32>
    %10 = "gawee.transpose"(%9) <{perm = array<i64: 0, 2, 1, 3>}> : (tensor<1x16x2x16xf32>) -> tensor<1x2x16x16xf32>
    %11 = "gawee.matmul"(%7, %arg2) : (tensor<1x16x32xf32>, tensor<32x32xf32>) -> tensor<1x16x32xf32>
    %cst_2 = arith.constant dense<[1, 16, 2, 16]> : tensor<4xi64>
    %12 = "gawee.reshape"(%11, %cst_2) : (tensor<1x16x32xf32>, tensor<4xi64>) -> tensor<1x16x2x16xf32>
    %13 = "gawee.transpose"(%12) <{perm = array<i64: 0, 2, 3, 1>}> : (tensor<1x16x2x16xf32>) -> tensor<1x2x16x16xf32>
    %14 = "gawee.matmul"(%7, %arg3) : (tensor<1x16x32xf32>, tensor<32x32xf32>) -> tensor<1x16x32xf32>
    %cst_3 = arith.constant dense<[1, 16, 2, 16]> : tensor<4xi64>
    %15 = "gawee.reshape"(%14, %cst_3) : (tensor<1x16x32xf32>, tensor<4xi64>) -> tensor<1x16x2x16xf32>
    %16 = "gawee.transpose"(%15) <{perm = array<i64: 0, 2, 1, 3>}> : (tensor<1x16x2x16xf32>) -> tensor<1x2x16x16xf32>
    %cst_4 = arith.constant dense<0> : tensor<i64>
    %cst_5 = arith.constant dense<16> : tensor<i64>
    %cst_6 = arith.constant dense<1> : tensor<i64>
    %17 = "gawee.range"(%cst_4, %cst_5, %cst_6) : (tensor<i64>, tensor<i64>, tensor<i64>) -> tensor<16xi64>
    %18 = "gawee.unsqueeze"(%17) <{axes = array<i64: 0>}> : (tensor<16xi64>) -> tensor<1x16xi64>
    %19 = "gawee.unsqueeze"(%17) <{axes = array<i64: 1>}> : (tensor<16xi64>) -> tensor<16x1xi64>
    %20 = tensor.empty() : tensor<16x16xi1>
    %21 = linalg.generic {indexing_maps = [#map2, #map3, #map4], iterator_types = ["parallel", "parallel"]} ins(%18, %19 : tensor<1x16xi64>, tensor<16x1xi64>) outs(%20 : tensor<16x16xi1>) {
    ^bb0(%in: i64, %in_0: i64, %out: i1):
      %r = arith.cmpi sle, %in, %in_0 : i64
      linalg.yield %r : i1
    } -> tensor<16x16xi1>
    %cst_7 = arith.constant dense<0.000000e+00> : tensor<f32>
    %cst_8 = arith.constant dense<0xFF800000> : tensor<f32>
    %22 = "gawee.where"(%21, %cst_7, %cst_8) : (tensor<16x16xi1>, tensor<f32>, tensor<f32>) -> tensor<16x16xf32>
    %23 = "gawee.matmul"(%10, %13) : (tensor<1x2x16x16xf32>, tensor<1x2x16x16xf32>) -> tensor<1x2x16x16xf32>
    %cst_9 = arith.constant dense<4.000000e+00> : tensor<f32>
    %24 = "gawee.div"(%23, %cst_9) : (tensor<1x2x16x16xf32>, tensor<f32>) -> tensor<1x2x16x16xf32>
    %25 = "gawee.add"(%24, %22) : (tensor<1x2x16x16xf32>, tensor<16x16xf32>) -> tensor<1x2x16x16xf32>
    %26 = "gawee.softmax"(%25) <{axis = 3 : i64}> : (tensor<1x2x16x16xf32>) -> tensor<1x2x16x16xf32>
    %27 = "gawee.matmul"(%26, %16) : (tensor<1x2x16x16xf32>, tensor<1x2x16x16xf32>) -> tensor<1x2x16x16xf32>
    %28 = "gawee.transpose"(%27) <{perm = array<i64: 0, 2, 1, 3>}> : (tensor<1x2x16x16xf32>) -> tensor<1x16x2x16xf32>
    %cst_10 = arith.constant dense<[1, 16, 32]> : tensor<3xi64>
    %29 = "gawee.reshape"(%28, %cst_10) : (tensor<1x16x2x16xf32>, tensor<3xi64>) -> tensor<1x16x32xf32>
    %30 = "gawee.gelu"(%29) : (tensor<1x16x32xf32>) -> tensor<1x16x32xf32>
    return %29, %30 : tensor<1x16x32xf32>, tensor<1x16x32xf32>
  }
}
