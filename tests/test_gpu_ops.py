"""Per-op parity of the CUDA backend against the CPU oracle (small and odd shapes)."""
import math

import numpy as np
import pytest

from tests.helpers import _arr, build, parity, rand_input

pytestmark = pytest.mark.gpu

F = "f32"


def test_binary_broadcast_and_ints():
    def g_(g):
        a = rand_input(g, (2, 3, 5, 7), 1)
        b = rand_input(g, (3, 1, 7), 2)
        c = rand_input(g, (1,), 3)
        i = rand_input(g, (4, 5), 4, dtype="i64", lo=-50, hi=50)
        j = rand_input(g, (5,), 5, dtype="i64", lo=1, hi=9)
        return [g.add(a, b), g.sub(b, a), g.mul(a, c), g.div(a, g.add(g.mul(b, b), c)),
                g.add(i, j), g.op("div", [i, j], None, "i64", (4, 5)), g.op("mul", [i, j], None, "i64", (4, 5))]
    parity(*build(g_))


@pytest.mark.parametrize("cols", [4, 5, 7, 64, 577])
def test_elementwise_rows_path(cols):
    """f32 elementwise ops whose output rows are contiguous take the row-run
    kernel: full, row-broadcast ([rows,1]), column-broadcast ([cols]) and
    transposed (inner stride != 1) operands, ragged row tails; IEEE add/mul/div
    are exact, so the result must equal the oracle bit for bit."""
    rows = 37

    def g_(g):
        x = rand_input(g, (2, rows, cols), 11)
        r = rand_input(g, (2, rows, 1), 12)
        w = rand_input(g, (cols,), 13)
        t = rand_input(g, (2, cols, rows), 14)
        tt = g.transpose(t, (0, 2, 1))
        y = g.mul(g.div(x, g.add(g.mul(r, r), r)), w)
        return [y, g.add(x, tt), g.sub(g.mul(x, r), w)]
    parity(*build(g_), atol=0.0, rtol=0.0)


def test_elementwise_fast_forms():
    """Programs the host recognises and the kernels evaluate without the
    interpreter: negate, square (x * x and powf(x, 2)), sqrt(x + eps),
    x / r * w with broadcast operands, a*b + c*d.  Dense operands take the
    flat float4 kernel, broadcast ones the row-run kernel.  All are IEEE
    single operations and match the oracle bit for bit, except powf(x, 2):
    the device evaluates it as the correctly rounded x * x, while the
    oracle calls libm powf (as the reference's lowering does), which can
    be one ulp away; hence the two-ulp relative bound."""
    def g_(g):
        x = rand_input(g, (2, 37, 64), 41)
        y = rand_input(g, (2, 37, 64), 42)
        r = rand_input(g, (2, 37, 1), 43)
        w = rand_input(g, (64,), 44)
        m = g.mul(rand_input(g, (2, 37, 6), 45), rand_input(g, (2, 37, 6), 46))
        # m is also an output, so sqrt(m + eps) stays a program of its own
        return [m, g.neg(x), g.mul(y, y), g.pow(x, g.const(2.0, F)),
                g.sqrt(g.add(m, g.const(1e-5, F))),
                g.mul(g.div(x, r), w),
                g.add(g.mul(x, y), g.mul(rand_input(g, (2, 37, 64), 47), w))]
    parity(*build(g_), atol=0.0, rtol=2.4e-7)


def test_unary_activations():
    def g_(g):
        x = rand_input(g, (3, 37, 11), 7, scale=3.0)
        outs = [g.relu(x), g.sigmoid(x), g.erf(x), g.op("tanh", [x], None, F, x.shape),
                g.op("gelu", [x], None, F, x.shape), g.sqrt(g.mul(x, x)),
                g.op("hard_sigmoid", [x], {"alpha": "2.000000e-01 : f64", "beta": "5.000000e-01 : f64"}, F, x.shape),
                g.op("hard_swish", [x], None, F, x.shape),
                g.op("leaky_relu", [x], {"alpha": "0.0099999997764825821 : f64"}, F, x.shape)]
        return outs
    parity(*build(g_), atol=2e-6, rtol=2e-6)


def test_relu_nan_and_signed_zero():
    def g_(g):
        x = g.input(F, (8,), lambda: np.array([-0.0, 0.0, -1.0, 2.0, np.nan, -np.inf, np.inf, -3.5], np.float32))
        return [g.relu(x)]
    got, want = parity(*build(g_))
    assert np.array_equal(np.signbit(got[0]), np.signbit(want[0]))


def test_compare_where_cast_maxmin():
    def g_(g):
        a = rand_input(g, (4, 6), 11)
        b = rand_input(g, (6,), 12)
        i = rand_input(g, (4, 6), 13, dtype="i64", lo=-3, hi=3)
        eq = g.op("equal", [i, g.const(0, "i64")], None, "i1", (4, 6))
        w = g.where(eq, a, g.mul(b, g.const(2.0, F)))
        c1 = g.cast(eq, 1, F)
        c2 = g.cast(g.mul(a, g.const(7.5, F)), 7, "i64")
        c3 = g.cast(i, 1, F)
        mx = g.op("max", [a, b, g.const(0.25, F)], None, F, (4, 6))
        mn = g.op("min", [a, b], None, F, (4, 6))
        return [w, c1, c2, c3, mx, mn, eq]
    parity(*build(g_))


@pytest.mark.parametrize("axes,keep", [([-1], True), ([1], False), ([0, 2], True), ([0, 1, 2], False)])
def test_reduce_mean_sum(axes, keep):
    def g_(g):
        x = rand_input(g, (5, 33, 130), 21)
        m = g.reduce_mean(x, axes, keep)
        shape = list(m.shape)
        s = g.op("reduce_sum", [x], {"axes": _arr(axes), "keepDims": "true" if keep else "false"}, F, tuple(shape))
        return [m, s]
    # sums of up to 21450 terms: fp32 summation order differs (tree vs sequential)
    parity(*build(g_), atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("shape,axis", [((3, 5, 17), -1), ((2, 3, 4, 1500), -1), ((3, 9, 4), 1)])
def test_softmax(shape, axis):
    def g_(g):
        x = rand_input(g, shape, 31, scale=4.0)
        return [g.softmax(x, axis)]
    parity(*build(g_), atol=1e-6, rtol=1e-5)


def test_gather_and_gather_elements():
    def g_(g):
        tab = rand_input(g, (50, 12), 41)
        ids = rand_input(g, (2, 7), 42, dtype="i64", lo=0, hi=50)
        x = rand_input(g, (4, 9, 3), 43)
        idx1 = g.const(np.array([8, 0, 3], np.int64), "i64")
        ge_idx = rand_input(g, (4, 5, 3), 44, dtype="i64", lo=0, hi=9)
        return [g.gather(tab, ids, 0), g.gather(x, idx1, 1),
                g.op("gather_elements", [x, ge_idx], {"axis": "1 : i64"}, F, (4, 5, 3))]
    parity(*build(g_))


def test_layout_views_and_copies():
    def g_(g):
        x = rand_input(g, (2, 6, 5, 4), 51)
        t = g.transpose(x, [0, 2, 3, 1])
        r = g.reshape(t, (2, 20, 6))            # needs a copy (transposed source)
        s = g.slice(x, [-5, 1], [6, 5], [1, 2], [2, 2])
        u = g.unsqueeze(s, [0])
        c = g.cat([x, g.mul(x, g.const(3.0, F))], 1)
        e = g.expand(rand_input(g, (1, 6, 1, 4), 52), (2, 6, 5, 4))
        sp = g.op_multi("split", [x], {"axis": "1 : i64", "splitSizes": _arr([2, 4])},
                        [(F, (2, 2, 5, 4)), (F, (2, 4, 5, 4))])
        sq = g.op("squeeze", [u], {"axes": _arr([0])}, F, s.shape)
        return [r, u, c, e, sp[0], sp[1], sq, g.add(t, g.const(1.0, F))]
    parity(*build(g_))


def test_tile_pad_resize():
    def g_(g):
        x = rand_input(g, (2, 3, 4), 61)
        reps = g.const([2, 1, 3], "i64")
        t = g.op("tile", [x, reps], None, F, (4, 3, 12))
        pads = g.const([0, 1, 2, 1, 0, 3], "i64")
        cv = g.const(-2.5, F)
        p = g.op("pad", [x, pads, cv], {"mode": '"constant"'}, F, (3, 4, 9))
        x4 = rand_input(g, (1, 2, 3, 5), 62)
        sc = g.const([1.0, 1.0, 2.0, 3.0], F)
        rz = g.op("resize", [x4, sc], {"mode": '"nearest"', "coordinateTransformationMode": '"asymmetric"',
                                       "nearestMode": '"floor"'}, F, (1, 2, 6, 15))
        return [t, p, rz]
    parity(*build(g_))


def test_pools():
    def g_(g):
        x = rand_input(g, (2, 5, 13, 11), 71)
        mp = g.op("max_pool", [x], {"kernelSize": _arr([3, 3]), "strides": _arr([2, 2]), "padding": _arr([1, 1]),
                                    "dilation": _arr([1, 1]), "ceilMode": "false"}, F, (2, 5, 7, 6))
        ap = g.op("average_pool", [x], {"kernelSize": _arr([2, 3]), "strides": _arr([2, 1]), "padding": _arr([0, 0]),
                                        "ceilMode": "false", "countIncludePad": "false"}, F, (2, 5, 6, 9))
        gp = g.op("global_average_pool", [x], None, F, (2, 5, 1, 1))
        ad = g.op("ad_avg_pool", [x], {"outputSize": _arr([1, 1])}, F, (2, 5, 1, 1))
        return [mp, ap, gp, ad]
    parity(*build(g_), atol=1e-6, rtol=1e-6)


def test_pools_channels_last():
    """Pools over a convolution's output, which the plan keeps channels-last,
    with C % 4 == 0: the float4 kernels, including the 3x3 stride-2 one that
    computes 1x2 output blocks, here with odd output extents (ragged blocks)
    and with and without padding."""
    def g_(g):
        x = rand_input(g, (2, 3, 15, 13), 72)
        wt = rand_input(g, (8, 3, 3, 3), 73, scale=0.3)
        b = rand_input(g, (8,), 74, scale=0.1)
        y = g.op("conv", [x, wt, b], {"strides": _arr([1, 1]), "padding": _arr([1, 1]), "dilation": _arr([1, 1])},
                 F, (2, 8, 15, 13))
        mp = g.op("max_pool", [y], {"kernelSize": _arr([3, 3]), "strides": _arr([2, 2]), "padding": _arr([1, 1]),
                                    "dilation": _arr([1, 1]), "ceilMode": "false"}, F, (2, 8, 8, 7))
        m0 = g.op("max_pool", [y], {"kernelSize": _arr([3, 3]), "strides": _arr([2, 2]), "padding": _arr([0, 0]),
                                    "dilation": _arr([1, 1]), "ceilMode": "false"}, F, (2, 8, 7, 6))
        ap = g.op("average_pool", [y], {"kernelSize": _arr([3, 3]), "strides": _arr([2, 2]), "padding": _arr([1, 1]),
                                        "ceilMode": "false", "countIncludePad": "true"}, F, (2, 8, 8, 7))
        m1 = g.op("max_pool", [y], {"kernelSize": _arr([3, 3]), "strides": _arr([1, 1]), "padding": _arr([1, 1]),
                                    "dilation": _arr([1, 1]), "ceilMode": "false"}, F, (2, 8, 15, 13))
        gp = g.op("global_average_pool", [y], None, F, (2, 8, 1, 1))
        return [mp, m0, ap, m1, gp]
    parity(*build(g_), atol=1e-6, rtol=1e-6)


def test_global_average_pool_channels_last_bits():
    """global_average_pool and ad_avg_pool over channels-last data (an NHWC
    argument seen through a transpose view): one thread per (n, c) row, summed
    in the reference's order (GaweeToLinalg.cpp:1327-1375: h, then w, from
    0, then divided by h*w), so the results match the oracle bit for bit."""
    def g_(g):
        xi = rand_input(g, (3, 7, 9, 40), 75)
        xt = g.transpose(xi, [0, 3, 1, 2])
        gp = g.op("global_average_pool", [xt], None, F, (3, 40, 1, 1))
        ad = g.op("ad_avg_pool", [xt], {"outputSize": _arr([1, 1])}, F, (3, 40, 1, 1))
        return [gp, ad]
    got, want = parity(*build(g_), atol=0, rtol=0)
    for k, (a, b) in enumerate(zip(got, want)):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"output{k}: bits differ"


def test_max_pool_signed_zero_and_nan_bits():
    """max_pool folds with arith.maximumf (GaweeToLinalg.cpp:565-706): NaN
    propagates and -0 < +0.  A channels-last input (an NHWC argument seen
    through a transpose view) holding mostly signed zeros, negatives, infs
    and a few NaNs; every non-NaN output must match the oracle bit for bit
    (the sign of zero included) and NaNs must sit in the same places."""
    rng = np.random.default_rng(91)
    vals = np.array([-0.0, 0.0, -1.0, -2.0, np.nan, -np.inf, np.inf], np.float32)
    p_lo = [0.55, 0.05, 0.2, 0.18, 0.01, 0.01, 0.0]   # channels 0-3: windows of only -0 and negatives
    p_hi = [0.3, 0.3, 0.15, 0.15, 0.03, 0.04, 0.03]   # channels 4-7
    x = np.concatenate([rng.choice(vals, (2, 9, 11, 4), p=p_lo), rng.choice(vals, (2, 9, 11, 4), p=p_hi)], axis=3)

    def g_(g):
        xi = g.input(F, (2, 9, 11, 8), lambda: x.astype(np.float32))
        xt = g.transpose(xi, [0, 3, 1, 2])
        outs = []
        for pad, (oh, ow), st in (((1, 1), (5, 6), 2), ((0, 0), (4, 5), 2), ((1, 1), (9, 11), 1)):
            outs.append(g.op("max_pool", [xt], {"kernelSize": _arr([3, 3]), "strides": _arr([st, st]),
                                                "padding": _arr(list(pad)), "dilation": _arr([1, 1]),
                                                "ceilMode": "false"}, F, (2, 8, oh, ow)))
        return outs
    got, want = parity(*build(g_), atol=0, rtol=0)
    for k, (a, b) in enumerate(zip(got, want)):
        ok = ~np.isnan(b)
        assert np.array_equal(a[ok].view(np.uint32), b[ok].view(np.uint32)), f"output{k}: bits differ"
        assert np.any(b[ok].view(np.uint32) == 0x80000000), f"output{k}: no -0 window in the case"


def test_range_shape_topk():
    def g_(g):
        r1 = g.range_(3, 40, 4)
        rf = g.op("range", [g.const(0.5, F), g.const(9.0, F), g.const(0.75, F)], None, F, (12,))
        x = g.input(F, (3, 10), lambda: np.array([[1, 5, 5, 2, 9, 9, 0, -1, 3, 9]] * 3, np.float32)
                    + np.arange(3, dtype=np.float32)[:, None])
        v, i = g.op_multi("topk", [x], {"k": "4 : i64", "axis": "1 : i64"}, [(F, (3, 4)), ("i64", (3, 4))])
        sh = g.op("shape", [x], {"start": "0 : i64", "end": "2 : i64"}, "i64", (2,))
        return [r1, rf, v, i, sh]
    parity(*build(g_))


def test_linalg_forms_from_emitter():
    def g_(g):
        x = rand_input(g, (3, 17), 81)
        p = g.pow(x, g.const(2.0, F))
        p3 = g.pow(g.relu(x), g.const(1.5, F))
        s, c = g.sin(g.mul(x, g.const(40.0, F))), g.cos(x)
        n = g.neg(x)
        r = g.range_(0, 17, 1)
        le = g.less_equal(g.unsqueeze(r, [0]), g.unsqueeze(r, [1]))
        return [p, p3, s, c, n, le]
    parity(*build(g_), atol=2e-6, rtol=2e-6)


def test_linalg_reduce_max():
    mlir = """
module {
  func.func @forward(%arg0: tensor<4x9xf32>) -> tensor<4xf32> {
    %cst = arith.constant 0xFF800000 : f32
    %0 = tensor.empty() : tensor<4xf32>
    %1 = linalg.fill ins(%cst : f32) outs(%0 : tensor<4xf32>) -> tensor<4xf32>
    %reduced = linalg.reduce ins(%arg0 : tensor<4x9xf32>) outs(%1 : tensor<4xf32>) dimensions = [1]
      (%in: f32, %init: f32) {
        %2 = arith.maximumf %in, %init : f32
        linalg.yield %2 : f32
      }
    return %reduced : tensor<4xf32>
  }
}
"""
    x = np.random.default_rng(3).standard_normal((4, 9)).astype(np.float32)
    parity(mlir, [x])


def test_batch_norm_and_flatten():
    """BatchNormOpLowering (GaweeToLinalg.cpp:1122-1173) per channel with the
    reference's operation order; FlattenOpLowering (813-870) as a view and as
    a copy of a transposed source."""
    def g_(g):
        x = rand_input(g, (2, 5, 7, 3), 81)
        w = g.weight((5,), lambda: np.random.default_rng(82).standard_normal(5).astype(np.float32))
        b = g.weight((5,), lambda: np.random.default_rng(83).standard_normal(5).astype(np.float32))
        mean = g.weight((5,), lambda: np.random.default_rng(84).standard_normal(5).astype(np.float32))
        var = g.weight((5,), lambda: np.random.default_rng(85).uniform(0.1, 2.0, 5).astype(np.float32))
        bn = g.op("batch_norm", [x, w, b, mean, var], {"affine": "true", "eps": "1.000000e-05 : f64"}, F,
                  (2, 5, 7, 3))
        f1 = g.op("flatten", [bn], {"startDim": "1 : i64", "endDim": "-1 : i64"}, F, (2, 105))
        t = g.transpose(x, [0, 2, 3, 1])
        f2 = g.op("flatten", [t], {"startDim": "1 : i64", "endDim": "2 : i64"}, F, (2, 21, 5))
        return [bn, f1, g.relu(f2)]
    got, want = parity(*build(g_), atol=0.0, rtol=0.0)  # same IEEE operations, same order: bit-exact


def test_golden_fixtures_on_cuda():
    """The committed torch-computed fixtures (tests/golden/) through the CUDA
    path, at the tolerance each fixture states."""
    import os

    from gawee_b200.runtime import Model
    from tests.helpers import compare
    gold = os.path.join(os.path.dirname(__file__), "golden")
    names = sorted(f[:-4] for f in os.listdir(gold) if f.endswith(".npz"))
    assert names
    for name in names:
        with open(os.path.join(gold, name + ".mlir")) as f:
            mlir = f.read()
        data = np.load(os.path.join(gold, name + ".npz"))
        args = [data[f"arg{i}"] for i in range(sum(k.startswith("arg") for k in data.files))]
        m = Model(mlir)
        try:
            outs = m.run(args)
        finally:
            m.close()
        for k, o in enumerate(outs):
            compare(o, data[f"out{k}"], atol=float(data["atol"]), rtol=1e-5, what=f"{name} output{k}")


def _names(mlir):
    from gawee_b200.runtime import plan_text
    return plan_text(mlir)


def test_fused_rms_and_layer_norm():
    """RMSNorm and LayerNorm chains as the emitter decomposes them (Pow /
    ReduceMean / Add / Sqrt / Div / Mul [/ Add], centering by Sub of a mean)
    run as one row kernel each, on a dense and on a strided (transposed)
    input, within fp32 rounding of the oracle's sequential sums.  Rows of up
    to 1024 aligned columns are held in registers, longer ones are streamed:
    576 and 1536 columns cover one of each."""
    from gawee_b200.synth import _layer_norm, _rms_norm

    def g_(g):
        x = rand_input(g, (2, 5, 96), 91, scale=3.0)
        xt = g.transpose(rand_input(g, (5, 2, 96), 92), [1, 0, 2])  # rows with two strides
        y = rand_input(g, (3, 7, 100), 93)                           # cols not a multiple of 4
        z = rand_input(g, (3, 4, 576), 94, scale=2.0)                # lanes hold 4 or 5 float4
        u = rand_input(g, (2, 3, 1536), 98)                          # longer than the register row
        return [_rms_norm(g, x, 1e-5), _rms_norm(g, xt, 1e-6), _layer_norm(g, y, 1e-12), _layer_norm(g, x, 1e-5),
                _rms_norm(g, z, 1e-5), _layer_norm(g, z, 1e-5), _rms_norm(g, u, 1e-6), _layer_norm(g, u, 1e-5)]
    mlir, args = build(g_)
    s = _names(mlir)
    assert s.count("rms_norm") == 4 and s.count("layer_norm") == 4, s
    parity(mlir, args, atol=2e-6, rtol=2e-6)


def test_fused_rope():
    """x * cos + rotate_half(x) * sin (Slice / Neg / Concat / Mul / Add) as
    one kernel, over a transposed [B, H, S, D] view with broadcast tables:
    the same IEEE operations as the graph, bit-exact."""
    def g_(g):
        x = g.transpose(rand_input(g, (2, 7, 3, 16), 95), [0, 2, 1, 3])     # [2, 3, 7, 16]
        cos = g.unsqueeze(rand_input(g, (7, 16), 96), [0, 1])
        sin = g.unsqueeze(rand_input(g, (7, 16), 97), [0, 1])
        d = 16
        x1 = g.slice(x, [0], [d // 2], [3])
        x2 = g.slice(x, [d // 2], [d], [3])
        rot = g.cat([g.neg(x2), x1], 3)
        return [g.add(g.mul(x, cos), g.mul(rot, sin))]
    mlir, args = build(g_)
    assert "rope" in _names(mlir)
    parity(mlir, args, atol=0.0, rtol=0.0)
