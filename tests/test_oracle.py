"""The CPU oracle: known-answer tests from hand-computed values, the reference's
own MLIR test inputs, and op-by-op agreement with torch on CPU."""
import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F_

from gawee_b200 import synth
from tests import torch_models as tm
from tests.helpers import _arr, build, compare, rand_input

F = "f32"
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def run(mlir, args, entry="forward"):
    import oracle
    return oracle.run(mlir, args, entry=entry)


# ---- known answers (values computed by hand) ------------------------------------------------

MATMUL_TEST = """
// shapes of the reference's middle/mlir/test/matmul_test.mlir
module {
  func.func @test_matmul_2d(%lhs: tensor<2x4xf32>, %rhs: tensor<4x3xf32>) -> tensor<2x3xf32> {
    %0 = "gawee.matmul"(%lhs, %rhs) : (tensor<2x4xf32>, tensor<4x3xf32>) -> tensor<2x3xf32>
    return %0 : tensor<2x3xf32>
  }
  func.func @test_matmul_batched(%lhs: tensor<1x2x3x4xf32>, %rhs: tensor<1x2x4x5xf32>) -> tensor<1x2x3x5xf32> {
    %0 = "gawee.matmul"(%lhs, %rhs) : (tensor<1x2x3x4xf32>, tensor<1x2x4x5xf32>) -> tensor<1x2x3x5xf32>
    return %0 : tensor<1x2x3x5xf32>
  }
}
"""


def test_kat_matmul_2d():
    a = np.arange(8, dtype=np.float32).reshape(2, 4)          # [[0,1,2,3],[4,5,6,7]]
    b = np.arange(12, dtype=np.float32).reshape(4, 3)         # [[0,1,2],...,[9,10,11]]
    got = run(MATMUL_TEST, [a, b], entry="test_matmul_2d")[0]
    # row 0: 0*[0,1,2]+1*[3,4,5]+2*[6,7,8]+3*[9,10,11] = [42,48,54]
    # row 1: 4*[0,1,2]+5*[3,4,5]+6*[6,7,8]+7*[9,10,11] = [114,136,158]
    assert np.array_equal(got, np.array([[42, 48, 54], [114, 136, 158]], np.float32))


def test_kat_matmul_batched():
    a = np.ones((1, 2, 3, 4), np.float32)
    a[0, 1] *= 2
    b = np.arange(40, dtype=np.float32).reshape(1, 2, 4, 5)
    got = run(MATMUL_TEST, [a, b], entry="test_matmul_batched")[0]
    # batch 0: column sums of b[0,0]; batch 1: 2 * column sums of b[0,1]
    s0 = np.array([30, 34, 38, 42, 46], np.float32)
    s1 = 2 * np.array([110, 114, 118, 122, 126], np.float32)
    assert np.array_equal(got[0, 0], np.tile(s0, (3, 1)))
    assert np.array_equal(got[0, 1], np.tile(s1, (3, 1)))


def test_kat_conv_padding_and_bias():
    # 1x1x3x3 input of ones, 1x1x3x3 kernel of ones, padding 1, stride 2, bias 0.5
    # outputs at (0,0),(0,2),(2,0),(2,2) of the padded sums: each sees a 2x2 corner -> 4 + 0.5
    def g_(g):
        x = g.input(F, (1, 1, 3, 3), lambda: np.ones((1, 1, 3, 3), np.float32))
        w = g.weight((1, 1, 3, 3), lambda: np.ones((1, 1, 3, 3), np.float32))
        b = g.weight((1,), lambda: np.full((1,), 0.5, np.float32))
        return [g.op("conv", [x, w, b], {"strides": _arr([2, 2]), "padding": _arr([1, 1]),
                                         "dilation": _arr([1, 1])}, F, (1, 1, 2, 2))]
    mlir, args = build(g_)
    assert np.array_equal(run(mlir, args)[0], np.full((1, 1, 2, 2), 4.5, np.float32))


def test_kat_batch_norm():
    # GaweeToLinalg.cpp:1122-1173: ((x - mean) / sqrt(var + eps)) * w + b per channel, eps rounded to f32
    x = np.array([[[[1.0, 3.0]], [[-2.0, 6.0]]]], np.float32)       # [1, 2, 1, 2]
    w = np.array([2.0, 0.5], np.float32)
    b = np.array([1.0, -1.0], np.float32)
    mean = np.array([1.0, 2.0], np.float32)
    var = np.array([4.0, 16.0 - 0.25], np.float32)                  # eps 0.25: sqrt(4.25), sqrt(16)

    def g_(g):
        xs = [g.input(F, a.shape, (lambda a=a: a)) for a in (x,)]
        ws = [g.weight(a.shape, (lambda a=a: a)) for a in (w, b, mean, var)]
        return [g.op("batch_norm", xs + ws, {"affine": "true", "eps": "2.500000e-01 : f64"}, F, x.shape)]
    got = run(*build(g_))[0]
    d0 = np.float32(np.sqrt(np.float32(4.25)))
    want = np.array([[[[(np.float32(0.0) / d0) * 2 + 1, (np.float32(2.0) / d0) * 2 + 1]],
                      [[(-4.0 / 4.0) * 0.5 - 1, (4.0 / 4.0) * 0.5 - 1]]]], np.float32)
    assert np.array_equal(got, want)
    assert got[0, 1, 0, 0] == -1.5 and got[0, 1, 0, 1] == -0.5


def test_kat_relu_maxpool_semantics():
    def g_(g):
        x = g.input(F, (1, 1, 2, 3), lambda: np.array([[[[-0.0, -2.0, np.nan], [1.0, -1.0, 0.0]]]], np.float32))
        r = g.relu(x)
        mp = g.op("max_pool", [x], {"kernelSize": _arr([2, 2]), "strides": _arr([1, 1]), "padding": _arr([1, 1]),
                                    "dilation": _arr([1, 1]), "ceilMode": "true"}, F, (1, 1, 3, 4))
        return [r, mp]
    mlir, args = build(g_)
    r, mp = run(mlir, args)
    # maximumf: relu(-0) = +0, NaN propagates
    assert r[0, 0, 0, 0] == 0.0 and not np.signbit(r[0, 0, 0, 0])
    assert np.isnan(r[0, 0, 0, 2])
    # -inf padding never wins; windows containing the NaN give NaN; ceilMode is ignored (type gives 3x4)
    want = np.array([[-0.0, -0.0, np.nan, np.nan], [1.0, 1.0, np.nan, np.nan], [1.0, 1.0, 0.0, 0.0]], np.float32)
    assert np.array_equal(np.isnan(mp[0, 0]), np.isnan(want))
    assert np.array_equal(mp[0, 0][~np.isnan(want)], want[~np.isnan(want)])


def test_kat_reduce_mean_is_sum_then_divide():
    x = np.array([[1.0, 2.0, 4.0], [0.5, 0.25, 0.125]], np.float32)

    def g_(g):
        v = g.input(F, (2, 3), lambda: x)
        return [g.reduce_mean(v, [1], True), g.reduce_mean(v, [0], False)]
    m1, m0 = run(*build(g_))
    assert np.array_equal(m1, np.array([[np.float32(7.0) / np.float32(3.0)], [np.float32(0.875) / np.float32(3.0)]]))
    assert np.array_equal(m0, (x[0] + x[1]) / np.float32(2.0))


def test_kat_topk_reference_selection_loop():
    # ties: first strictly larger value wins the scan -> lowest index first
    x = np.array([[3.0, 7.0, 7.0, -1.0, 7.0]], np.float32)

    def g_(g):
        v = g.input(F, (1, 5), lambda: x)
        return g.op_multi("topk", [v], {"k": "4 : i64", "axis": "1 : i64"}, [(F, (1, 4)), ("i64", (1, 4))])
    vals, idx = run(*build(g_))
    assert np.array_equal(vals, np.array([[7, 7, 7, 3]], np.float32))
    assert np.array_equal(idx, np.array([[1, 2, 4, 0]], np.int64))


def test_kat_cast_gather_slice_where_range():
    def g_(g):
        f = g.input(F, (4,), lambda: np.array([-2.7, -0.5, 0.5, 2.9], np.float32))
        b = g.input("i1", (4,), lambda: np.array([1, 0, 1, 0], np.bool_))
        tab = g.input(F, (3, 2), lambda: np.array([[0, 1], [10, 11], [20, 21]], np.float32))
        ids = g.input("i64", (2, 2), lambda: np.array([[2, 0], [1, 1]], np.int64))
        return [g.cast(f, 7, "i64"), g.cast(b, 1, F), g.gather(tab, ids, 0),
                g.slice(f, [-3], [4], [0], [2]), g.where(b, f, g.const(9.0, F)), g.range_(2, 11, 3)]
    c1, c2, ga, sl, wh, rg = run(*build(g_))
    assert np.array_equal(c1, np.array([-2, 0, 0, 2], np.int64))          # fptosi truncates
    assert np.array_equal(c2, np.array([1, 0, 1, 0], np.float32))         # i1 -> uitofp
    assert np.array_equal(ga, np.array([[[20, 21], [0, 1]], [[10, 11], [10, 11]]], np.float32))
    assert np.array_equal(sl, np.array([-0.5, 2.9], np.float32))          # start -3 -> 1, step 2
    assert np.array_equal(wh, np.array([-2.7, 9.0, 0.5, 9.0], np.float32))
    assert np.array_equal(rg, np.array([2, 5, 8], np.int64))


def test_gather_out_of_range_is_an_error():
    import oracle

    def g_(g):
        tab = g.input(F, (3, 2), lambda: np.zeros((3, 2), np.float32))
        ids = g.input("i64", (1,), lambda: np.array([-1], np.int64))      # the reference does not wrap
        return [g.gather(tab, ids, 0)]
    with pytest.raises(oracle.OracleError, match="gather index out of range"):
        run(*build(g_))


# ---- committed fixtures --------------------------------------------------------------------------

@pytest.mark.parametrize("name", sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz")))
def test_golden_fixtures(name):
    """Fixtures made by tests/golden/make_golden.py with torch (an independent implementation)."""
    with open(os.path.join(GOLDEN, name + ".mlir")) as f:
        mlir = f.read()
    data = np.load(os.path.join(GOLDEN, name + ".npz"))
    args = [data[f"arg{i}"] for i in range(sum(k.startswith("arg") for k in data.files))]
    outs = run(mlir, args)
    for k, o in enumerate(outs):
        compare(o, data[f"out{k}"], atol=float(data["atol"]), rtol=1e-5, what=f"{name} output{k}")


# ---- op-by-op agreement with torch -----------------------------------------------------------------

def test_ops_against_torch():
    def g_(g):
        x = rand_input(g, (2, 3, 9, 8), 1)
        y = rand_input(g, (3, 1, 8), 2)
        return [g.add(x, y), g.div(x, g.add(g.mul(y, y), g.const(1.0, F))), g.sigmoid(x),
                g.op("gelu", [x], None, F, x.shape), g.softmax(x, 2), g.reduce_mean(x, [1, 3], False),
                g.op("max_pool", [x], {"kernelSize": _arr([3, 2]), "strides": _arr([2, 2]), "padding": _arr([1, 0]),
                                       "dilation": _arr([1, 1]), "ceilMode": "false"}, F, (2, 3, 5, 4)),
                g.transpose(x, [0, 2, 3, 1]), g.erf(x)]
    mlir, args = build(g_)
    outs = run(mlir, args)
    x, y = torch.from_numpy(args[0]), torch.from_numpy(args[1])
    want = [x + y, x / (y * y + 1), torch.sigmoid(x), F_.gelu(x), torch.softmax(x, 2), x.mean((1, 3)),
            F_.max_pool2d(x, (3, 2), (2, 2), (1, 0)), x.permute(0, 2, 3, 1), torch.erf(x)]
    for k, (o, w) in enumerate(zip(outs, want)):
        compare(o, w.numpy(), 2e-6, 2e-6, f"op {k}")


@pytest.mark.parametrize("case", ["resnet", "bert", "llama", "gqa"])
def test_models_against_torch(case):
    if case == "resnet":
        g = synth.resnet18(2, image=64, widths=(8, 16, 16, 32), classes=10)
        ref = lambda a: tm.resnet18(a, (8, 16, 16, 32))
    elif case == "bert":
        g = synth.bert_tiny(seq=32, vocab=100, max_pos=64)
        ref = tm.bert_tiny
    elif case == "llama":
        g = synth.llama(2, 16, dim=48, layers=2, heads=2, ffn=64, vocab=50)
        ref = lambda a: tm.llama(a, 48, 2, 2)
    else:
        g = synth.llama(2, 16, dim=96, layers=2, heads=6, kv_heads=2, ffn=64, vocab=50)
        ref = lambda a: tm.llama(a, 96, 2, 6, 2)
    args = g.make_args()
    compare(run(g.mlir, args)[0], ref(args).astype(np.float32), 5e-5, 1e-5, case)


def test_full_size_models_against_torch():
    """Configs 0 and 1 at full size (seconds on the oracle)."""
    for g, ref in [(synth.resnet18(1), tm.resnet18), (synth.bert_tiny(), tm.bert_tiny)]:
        args = g.make_args()
        compare(run(g.mlir, args)[0], ref(args).astype(np.float32), g.atol, 1e-4, g.name)
