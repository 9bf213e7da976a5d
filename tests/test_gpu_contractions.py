"""Tensor-core contractions (3xTF32 tcgen05) against the oracle's sequential fp32 sums."""
import math

import numpy as np
import pytest

from tests.helpers import _arr, build, compare, parity, rand_input

pytestmark = pytest.mark.gpu

F = "f32"


@pytest.mark.parametrize("m,k,n", [(1, 4, 1), (7, 12, 5), (128, 32, 64), (129, 33 * 4, 130), (300, 1000, 257),
                                   (64, 4608, 512), (1000, 64, 3)])
def test_matmul_2d(m, k, n):
    def g_(g):
        a = rand_input(g, (m, k), 1)
        b = rand_input(g, (k, n), 2)
        return [g.matmul(a, b)]
    # fp32-level error: a few ulps of the sum of |a*b| terms
    parity(*build(g_), atol=1e-4 * max(1.0, np.sqrt(k) / 8), rtol=1e-4)


def _scaled_parity(mlir, args, rel=2e-5):
    """fp32 sums in a different order agree to a few ulps of the output scale:
    compare with an absolute tolerance proportional to max|output|."""
    import oracle
    from gawee_b200.runtime import Model
    want = oracle.run(mlir, args)
    m = Model(mlir)
    try:
        got = m.run(args)
    finally:
        m.close()
    for k, (a, b) in enumerate(zip(got, want)):
        compare(a, b, rel * float(np.max(np.abs(b))), 0.0, f"output{k}")


def test_matmul_batched_broadcast():
    def g_(g):
        a = rand_input(g, (2, 3, 70, 48), 3)
        b = rand_input(g, (3, 48, 90), 4)        # batch broadcast over the leading dim
        c = rand_input(g, (1, 3, 90, 20), 5)     # size-1 batch dim broadcast
        d = rand_input(g, (20, 33), 6)           # 2-D rhs, batched lhs
        ab = g.matmul(a, b)
        return [ab, g.matmul(ab, c), g.matmul(g.matmul(ab, c), d)]
    _scaled_parity(*build(g_))


def test_matmul_transposed_operands():
    def g_(g):
        q = rand_input(g, (2, 50, 4, 16), 7)     # [b, s, h, d]
        k = rand_input(g, (2, 50, 4, 16), 8)
        qt = g.transpose(q, [0, 2, 1, 3])
        kt = g.transpose(k, [0, 2, 3, 1])
        s = g.matmul(qt, kt)                     # [b, h, s, s]
        return [s, g.matmul(s, g.transpose(k, [0, 2, 1, 3]))]
    parity(*build(g_), atol=2e-4, rtol=1e-4)


def test_linear_bias_and_epilogue():
    def g_(g):
        x = rand_input(g, (37, 96), 9)
        w = rand_input(g, (70, 96), 10)
        b = rand_input(g, (70,), 11)
        y = g.linear(x, w, b)
        return [g.relu(y), g.linear(g.relu(y), rand_input(g, (5, 70), 12), rand_input(g, (5,), 13))]
    parity(*build(g_), atol=2e-4, rtol=1e-4)


def test_matmul_fused_epilogues():
    def g_(g):
        x = rand_input(g, (3, 40, 64), 14)
        w = rand_input(g, (64, 96), 15)
        bias = rand_input(g, (96,), 16)
        y = g.add(g.matmul(x, w), bias)
        gl = g.mul(g.mul(y, g.add(g.erf(g.div(y, g.const(1.4142135381698608, F))), g.const(1.0, F))),
                   g.const(0.5, F))
        gate = g.matmul(x, rand_input(g, (64, 96), 17))
        up = g.matmul(x, rand_input(g, (64, 96), 18))
        sw = g.mul(g.mul(gate, g.sigmoid(gate)), up)
        return [gl, sw]
    parity(*build(g_), atol=2e-4, rtol=1e-4)


@pytest.mark.parametrize("scale", [8.0, 6.928203230275509])
def test_attention_score_epilogue(scale):
    """Batched Q.K^T with the score epilogue the emitter produces: divide by a
    constant, add a broadcast mask.  A power-of-two divisor takes the exact
    reciprocal-multiply path, any other the IEEE division; both must match the
    oracle, as must a residual add on a second product."""
    def g_(g):
        q = rand_input(g, (2, 3, 130, 64), 31)
        k = rand_input(g, (2, 3, 64, 136), 32)
        mask = rand_input(g, (1, 1, 130, 136), 33, scale=5.0)
        sc = g.add(g.div(g.matmul(q, k), g.const(scale, F)), mask)
        res = rand_input(g, (2, 3, 130, 136), 34)
        return [sc, g.add(res, g.matmul(q, k))]
    parity(*build(g_), atol=2e-4, rtol=1e-4)


CONVS = [
    # (N, C, H, W, F, k, stride, pad, dil)
    (1, 3, 33, 31, 16, 7, 2, 3, 1),     # stem-like, C=3 -> padded to 4 channels
    (2, 16, 14, 14, 32, 3, 1, 1, 1),
    (1, 32, 15, 13, 64, 3, 2, 1, 1),
    (2, 64, 7, 7, 128, 3, 1, 1, 1),
    (2, 24, 9, 9, 40, 1, 2, 0, 1),
    (1, 8, 20, 20, 24, 3, 1, 2, 2),     # dilation 2
    (1, 12, 6, 5, 200, 3, 1, 0, 1),     # N tail beyond one 128 tile, no padding
]


@pytest.mark.parametrize("n,c,h,w,f,k,s,p,d", CONVS)
def test_conv(n, c, h, w, f, k, s, p, d):
    ho = (h + 2 * p - d * (k - 1) - 1) // s + 1
    wo = (w + 2 * p - d * (k - 1) - 1) // s + 1

    def g_(g):
        x = rand_input(g, (n, c, h, w), 21)
        wt = rand_input(g, (f, c, k, k), 22, scale=float(np.sqrt(2.0 / (c * k * k))))
        b = rand_input(g, (f,), 23, scale=0.1)
        y = g.op("conv", [x, wt, b], {"strides": _arr([s, s]), "padding": _arr([p, p]), "dilation": _arr([d, d])},
                 F, (n, f, ho, wo))
        return [y, g.relu(y)]
    parity(*build(g_), atol=1e-4, rtol=1e-4)


def test_conv_residual_block():
    def g_(g):
        x = g.relu(rand_input(g, (2, 32, 10, 10), 31))
        w1 = rand_input(g, (32, 32, 3, 3), 32, scale=0.08)
        w2 = rand_input(g, (32, 32, 3, 3), 33, scale=0.08)
        b1, b2 = rand_input(g, (32,), 34, scale=0.01), rand_input(g, (32,), 35, scale=0.01)
        att = {"strides": _arr([1, 1]), "padding": _arr([1, 1]), "dilation": _arr([1, 1])}
        y = g.relu(g.op("conv", [x, w1, b1], att, F, (2, 32, 10, 10)))
        y = g.op("conv", [y, w2, b2], att, F, (2, 32, 10, 10))
        return [g.relu(g.add(y, x))]
    parity(*build(g_), atol=1e-4, rtol=1e-4)


def _run_with_split_cap(mlir, args, cap):
    import os

    from gawee_b200.runtime import Model
    old = os.environ.get("GAWEE_MAX_KSPLIT")
    os.environ["GAWEE_MAX_KSPLIT"] = str(cap)
    try:
        m = Model(mlir)
    finally:
        if old is None:
            del os.environ["GAWEE_MAX_KSPLIT"]
        else:
            os.environ["GAWEE_MAX_KSPLIT"] = old
    try:
        names = [n for n, _, _ in m.kernels()]
        outs = [m.run(args)[0] for _ in range(2)]  # eager, then the replayed graph
    finally:
        m.close()
    return names, outs


@pytest.mark.parametrize("case", ["gemm", "conv_residual", "conv_stride2"])
def test_split_k_matches_oracle_and_unsplit(case):
    """Small-M contractions split along k (partial sums in a workspace, a
    reduce kernel adds them in split order and applies bias / residual /
    ReLU): same results as the unsplit kernel and the oracle, within the
    fp32 tolerance of the contraction tests."""
    import oracle

    def g_(g):
        if case == "gemm":
            a = rand_input(g, (49, 4608), 11)
            b = rand_input(g, (4608, 520), 12)
            return [g.matmul(a, b)]
        x = rand_input(g, (1, 256, 14, 14) if case == "conv_stride2" else (1, 512, 7, 7), 13)
        cin = x.shape[1]
        cout = 512
        stride = 2 if case == "conv_stride2" else 1
        w = g.normal((cout, cin, 3, 3), math.sqrt(2.0 / (cin * 9)))
        bias = g.normal((cout,), 0.01)
        y = g.op("conv", [x, w, bias], {"strides": _arr([stride, stride]), "padding": _arr([1, 1]),
                                        "dilation": _arr([1, 1])}, F, (1, cout, 7, 7))
        if case == "conv_residual":
            y = g.relu(g.add(y, x))
        return [y]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0]
    names1, outs1 = _run_with_split_cap(mlir, args, 1)
    names, outs = _run_with_split_cap(mlir, args, 32)
    assert not any("split-k" in n for n in names1)
    assert any("split-k" in n for n in names), names
    k = 4608 if case == "gemm" else args[0].shape[1] * 9
    atol = 1e-4 * max(1.0, np.sqrt(k) / 8)
    for o in outs1 + outs:
        compare(o, want, atol, 1e-4, case)


def _run_env(mlir, args, env):
    import os

    from gawee_b200.runtime import Model
    old = {k: os.environ.get(k) for k in env}
    os.environ.update({k: str(v) for k, v in env.items()})
    try:
        m = Model(mlir)
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v
    try:
        names = [n for n, _, _ in m.kernels()]
        outs = [m.run(args) for _ in range(2)]  # eager, then the replayed graph
    finally:
        m.close()
    return names, outs


TMA_CONVS = [
    # (N, C, H, W, F, k, stride, pad, dil): channel counts that are multiples of 32, or 4, 8 and 16,
    # take the TMA kernel
    (3, 32, 9, 11, 40, 3, 1, 1, 1),     # tiles span images; F not a multiple of 64
    (2, 64, 17, 17, 64, 3, 2, 1, 1),    # stride 2
    (1, 96, 12, 10, 130, 5, 1, 2, 1),   # 5x5, three 32-channel k-blocks per tap
    (2, 32, 13, 13, 48, 3, 1, 2, 2),    # dilation 2
    (2, 64, 14, 14, 128, 1, 2, 0, 1),   # 1x1 stride-2 downsample
    (1, 32, 23, 21, 64, 7, 2, 3, 1),    # 7x7 stride 2 pad 3: corners -3 / -3
    # 4, 8 or 16 channels (3 is padded to 4): tap blocks, several taps per k-block
    (2, 3, 30, 27, 64, 7, 2, 3, 1),     # the ResNet stem's shape: 49 taps, 7 k-blocks, last repeats tap 48
    (1, 4, 19, 19, 40, 3, 1, 1, 1),     # 9 taps of 4 channels: 2 k-blocks (8 + 1 taps)
    (2, 8, 15, 16, 64, 3, 1, 1, 1),     # 4 taps per k-block
    (1, 16, 13, 11, 72, 5, 2, 2, 1),    # 2 taps per k-block, stride 2
    (1, 8, 12, 12, 64, 3, 1, 2, 2),     # dilation 2 with tap blocks
]


@pytest.mark.parametrize("n,c,h,w,f,k,s,p,d", TMA_CONVS)
def test_conv_tma_im2col_matches_gather_and_oracle(n, c, h, w, f, k, s, p, d):
    """The TMA-fed kernel (im2col tensor map for A) against the oracle and
    against the warp-gather kernel on the same graph."""
    import oracle
    ho = (h + 2 * p - d * (k - 1) - 1) // s + 1
    wo = (w + 2 * p - d * (k - 1) - 1) // s + 1

    def g_(g):
        x = rand_input(g, (n, c, h, w), 41)
        wt = rand_input(g, (f, c, k, k), 42, scale=float(np.sqrt(2.0 / (c * k * k))))
        b = rand_input(g, (f,), 43, scale=0.1)
        y = g.op("conv", [x, wt, b], {"strides": _arr([s, s]), "padding": _arr([p, p]), "dilation": _arr([d, d])},
                 F, (n, f, ho, wo))
        return [g.relu(y)]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0]
    names, outs = _run_env(mlir, args, {"GAWEE_MAX_KSPLIT": 1, "GAWEE_TC_TMA_TAPS": 1})
    names_g, outs_g = _run_env(mlir, args, {"GAWEE_MAX_KSPLIT": 1, "GAWEE_TC_TMA": 0})
    assert any(("tma im2col taps" if c % 32 else "tma im2col") in nm for nm in names), names
    assert not any("tma" in nm for nm in names_g), names_g
    for o in outs + outs_g:
        compare(o[0], want, 1e-4, 1e-4, "conv")


@pytest.mark.parametrize("m,k,n", [(1, 36, 70), (200, 300, 130), (129, 64, 64), (517, 1000, 257)])
def test_gemm_tma_rows_matches_oracle(m, k, n):
    """Unbatched GEMMs take A through a tiled tensor map (K tails zero-filled by the copy engine)."""
    import oracle

    def g_(g):
        a = rand_input(g, (m, k), 51)
        b = rand_input(g, (k, n), 52)
        return [g.matmul(a, b)]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0]
    names, outs = _run_env(mlir, args, {})
    assert any("[tma]" in nm for nm in names), names
    for o in outs:
        compare(o[0], want, 1e-4 * max(1.0, np.sqrt(k) / 8), 1e-4, "gemm")


def test_batched_lhs_rows_merge_into_one_gemm():
    """A batched lhs times a 2-D rhs whose batch dims only continue the rows
    runs as one unbatched GEMM (the TMA kernel), residual epilogue included."""
    import oracle

    def g_(g):
        x = rand_input(g, (4, 50, 36), 61)
        w = rand_input(g, (36, 72), 62)
        r = rand_input(g, (4, 50, 72), 63)
        w2 = rand_input(g, (72, 36), 64)
        y = g.add(g.matmul(x, w), r)           # residual fused into the epilogue (aux rows merge too)
        return [y, g.matmul(g.transpose(y, [1, 0, 2]), w2)]  # rows do not continue: stays batched
    mlir, args = build(g_)
    want = oracle.run(mlir, args)
    names, outs = _run_env(mlir, args, {})
    assert sum("[tma]" in nm for nm in names) == 1, names
    for o in outs:
        for k in range(2):
            compare(o[k], want[k], 2e-4, 1e-4, f"output{k}")


AUX_GEMMS = [
    # (m, k, n, epilogue): the TMA kernel stages the epilogue's operand tile in shared memory
    (300, 576, 200, "add"),       # partial M and N tiles; the tile loaded mid-unit (18 k-blocks)
    (9000, 64, 576, "add"),       # 2 k-blocks: loaded with the unit's first; 2-3 tiles per CTA
    (12800, 576, 512, "swiglu"),  # (gate * sigmoid(gate)) * up, one operand tile; 2-3 tiles per CTA
    (517, 320, 64, "divc"),       # BN 64; (acc / 6.93) + r, the IEEE division
    (260, 96, 40, "mulc"),        # BN 64, partial N; (acc / 8) + r as an exact multiply
]


@pytest.mark.parametrize("m,k,n,epi", AUX_GEMMS)
def test_gemm_aux_staged_epilogue_matches_oracle_and_global_reads(m, k, n, epi):
    """The residual / fast-epilogue operand through a TMA-staged shared-memory
    tile (GAWEE_TC_TMA_AUX=1): the oracle's values, and bit for bit the
    epilogue that reads the operand from global memory (GAWEE_TC_TMA_AUX=0)."""
    import oracle

    ws = float(1.0 / np.sqrt(k))  # unit-variance products, as in a trained layer

    def g_(g):
        a = rand_input(g, (m, k), 71)
        y = g.matmul(a, rand_input(g, (k, n), 72, scale=ws))
        if epi == "swiglu":
            gate = g.matmul(a, rand_input(g, (k, n), 73, scale=ws))
            return [g.mul(g.mul(gate, g.sigmoid(gate)), y)]
        r = rand_input(g, (m, n), 74)
        if epi == "divc":
            y = g.div(y, g.const(6.928203230275509, F))
        elif epi == "mulc":
            y = g.div(y, g.const(8.0, F))
        return [g.add(y, r)]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0]
    names, outs = _run_env(mlir, args, {"GAWEE_MAX_KSPLIT": 1, "GAWEE_TC_TMA_AUX": 1})
    names_g, outs_g = _run_env(mlir, args, {"GAWEE_MAX_KSPLIT": 1, "GAWEE_TC_TMA_AUX": 0})
    assert any("[tma]" in nm and "[aux smem]" in nm for nm in names), names
    assert not any("[aux smem]" in nm for nm in names_g), names_g
    for o in outs:
        compare(o[0], want, 1e-4, 1e-4, epi)
        np.testing.assert_array_equal(o[0], outs_g[0][0])


@pytest.mark.parametrize("f", [64, 128])
def test_conv_residual_aux_staged_matches_oracle_and_global_reads(f):
    """A residual block on the im2col TMA kernel (BN 64 and 128): the
    residual tile staged in shared memory gives the oracle's values and the
    same bits as the epilogue's global reads."""
    import oracle

    def g_(g):
        att = {"strides": _arr([1, 1]), "padding": _arr([1, 1]), "dilation": _arr([1, 1])}
        # the block's input is a convolution's output, as in ResNet (channels-last, so the residual fuses)
        w0 = rand_input(g, (f, 32, 3, 3), 80, scale=float(np.sqrt(2.0 / (9 * 32))))
        x = g.relu(g.op("conv", [rand_input(g, (3, 32, 17, 15), 81), w0, rand_input(g, (f,), 86, scale=0.1)],
                        att, F, (3, f, 17, 15)))
        w1 = rand_input(g, (f, f, 3, 3), 82, scale=float(np.sqrt(2.0 / (9 * f))))
        w2 = rand_input(g, (f, f, 3, 3), 83, scale=float(np.sqrt(2.0 / (9 * f))))
        b1, b2 = rand_input(g, (f,), 84, scale=0.1), rand_input(g, (f,), 85, scale=0.1)
        y = g.relu(g.op("conv", [x, w1, b1], att, F, (3, f, 17, 15)))
        y = g.op("conv", [y, w2, b2], att, F, (3, f, 17, 15))
        z = g.relu(g.add(y, x))
        # and a 1x1 convolution reads the block's output, which so stays channels-last
        w3 = rand_input(g, (32, f, 1, 1), 87, scale=float(np.sqrt(1.0 / f)))
        one = {"strides": _arr([1, 1]), "padding": _arr([0, 0]), "dilation": _arr([1, 1])}
        return [g.op("conv", [z, w3, rand_input(g, (32,), 88, scale=0.1)], one, F, (3, 32, 17, 15))]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0]
    names, outs = _run_env(mlir, args, {"GAWEE_MAX_KSPLIT": 1, "GAWEE_TC_TMA_AUX": 1})
    names_g, outs_g = _run_env(mlir, args, {"GAWEE_MAX_KSPLIT": 1, "GAWEE_TC_TMA_AUX": 0})
    assert any("conv+add+relu [tma im2col] [aux smem]" in nm for nm in names), names
    assert not any("[aux smem]" in nm for nm in names_g), names_g
    for o in outs:
        compare(o[0], want, 1e-4, 1e-4, "residual block")
        np.testing.assert_array_equal(o[0], outs_g[0][0])
