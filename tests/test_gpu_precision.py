"""The single-pass TF32 precision mode (gawee_set_precision) against its stated
error bound, and the default fp32 mode (three TF32 passes) unchanged around it.

Bound of one TF32 pass: both operands enter the tensor core truncated to 10
explicit mantissa bits (relative error below 2^-10 each, toward zero), so each
product is low by less than 2^-9 |a*b| and an output is off by at most
2^-9 * sum_k |a_k * b_k|, plus the fp32 accumulation term (a few ulps of the
same sum per promotion round; K * 2^-22 covers it generously here).
"""
import numpy as np
import pytest

from tests.helpers import _arr, build, compare, rand_input

pytestmark = pytest.mark.gpu

F = "f32"


def _run(mlir, args, precision):
    from gawee_b200.runtime import Model
    m = Model(mlir, precision=precision)
    try:
        assert m.precision == precision
        return m.run(args), m.run(args)  # eager, then the captured graph
    finally:
        m.close()


def _bound(abs_dot, k):
    return (2.0 ** -9 + k * 2.0 ** -22) * abs_dot + 1e-30


@pytest.mark.parametrize("m,k,n", [(300, 1000, 257), (129, 132, 130), (64, 4608, 64), (1000, 64, 3)])
def test_tf32_gemm_within_bound(m, k, n):
    import oracle

    def g_(g):
        return [g.matmul(rand_input(g, (m, k), 1), rand_input(g, (k, n), 2))]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0].astype(np.float64)
    bound = _bound(np.abs(args[0].astype(np.float64)) @ np.abs(args[1].astype(np.float64)), k)
    for got in _run(mlir, args, "tf32"):
        err = np.abs(got[0].astype(np.float64) - want)
        assert np.all(err <= bound), f"max err/bound {float(np.max(err / bound)):.3f}"
        # and it is a different computation from the fp32 mode: errors well above fp32's
        assert float(np.max(err)) > 1e-6 * float(np.max(np.abs(want)))


@pytest.mark.parametrize("n,c,h,w,f,k,s,p", [(2, 64, 14, 14, 64, 3, 1, 1),    # TMA kernel, BN 64 (folded)
                                             (1, 128, 9, 9, 256, 3, 2, 1),    # TMA kernel, BN 128
                                             (1, 3, 20, 20, 64, 7, 2, 3)])    # gather kernel (stem)
def test_tf32_conv_within_bound(n, c, h, w, f, k, s, p):
    import oracle
    ho = (h + 2 * p - k) // s + 1

    def g_(g):
        x = rand_input(g, (n, c, h, w), 11)
        wt = rand_input(g, (f, c, k, k), 12, scale=float(np.sqrt(2.0 / (c * k * k))))
        return [g.op("conv", [x, wt, g.const(np.zeros(f, np.float32), F, (f,))],
                     {"strides": _arr([s, s]), "padding": _arr([p, p]), "dilation": _arr([1, 1])}, F,
                     (n, f, ho, ho))]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0].astype(np.float64)
    # sum |x| |w| over each output's window: the same convolution of the absolute values
    abs_dot = oracle.run(mlir, [np.abs(a) for a in args])[0].astype(np.float64)
    bound = _bound(abs_dot, c * k * k)
    for got in _run(mlir, args, "tf32"):
        err = np.abs(got[0].astype(np.float64) - want)
        assert np.all(err <= bound), f"max err/bound {float(np.max(err / bound)):.3f}"


def test_tf32_attention_close_and_fp32_restored():
    """Fused attention in one pass: the scores lose TF32 precision, so only a
    loose closeness is claimed; switching back to fp32 on the same context
    recaptures the graph and restores parity at the reference tolerance."""
    import oracle
    from gawee_b200.runtime import Model
    B, H, S, D = 1, 2, 160, 64

    def g_(g):
        q = rand_input(g, (B, H, S, D), 21)
        kk = rand_input(g, (B, H, S, D), 22)
        v = rand_input(g, (B, H, S, D), 23)
        sc = g.div(g.matmul(q, g.transpose(kk, [0, 1, 3, 2])), g.const(8.0, F))
        return [g.matmul(g.softmax(sc, -1), v)]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0]
    m = Model(mlir)
    try:
        assert any("attention" in n for n, _, _ in m.kernels())
        fp32_a = m.run(args)[0]
        m.run(args)
        m.set_precision("tf32")
        t1 = m.run(args)[0]
        t2 = m.run(args)[0]
        m.set_precision("fp32")
        fp32_b = m.run(args)[0]
        fp32_c = m.run(args)[0]
    finally:
        m.close()
    compare(fp32_a, want, 5e-5, 1e-4, "fp32 before")
    np.testing.assert_array_equal(fp32_b, fp32_a)
    np.testing.assert_array_equal(fp32_c, fp32_a)
    np.testing.assert_array_equal(t1, t2)
    assert float(np.max(np.abs(t1 - want))) < 2e-2
    assert float(np.max(np.abs(t1 - want))) > 1e-6


def test_tf32_resnet_logits_close():
    """A whole model in one pass: no parity claim, only a closeness figure
    (the logits' max error relative to their scale), printed for the record."""
    import oracle
    from gawee_b200 import synth
    g = synth.resnet18(1, image=64)
    args = g.make_args()
    want = oracle.run(g.mlir, args)[0]
    got, got2 = _run(g.mlir, args, "tf32")
    np.testing.assert_array_equal(got[0], got2[0])
    rel = float(np.max(np.abs(got[0] - want))) / float(np.max(np.abs(want)))
    print(f"resnet18 b1 64x64 tf32: max |err| / max |logit| = {rel:.2e}")
    assert rel < 1e-2


def test_precision_api_rejects_unknown_modes():
    from gawee_b200.runtime import Model
    from gawee_b200 import synth
    g = synth.resnet18(1, image=32)
    m = Model(g.mlir)
    try:
        assert m.precision == "fp32"
        assert m._lib.gawee_set_precision(m._h, 7) == 1
        assert m._lib.gawee_precision(None) == -1
        with pytest.raises(ValueError):
            m.set_precision("fp8")
    finally:
        m.close()


# ---- BF16 mode ---------------------------------------------------------------------------
# Bound of one bf16 pass: both operands rounded to nearest bf16 (8 significant
# bits: relative error at most 2^-9 each), so each product is off by less than
# (2^-8 + 2^-18) |a*b|, and an output by at most 2^-8 * sum_k |a_k * b_k| plus
# the fp32 accumulation term (K * 2^-22 of the same sum covers it here).

def _bound_bf16(abs_dot, k):
    return (2.0 ** -8 + 2.0 ** -18 + k * 2.0 ** -22) * abs_dot + 1e-30


def _run_names(mlir, args, precision):
    from gawee_b200.runtime import Model
    m = Model(mlir, precision=precision)
    try:
        assert m.precision == precision
        names = [n for n, _, _ in m.kernels()]
        return names, (m.run(args), m.run(args))
    finally:
        m.close()


@pytest.mark.parametrize("m,k,n", [(300, 1000, 257), (129, 132, 130), (64, 4608, 64), (1000, 64, 40)])
def test_bf16_gemm_within_bound(m, k, n):
    """GEMMs on the TMA kernel (BN 128 and 64) in the BF16 mode: inside the
    stated bound, and a different computation from the fp32 mode."""
    import oracle

    def g_(g):
        return [g.matmul(rand_input(g, (m, k), 1), rand_input(g, (k, n), 2))]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0].astype(np.float64)
    bound = _bound_bf16(np.abs(args[0].astype(np.float64)) @ np.abs(args[1].astype(np.float64)), k)
    names, outs = _run_names(mlir, args, "bf16")
    assert any("[tma]" in nm and "[bf16]" in nm for nm in names), names
    for got in outs:
        err = np.abs(got[0].astype(np.float64) - want)
        assert np.all(err <= bound), f"max err/bound {float(np.max(err / bound)):.3f}"
        assert float(np.max(err)) > 1e-5 * float(np.max(np.abs(want)))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])


@pytest.mark.parametrize("n,c,h,w,f,k,s,p", [(2, 64, 14, 14, 64, 3, 1, 1),    # im2col TMA, BN 64
                                             (1, 128, 9, 9, 256, 3, 2, 1)])   # im2col TMA, BN 128
def test_bf16_conv_within_bound(n, c, h, w, f, k, s, p):
    import oracle
    ho = (h + 2 * p - k) // s + 1

    def g_(g):
        x = rand_input(g, (n, c, h, w), 11)
        wt = rand_input(g, (f, c, k, k), 12, scale=float(np.sqrt(2.0 / (c * k * k))))
        return [g.op("conv", [x, wt, g.const(np.zeros(f, np.float32), F, (f,))],
                     {"strides": _arr([s, s]), "padding": _arr([p, p]), "dilation": _arr([1, 1])}, F,
                     (n, f, ho, ho))]
    mlir, args = build(g_)
    want = oracle.run(mlir, args)[0].astype(np.float64)
    abs_dot = oracle.run(mlir, [np.abs(a) for a in args])[0].astype(np.float64)
    bound = _bound_bf16(abs_dot, c * k * k)
    names, outs = _run_names(mlir, args, "bf16")
    assert any("[tma im2col]" in nm and "[bf16]" in nm for nm in names), names
    for got in outs:
        err = np.abs(got[0].astype(np.float64) - want)
        assert np.all(err <= bound), f"max err/bound {float(np.max(err / bound)):.3f}"


def test_bf16_resnet_logits_close_and_fp32_restored():
    """A whole model in the BF16 mode (the stem and other gather-kernel ops in
    single-pass TF32): no parity claim, a closeness figure printed for the
    record; switching back to fp32 on the same context gives the fp32 bits."""
    import oracle
    from gawee_b200 import synth
    from gawee_b200.runtime import Model
    g = synth.resnet18(2, image=64)
    args = g.make_args()
    want = oracle.run(g.mlir, args)[0]
    m = Model(g.mlir)
    try:
        fp32_a = m.run(args)[0]
        m.run(args)
        m.set_precision("bf16")
        b1 = m.run(args)[0]
        b2 = m.run(args)[0]
        m.set_precision("fp32")
        fp32_b = m.run(args)[0]
        m.set_precision("bf16")  # the bf16 planes are kept and still current
        b3 = m.run(args)[0]
    finally:
        m.close()
    np.testing.assert_array_equal(fp32_b, fp32_a)
    np.testing.assert_array_equal(b1, b2)
    np.testing.assert_array_equal(b3, b1)
    rel = float(np.max(np.abs(b1 - want))) / float(np.max(np.abs(want)))
    print(f"resnet18 b2 64x64 bf16: max |err| / max |logit| = {rel:.2e}")
    assert 1e-5 < rel < 5e-2


def test_bf16_gqa_decoder_close():
    """A GQA decoder in the BF16 mode: merged Q/K/V GEMM, residual and SwiGLU
    epilogues with the staged operand in bf16, attention in single-pass TF32.
    A closeness figure against the oracle, and the fp32 bits after switching
    back."""
    import oracle
    from gawee_b200 import synth
    from gawee_b200.runtime import Model
    g = synth.llama(2, 64, dim=576, layers=2, heads=9, kv_heads=3, ffn=1536, vocab=4096, name="decoder_l2_bf16")
    args = g.make_args()
    want = oracle.run(g.mlir, args)[0]
    m = Model(g.mlir)
    try:
        fp32_a = m.run(args)[0]
        m.set_precision("bf16")
        names = [n for n, _, _ in m.kernels()]
        b1 = m.run(args)[0]
        b2 = m.run(args)[0]
        m.set_precision("fp32")
        fp32_b = m.run(args)[0]
    finally:
        m.close()
    assert any(n.startswith("matmul3") and "[bf16]" in n for n in names), names
    assert any("sigmoid" in n and "[aux smem]" in n and "[bf16]" in n for n in names), names
    np.testing.assert_array_equal(fp32_b, fp32_a)
    np.testing.assert_array_equal(b1, b2)
    rel = float(np.max(np.abs(b1 - want))) / float(np.max(np.abs(want)))
    print(f"decoder 2 layers b2 s64 bf16: max |err| / max |logit| = {rel:.2e}")
    assert 1e-5 < rel < 5e-2
