"""The fused attention op against the oracle.

The planner folds matmul(Q, K^T) -> div(c) -> add(mask) -> softmax(-1) ->
matmul(., V) (GaweeToLinalg.cpp:959-1112, 1377-1441, 1885-1900), with the GQA
head expansion unsqueeze -> expand -> reshape of K and V, into one tcgen05
kernel with an online softmax.  Cases: sequence tails (S not a multiple of
128), head dims 32 / 48 / 64, GQA, causal -inf masks (whole key tiles
skipped), a padding mask broadcast over rows, no mask at all, a power-of-two and a
non-power-of-two divisor, and an output consumed in [B, S, H, D] order.
"""
import math

import numpy as np
import pytest

from tests.helpers import build, compare, rand_input

pytestmark = pytest.mark.gpu

F = "f32"


def _graph(B, H, Hkv, S, D, mask_kind, c, transpose_out):
    def g_(g):
        q = rand_input(g, (B, H, S, D), 1)
        k = rand_input(g, (B, Hkv, S, D), 2)
        v = rand_input(g, (B, Hkv, S, D), 3)
        if Hkv != H:
            rep = H // Hkv
            k = g.reshape(g.expand(g.unsqueeze(k, [2]), (B, Hkv, rep, S, D)), (B, H, S, D))
            v = g.reshape(g.expand(g.unsqueeze(v, [2]), (B, Hkv, rep, S, D)), (B, H, S, D))
        if mask_kind == "none":
            mask = None
        elif mask_kind == "causal":
            r = g.range_(0, S, 1)
            allowed = g.less_equal(g.unsqueeze(r, [0]), g.unsqueeze(r, [1]))
            mask = g.where(allowed, g.const(0.0, F), g.const(float("-inf"), F))
        else:  # padding mask over keys, broadcast over heads and rows: the last keys of batch 1 are -inf
            m = np.zeros((B, 1, 1, S), np.float32)
            m[-1, 0, 0, S - S // 3:] = -np.inf
            m[0, 0, 0, 1] = -10000.0
            mask = g.const(m, F, (B, 1, 1, S))
        s = g.div(g.matmul(q, g.transpose(k, [0, 1, 3, 2])), g.const(c, F))
        if mask is not None:
            s = g.add(s, mask)
        o = g.matmul(g.softmax(s, -1), v)
        if transpose_out:
            o = g.reshape(g.transpose(o, [0, 2, 1, 3]), (B, S, H * D))
        return [o]
    return build(g_)


CASES = [
    # B, H, Hkv, S, D, mask, divisor, output transposed
    (2, 3, 3, 200, 64, "causal", 8.0, True),
    (1, 9, 3, 384, 64, "causal", 8.0, True),          # GQA 3:1, three key tiles
    (2, 2, 2, 130, 48, "causal", math.sqrt(48), False),  # head dim 48, non-power-of-two divisor
    (2, 2, 1, 96, 32, "padding", math.sqrt(32), True),   # padding mask, GQA 2:1
    (1, 2, 2, 256, 64, "padding", 8.0, False),
    (2, 4, 2, 160, 64, "none", 8.0, False),             # no mask: softmax straight over the scaled scores
]


@pytest.mark.parametrize("B,H,Hkv,S,D,mask,c,tr", CASES)
def test_fused_attention_matches_oracle(B, H, Hkv, S, D, mask, c, tr):
    import oracle
    from gawee_b200.runtime import Model
    mlir, args = _graph(B, H, Hkv, S, D, mask, c, tr)
    want = oracle.run(mlir, args)[0]
    m = Model(mlir)
    try:
        names = [n for n, _, _ in m.kernels()]
        assert "attention" in names, names
        assert not any("softmax" in n for n in names), names
        for _ in range(2):  # eager, then the replayed graph
            got = m.run(args)[0]
            compare(got, want, 5e-5, 1e-4, f"attention {B}x{H}/{Hkv}x{S}x{D} {mask}")
    finally:
        m.close()
