"""Generate the golden fixtures in this directory.

Each fixture is a small gawee-dialect graph (`<name>.mlir`) plus an npz with
its seeded arguments (`argN`), the expected outputs (`outN`) computed with
torch on CPU in float64 and rounded to float32 (an implementation independent
of the oracle and of the CUDA backend), and the tolerance (`atol`).

The reference repository ships no golden vectors for its lowering (its
tests/*.py are empty), so these are the known-answer vectors the oracle is
pinned to; the graph shapes follow the reference's own MLIR test inputs
(middle/mlir/test/matmul_test.mlir, simple_test.mlir) and small versions of
the benchmark blocks.

    python tests/golden/make_golden.py
"""
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from gawee_b200.synth import GraphBuilder, _arr  # noqa: E402


def t64(a):
    return torch.from_numpy(np.asarray(a)).to(torch.float64)


def save(name, g, outs, fn, atol):
    mlir = g.finish(outs)
    args = [np.ascontiguousarray(a.make()) for a in g.args]
    want = fn(*[t64(a) if a.dtype == np.float32 else torch.from_numpy(a) for a in args])
    if not isinstance(want, (list, tuple)):
        want = [want]
    data = {f"arg{i}": a for i, a in enumerate(args)}
    for i, w in enumerate(want):
        data[f"out{i}"] = w.to(torch.float32).numpy() if w.is_floating_point() else w.numpy()
    data["atol"] = np.float64(atol)
    with open(os.path.join(HERE, name + ".mlir"), "w") as f:
        f.write(mlir)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **data)


def rnd(g, shape, seed, scale=1.0):
    return g.input("f32", shape, lambda: (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32))


def main():
    # 1. matmul_test.mlir shapes: 2x4 . 4x3 and batched 1x2x3x4 . 1x2x4x5
    g = GraphBuilder("golden:matmul")
    a, b = rnd(g, (2, 4), 1), rnd(g, (4, 3), 2)
    c, d = rnd(g, (1, 2, 3, 4), 3), rnd(g, (1, 2, 4, 5), 4)
    save("matmul_test", g, [g.matmul(a, b), g.matmul(c, d)], lambda a, b, c, d: [a @ b, c @ d], 1e-6)

    # 2. simple_test.mlir ops (add, relu, conv 1x3x32x32 with 16x3x3x3) with an explicit bias
    g = GraphBuilder("golden:simple")
    x0, x1 = rnd(g, (2, 3), 5), rnd(g, (2, 3), 6)
    xi, w = rnd(g, (1, 3, 32, 32), 7), rnd(g, (16, 3, 3, 3), 8, 0.3)
    bias = rnd(g, (16,), 9, 0.1)
    conv = g.op("conv", [xi, w, bias], {"strides": _arr([1, 1]), "padding": _arr([0, 0]),
                                        "dilation": _arr([1, 1])}, "f32", (1, 16, 30, 30))
    save("simple_test", g, [g.add(x0, x1), g.relu(x0), conv],
         lambda x0, x1, xi, w, b: [x0 + x1, torch.relu(x0), F.conv2d(xi, w, b)], 1e-5)

    # 3. residual block with downsample (ResNet stage entry), maxpool and global average pool
    g = GraphBuilder("golden:resblock")
    x = rnd(g, (2, 8, 12, 12), 10)
    att = lambda s, p: {"strides": _arr([s, s]), "padding": _arr([p, p]), "dilation": _arr([1, 1])}
    w1, b1 = rnd(g, (16, 8, 3, 3), 11, 0.2), rnd(g, (16,), 12, 0.01)
    w2, b2 = rnd(g, (16, 16, 3, 3), 13, 0.15), rnd(g, (16,), 14, 0.01)
    wd, bd = rnd(g, (16, 8, 1, 1), 15, 0.3), rnd(g, (16,), 16, 0.01)
    mp = g.op("max_pool", [x], {"kernelSize": _arr([3, 3]), "strides": _arr([1, 1]), "padding": _arr([1, 1]),
                                "dilation": _arr([1, 1]), "ceilMode": "false"}, "f32", (2, 8, 12, 12))
    y = g.relu(g.op("conv", [mp, w1, b1], att(2, 1), "f32", (2, 16, 6, 6)))
    y = g.op("conv", [y, w2, b2], att(1, 1), "f32", (2, 16, 6, 6))
    idn = g.op("conv", [mp, wd, bd], att(2, 0), "f32", (2, 16, 6, 6))
    h = g.relu(g.add(y, idn))
    gp = g.op("global_average_pool", [h], None, "f32", (2, 16, 1, 1))

    def resblock(x, w1, b1, w2, b2, wd, bd):
        m = F.max_pool2d(x, 3, 1, 1)
        y = F.relu(F.conv2d(m, w1, b1, 2, 1))
        y = F.conv2d(y, w2, b2, 1, 1)
        h = F.relu(y + F.conv2d(m, wd, bd, 2, 0))
        return [h, h.mean((2, 3), keepdim=True)]
    save("resblock", g, [h, gp], resblock, 1e-5)

    # 4. attention block with LayerNorm chain, masked softmax and GELU (BERT layer shape, small)
    g = GraphBuilder("golden:attention")
    s_, hid, nh = 16, 32, 2
    hd = hid // nh
    x = rnd(g, (1, s_, hid), 20)
    wq, wk, wv = rnd(g, (hid, hid), 21, 0.2), rnd(g, (hid, hid), 22, 0.2), rnd(g, (hid, hid), 23, 0.2)
    mean = g.reduce_mean(x, [-1])
    xc = g.sub(x, mean)
    var = g.reduce_mean(g.pow(xc, g.const(2.0, "f32")), [-1])
    ln = g.div(xc, g.sqrt(g.add(var, g.const(1e-12, "f32"))))
    q = g.transpose(g.reshape(g.matmul(ln, wq), (1, s_, nh, hd)), [0, 2, 1, 3])
    k = g.transpose(g.reshape(g.matmul(ln, wk), (1, s_, nh, hd)), [0, 2, 3, 1])
    v = g.transpose(g.reshape(g.matmul(ln, wv), (1, s_, nh, hd)), [0, 2, 1, 3])
    r = g.range_(0, s_, 1)
    allowed = g.less_equal(g.unsqueeze(r, [0]), g.unsqueeze(r, [1]))
    mask = g.where(allowed, g.const(0.0, "f32"), g.const(float("-inf"), "f32"))
    p = g.softmax(g.add(g.div(g.matmul(q, k), g.const(math.sqrt(hd), "f32")), mask), -1)
    o = g.reshape(g.transpose(g.matmul(p, v), [0, 2, 1, 3]), (1, s_, hid))
    gel = g.op("gelu", [o], None, "f32", o.shape)

    def attention(x, wq, wk, wv):
        m = x.mean(-1, keepdim=True)
        xc = x - m
        ln = xc / torch.sqrt((xc * xc).mean(-1, keepdim=True) + 1e-12)
        q = (ln @ wq).view(1, s_, nh, hd).transpose(1, 2)
        k = (ln @ wk).view(1, s_, nh, hd).transpose(1, 2)
        v = (ln @ wv).view(1, s_, nh, hd).transpose(1, 2)
        sc = q @ k.transpose(-1, -2) / math.sqrt(hd) + torch.full((s_, s_), float("-inf"), dtype=torch.float64).triu(1)
        o = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(1, s_, hid)
        return [o, F.gelu(o)]
    save("attention", g, [o, gel], attention, 2e-5)

    # 5. embedding gather + RoPE rotate-half (Sin/Cos/Neg/Slice/Concat)
    g = GraphBuilder("golden:rope")
    ids = g.input("i64", (2, 6), lambda: np.random.default_rng(30).integers(0, 40, (2, 6)))
    tab = rnd(g, (40, 8), 31)
    e = g.gather(tab, ids, 0)
    ang = g.mul(g.cast(g.unsqueeze(g.range_(0, 6, 1), [1]), 1, "f32"), g.const(np.full((1, 8), 0.7, np.float32), "f32"))
    x1 = g.slice(e, [0], [4], [2])
    x2 = g.slice(e, [4], [8], [2])
    rot = g.cat([g.neg(x2), x1], 2)
    out = g.add(g.mul(e, g.cos(ang)), g.mul(rot, g.sin(ang)))

    def rope(ids, tab):
        e = tab[ids]
        ang = torch.arange(6, dtype=torch.float64)[:, None] * torch.full((1, 8), float(np.float32(0.7)), dtype=torch.float64)
        rot = torch.cat([-e[..., 4:], e[..., :4]], -1)
        return [e * torch.cos(ang) + rot * torch.sin(ang)]
    save("rope", g, [out], rope, 1e-6)


if __name__ == "__main__":
    main()
