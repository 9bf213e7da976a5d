"""Synthetic gawee-dialect graphs for the five benchmark configurations.

The reference benchmarks real ONNX exports (torchvision ResNet-18, HF bert-tiny,
tinyllama-15M, SmolLM-135M) that are not available offline.  This module builds
the same architectures directly as gawee-dialect MLIR, in the form
`gawee-onnx-translate` prints for the corresponding ONNX graph
(middle/mlir/lib/Emit/ONNXMLIREmitter.cpp):

* `func.func @forward` takes the graph inputs first, then every float
  initializer as a runtime argument (ONNXMLIREmitter.cpp:2932-2975);
* integer initializers and Constant nodes become `arith.constant`
  (ONNXMLIREmitter.cpp:2982-2999, 2202-2238);
* Pow, Neg, Sin, Cos, Less, LessOrEqual, And, Mod and IsNaN are emitted directly
  as `linalg.generic` with a numpy broadcast map (ONNXMLIREmitter.cpp:420-476,
  846-1027, 2074-2124, 2348-2375), everything else as a `gawee.*` op in MLIR's
  generic operation syntax with inherent attributes as properties;
* Gemm becomes `gawee.linear` (2664-2746), Flatten becomes `gawee.reshape`
  with a constant shape (2630-2662), Conv/MaxPool pads are cut to their first
  two values (713-727, 1409-1418).

Weights and inputs are seeded numpy draws with the distributions named by the
workload definitions (Kaiming-normal conv weights with the BatchNorm folded into
a N(0, 0.01) conv bias; N(0, 0.02) transformer weights; LayerNorm gamma 1 / beta
0; uniform token ids).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

_NP_DTYPE = {"f32": np.float32, "f64": np.float64, "i64": np.int64, "i32": np.int32,
             "i1": np.bool_}


def type_str(dtype: str, shape: Sequence[int]) -> str:
    if len(shape) == 0:
        return f"tensor<{dtype}>"
    return "tensor<" + "x".join(str(int(d)) for d in shape) + f"x{dtype}>"


def _fmt_float(v: float) -> str:
    v = float(np.float32(v))
    if math.isinf(v):
        return "0xFF800000" if v < 0 else "0x7F800000"
    if math.isnan(v):
        return "0x7FC00000"
    s = f"{v:.6e}"
    if float(np.float32(float(s))) == v:
        return s
    return repr(float(np.float32(v))).replace("e", "E")


def _fmt_dense(arr: np.ndarray, dtype: str) -> str:
    """MLIR DenseElementsAttr payload: splat, nested list, or hex when large."""
    flat = arr.reshape(-1)
    if flat.size > 0 and np.all(flat == flat[0]):
        v = flat[0]
        return _fmt_float(v) if dtype.startswith("f") else (
            ("true" if v else "false") if dtype == "i1" else str(int(v)))
    if flat.size > 100:
        raw = np.ascontiguousarray(arr.astype(_NP_DTYPE[dtype])).tobytes()
        return '"0x' + raw.hex().upper() + '"'

    def rec(a):
        if a.ndim == 0:
            x = a.item()
            if dtype.startswith("f"):
                return _fmt_float(x)
            if dtype == "i1":
                return "true" if x else "false"
            return str(int(x))
        return "[" + ", ".join(rec(s) for s in a) + "]"
    return rec(arr)


@dataclass
class Val:
    name: str
    dtype: str
    shape: Tuple[int, ...]

    @property
    def type(self) -> str:
        return type_str(self.dtype, self.shape)


@dataclass
class ArgSpec:
    name: str
    dtype: str
    shape: Tuple[int, ...]
    kind: str  # "input" or "weight"
    make: Callable[[], np.ndarray] = field(repr=False, default=None)


def _broadcast_map(in_shape, out_shape) -> str:
    rank = len(out_shape)
    dims = ", ".join(f"d{i}" for i in range(rank))
    if len(in_shape) == 0:
        return f"affine_map<({dims}) -> ()>"
    lead = rank - len(in_shape)
    exprs = []
    for i, d in enumerate(in_shape):
        od = lead + i
        exprs.append("0" if (d == 1 and out_shape[od] != 1) else f"d{od}")
    return f"affine_map<({dims}) -> ({', '.join(exprs)})>"


def broadcast_shape(a, b):
    r = max(len(a), len(b))
    a = (1,) * (r - len(a)) + tuple(a)
    b = (1,) * (r - len(b)) + tuple(b)
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            raise ValueError(f"cannot broadcast {a} {b}")
        out.append(max(x, y))
    return tuple(out)


class GraphBuilder:
    """Builds one `func.func @forward` the way the ONNX emitter prints it."""

    def __init__(self, source: str, seed: int = 42):
        self.source = source
        self.rng = np.random.default_rng(seed)
        self.args: List[ArgSpec] = []
        self.lines: List[str] = []
        self.maps: Dict[str, str] = {}
        self._n = 0
        self._cst = 0
        self._empty_cache = None

    # -- values -----------------------------------------------------------
    def _new(self) -> str:
        n = f"%{self._n}"
        self._n += 1
        return n

    def _new_cst(self) -> str:
        n = "%cst" if self._cst == 0 else f"%cst_{self._cst - 1}"
        self._cst += 1
        return n

    def input(self, dtype: str, shape, make: Callable[[], np.ndarray]) -> Val:
        name = f"%arg{len(self.args)}"
        self.args.append(ArgSpec(name, dtype, tuple(shape), "input", make))
        return Val(name, dtype, tuple(shape))

    def weight(self, shape, make: Callable[[], np.ndarray]) -> Val:
        name = f"%arg{len(self.args)}"
        self.args.append(ArgSpec(name, "f32", tuple(shape), "weight", make))
        return Val(name, "f32", tuple(shape))

    def normal(self, shape, std: float) -> Val:
        seed = int(self.rng.integers(0, 2**63 - 1))

        def make():
            r = np.random.default_rng(seed)
            return (r.standard_normal(size=shape, dtype=np.float32) * np.float32(std))
        return self.weight(shape, make)

    def filled(self, shape, value: float) -> Val:
        return self.weight(shape, lambda: np.full(shape, value, dtype=np.float32))

    def const(self, values, dtype: str, shape=None) -> Val:
        arr = np.asarray(values, dtype=_NP_DTYPE[dtype])
        if shape is not None:
            arr = arr.reshape(shape)
        name = self._new_cst()
        t = type_str(dtype, arr.shape)
        self.lines.append(f"{name} = arith.constant dense<{_fmt_dense(arr, dtype)}> : {t}")
        return Val(name, dtype, tuple(arr.shape))

    def map_alias(self, text: str) -> str:
        if text not in self.maps:
            self.maps[text] = "#map" if not self.maps else f"#map{len(self.maps)}"
        return self.maps[text]

    # -- ops ----------------------------------------------------------------
    def op(self, name: str, operands: Sequence[Val], attrs: Optional[Dict[str, str]],
           out_dtype: str, out_shape) -> Val:
        res = self._new()
        props = ""
        if attrs:
            props = " <{" + ", ".join(f"{k} = {attrs[k]}" for k in sorted(attrs)) + "}>"
        ins = ", ".join(o.name for o in operands)
        tys = ", ".join(o.type for o in operands)
        out = Val(res, out_dtype, tuple(out_shape))
        self.lines.append(f'{res} = "gawee.{name}"({ins}){props} : ({tys}) -> {out.type}')
        return out

    def op_multi(self, name, operands, attrs, outs: Sequence[Tuple[str, tuple]]) -> List[Val]:
        res = self._new()
        props = ""
        if attrs:
            props = " <{" + ", ".join(f"{k} = {attrs[k]}" for k in sorted(attrs)) + "}>"
        ins = ", ".join(o.name for o in operands)
        tys = ", ".join(o.type for o in operands)
        vals = [Val(f"{res}#{i}", d, tuple(s)) for i, (d, s) in enumerate(outs)]
        out_tys = ", ".join(v.type for v in vals)
        self.lines.append(f'{res}:{len(vals)} = "gawee.{name}"({ins}){props} : ({tys}) -> ({out_tys})')
        return vals

    def generic(self, inputs: Sequence[Val], out_dtype: str, out_shape, body: Callable[[List[str]], List[str]]) -> Val:
        """`linalg.generic` with numpy-broadcast maps (ONNXMLIREmitter.cpp:420-476).

        `body` receives the block-argument names and returns body lines whose
        last defined value is yielded.
        """
        out_shape = tuple(out_shape)
        rank = len(out_shape)
        empty = self._new()
        ety = type_str(out_dtype, out_shape)
        self.lines.append(f"{empty} = tensor.empty() : {ety}")
        maps = [self.map_alias(_broadcast_map(v.shape, out_shape)) for v in inputs]
        maps.append(self.map_alias(_broadcast_map(out_shape, out_shape)))
        its = ", ".join(['"parallel"'] * rank)
        res = self._new()
        ins = ", ".join(v.name for v in inputs)
        tys = ", ".join(v.type for v in inputs)
        bnames = ["%in"] + [f"%in_{i}" for i in range(len(inputs) - 1)]
        bargs = ", ".join(f"{n}: {v.dtype}" for n, v in zip(bnames, inputs)) + f", %out: {out_dtype}"
        blines = body(bnames)
        self.lines.append(
            f"{res} = linalg.generic {{indexing_maps = [{', '.join(maps)}], iterator_types = [{its}]}} "
            f"ins({ins} : {tys}) outs({empty} : {ety}) {{")
        self.lines.append(f"^bb0({bargs}):")
        for bl in blines:
            self.lines.append("  " + bl)
        last = blines[-1].split("=")[0].strip()
        self.lines.append(f"  linalg.yield {last} : {out_dtype}")
        self.lines.append(f"}} -> {ety}")
        return Val(res, out_dtype, out_shape)

    # -- ONNX-node helpers (what the emitter produces for each ONNX op) -----
    def add(self, a, b):
        return self.op("add", [a, b], None, a.dtype, broadcast_shape(a.shape, b.shape))

    def sub(self, a, b):
        return self.op("sub", [a, b], None, a.dtype, broadcast_shape(a.shape, b.shape))

    def mul(self, a, b):
        return self.op("mul", [a, b], None, a.dtype, broadcast_shape(a.shape, b.shape))

    def div(self, a, b):
        return self.op("div", [a, b], None, a.dtype, broadcast_shape(a.shape, b.shape))

    def relu(self, x):
        return self.op("relu", [x], None, x.dtype, x.shape)

    def sigmoid(self, x):
        return self.op("sigmoid", [x], None, x.dtype, x.shape)

    def erf(self, x):
        return self.op("erf", [x], None, x.dtype, x.shape)

    def sqrt(self, x):
        return self.op("sqrt", [x], None, x.dtype, x.shape)

    def pow(self, x, y):
        shape = broadcast_shape(x.shape, y.shape)
        return self.generic([x, y], x.dtype, shape, lambda n: [f"%r = math.powf {n[0]}, {n[1]} : {x.dtype}"])

    def neg(self, x):
        return self.generic([x], x.dtype, x.shape, lambda n: [f"%r = arith.negf {n[0]} : {x.dtype}"])

    def sin(self, x):
        return self.generic([x], x.dtype, x.shape, lambda n: [f"%r = math.sin {n[0]} : {x.dtype}"])

    def cos(self, x):
        return self.generic([x], x.dtype, x.shape, lambda n: [f"%r = math.cos {n[0]} : {x.dtype}"])

    def less_equal(self, a, b):
        shape = broadcast_shape(a.shape, b.shape)
        pred = "arith.cmpf ole" if a.dtype.startswith("f") else "arith.cmpi sle"
        return self.generic([a, b], "i1", shape, lambda n: [f"%r = {pred}, {n[0]}, {n[1]} : {a.dtype}"])

    def matmul(self, a, b):
        batch = broadcast_shape(a.shape[:-2], b.shape[:-2])
        return self.op("matmul", [a, b], None, a.dtype, tuple(batch) + (a.shape[-2], b.shape[-1]))

    def linear(self, x, w, b):
        return self.op("linear", [x, w, b], None, x.dtype, x.shape[:-1] + (w.shape[0],))

    def reshape(self, x, shape):
        s = self.const(list(shape), "i64")
        return self.op("reshape", [x, s], None, x.dtype, tuple(shape))

    def transpose(self, x, perm):
        shape = tuple(x.shape[p] for p in perm)
        return self.op("transpose", [x], {"perm": _arr(perm)}, x.dtype, shape)

    def unsqueeze(self, x, axes):
        shape = list(x.shape)
        for a in sorted(axes):
            shape.insert(a, 1)
        return self.op("unsqueeze", [x], {"axes": _arr(axes)}, x.dtype, tuple(shape))

    def reduce_mean(self, x, axes, keepdims=True):
        r = len(x.shape)
        ax = sorted(a % r for a in axes)
        shape = [1 if i in ax else d for i, d in enumerate(x.shape)] if keepdims else \
            [d for i, d in enumerate(x.shape) if i not in ax]
        return self.op("reduce_mean", [x], {"axes": _arr(axes), "keepDims": "true" if keepdims else "false"},
                       x.dtype, tuple(shape))

    def softmax(self, x, axis=-1):
        return self.op("softmax", [x], {"axis": f"{axis % len(x.shape)} : i64"}, x.dtype, x.shape)

    def gather(self, data, idx, axis=0):
        shape = data.shape[:axis] + idx.shape + data.shape[axis + 1:]
        return self.op("gather", [data, idx], {"axis": f"{axis} : i64"}, data.dtype, shape)

    def slice(self, x, starts, ends, axes, steps=None):
        steps = steps or [1] * len(starts)
        shape = list(x.shape)
        for s, e, a, st in zip(starts, ends, axes, steps):
            d = x.shape[a]
            s2 = s + d if s < 0 else s
            e2 = e + d if e < 0 else min(e, d)
            shape[a] = (e2 - s2 + st - 1) // st
        cs = [self.const(v, "i64") for v in (starts, ends, axes, steps)]
        return self.op("slice", [x] + cs, None, x.dtype, tuple(shape))

    def cat(self, xs, axis):
        shape = list(xs[0].shape)
        shape[axis] = sum(v.shape[axis] for v in xs)
        return self.op("cat", list(xs), {"axis": f"{axis} : i64"}, xs[0].dtype, tuple(shape))

    def cast(self, x, to_onnx: int, dtype: str):
        return self.op("cast", [x], {"toType": f"{to_onnx} : i64"}, dtype, x.shape)

    def where(self, c, a, b):
        shape = broadcast_shape(broadcast_shape(c.shape, a.shape), b.shape)
        return self.op("where", [c, a, b], None, a.dtype, shape)

    def expand(self, x, shape):
        s = self.const(list(shape), "i64")
        return self.op("expand", [x, s], None, x.dtype, tuple(shape))

    def range_(self, start, limit, delta, dtype="i64"):
        n = max(0, (limit - start + delta - 1) // delta)
        cs = [self.const(v, dtype) for v in (start, limit, delta)]
        return self.op("range", cs, None, dtype, (n,))

    def finish(self, outputs: Sequence[Val]) -> str:
        args = ", ".join(f"{a.name}: {type_str(a.dtype, a.shape)}" for a in self.args)
        if len(outputs) == 1:
            rets = outputs[0].type
        else:
            rets = "(" + ", ".join(o.type for o in outputs) + ")"
        out = []
        for text, alias in self.maps.items():
            out.append(f"{alias} = {text}")
        out.append("module {")
        out.append(f'  func.func @forward({args}) -> {rets} attributes {{gawee.onnx_source = "{self.source}"}} {{')
        for ln in self.lines:
            out.append("    " + ln)
        out.append("    return " + ", ".join(o.name for o in outputs) + " : " +
                   ", ".join(o.type for o in outputs))
        out.append("  }")
        out.append("}")
        return "\n".join(out) + "\n"


def _arr(vals) -> str:
    vals = list(vals)
    if not vals:
        return "array<i64>"
    return "array<i64: " + ", ".join(str(int(v)) for v in vals) + ">"


@dataclass
class SynthGraph:
    """A built graph: MLIR text plus a recipe for its runtime arguments."""
    name: str
    mlir: str
    args: List[ArgSpec]
    out_shapes: List[Tuple[int, ...]]
    atol: float
    batch: int
    tokens_per_item: int
    flop: int

    def make_args(self) -> List[np.ndarray]:
        out = []
        for a in self.args:
            arr = np.ascontiguousarray(a.make())
            if arr.dtype != _NP_DTYPE[a.dtype] or tuple(arr.shape) != a.shape:
                raise AssertionError(f"arg {a.name}: {arr.dtype}{arr.shape} vs {a.dtype}{a.shape}")
            out.append(arr)
        return out


# ---------------------------------------------------------------------------
# ResNet-18 (configs 0 and 3)
# ---------------------------------------------------------------------------

def _conv(g: GraphBuilder, x: Val, cout: int, k: int, stride: int, pad: int, flops: list) -> Val:
    cin = x.shape[1]
    fan_in = cin * k * k
    std = math.sqrt(2.0 / fan_in)
    w = g.normal((cout, cin, k, k), std)
    b = g.normal((cout,), 0.01)
    n, _, h, wd = x.shape
    ho = (h + 2 * pad - k) // stride + 1
    wo = (wd + 2 * pad - k) // stride + 1
    flops[0] += 2 * n * cout * ho * wo * cin * k * k
    return g.op("conv", [x, w, b], {"strides": _arr([stride, stride]), "padding": _arr([pad, pad]),
                                    "dilation": _arr([1, 1])}, "f32", (n, cout, ho, wo))


def resnet18(batch: int = 1, image: int = 224, widths=(64, 128, 256, 512), classes: int = 1000,
             seed: int = 42) -> SynthGraph:
    g = GraphBuilder(f"synthetic:resnet18_b{batch}", seed)
    flops = [0]
    x = g.input("f32", (batch, 3, image, image),
                lambda: np.random.default_rng(seed + 1).standard_normal((batch, 3, image, image), dtype=np.float32))
    h = g.relu(_conv(g, x, widths[0], 7, 2, 3, flops))
    n, c, hh, ww = h.shape
    ho, wo = (hh + 2 - 3) // 2 + 1, (ww + 2 - 3) // 2 + 1
    h = g.op("max_pool", [h], {"kernelSize": _arr([3, 3]), "strides": _arr([2, 2]), "padding": _arr([1, 1]),
                               "dilation": _arr([1, 1]), "ceilMode": "false"}, "f32", (n, c, ho, wo))
    cin = widths[0]
    for si, cout in enumerate(widths):
        for bi in range(2):
            stride = 2 if (si > 0 and bi == 0) else 1
            identity = h
            y = g.relu(_conv(g, h, cout, 3, stride, 1, flops))
            y = _conv(g, y, cout, 3, 1, 1, flops)
            if stride != 1 or cin != cout:
                identity = _conv(g, h, cout, 1, stride, 0, flops)
            h = g.relu(g.add(y, identity))
            cin = cout
    n, c = h.shape[0], h.shape[1]
    h = g.op("global_average_pool", [h], None, "f32", (n, c, 1, 1))
    h = g.reshape(h, (n, c))
    wfc = g.normal((classes, c), 1.0 / math.sqrt(c))
    bfc = g.normal((classes,), 0.01)
    flops[0] += 2 * n * c * classes
    y = g.linear(h, wfc, bfc)
    return SynthGraph(f"resnet18_b{batch}", g.finish([y]), g.args, [y.shape], 1e-4, batch, 1, flops[0])


# ---------------------------------------------------------------------------
# BERT-tiny encoder (config 1)
# ---------------------------------------------------------------------------

def _layer_norm(g: GraphBuilder, x: Val, eps: float) -> Val:
    d = x.shape[-1]
    gamma = g.filled((d,), 1.0)
    beta = g.filled((d,), 0.0)
    mean = g.reduce_mean(x, [-1])
    xc = g.sub(x, mean)
    var = g.reduce_mean(g.pow(xc, g.const(2.0, "f32")), [-1])
    std = g.sqrt(g.add(var, g.const(eps, "f32")))
    return g.add(g.mul(g.div(xc, std), gamma), beta)


def _dense(g: GraphBuilder, x: Val, din: int, dout: int, flops: list, bias: bool = True) -> Val:
    w = g.normal((din, dout), 0.02)
    rows = int(np.prod(x.shape[:-1]))
    flops[0] += 2 * rows * din * dout
    y = g.matmul(x, w)
    if bias:
        y = g.add(y, g.normal((dout,), 0.02))
    return y


def bert_tiny(batch: int = 1, seq: int = 128, hidden: int = 128, layers: int = 2, heads: int = 2,
              ffn: int = 512, vocab: int = 30522, max_pos: int = 512, type_vocab: int = 2,
              seed: int = 42) -> SynthGraph:
    g = GraphBuilder(f"synthetic:bert_tiny_s{seq}", seed)
    flops = [0]
    hd = hidden // heads
    ids = g.input("i64", (batch, seq), lambda: np.random.default_rng(seed + 1).integers(0, vocab, (batch, seq), dtype=np.int64))
    tt = g.input("i64", (batch, seq), lambda: np.zeros((batch, seq), dtype=np.int64))
    mask = g.input("i64", (batch, seq), lambda: np.ones((batch, seq), dtype=np.int64))
    wemb = g.normal((vocab, hidden), 0.02)
    pemb = g.normal((max_pos, hidden), 0.02)
    temb = g.normal((type_vocab, hidden), 0.02)
    pos_ids = g.const(np.arange(max_pos, dtype=np.int64).reshape(1, max_pos), "i64")
    pos = g.slice(pos_ids, [0], [seq], [1])
    e = g.add(g.add(g.gather(wemb, ids), g.gather(temb, tt)), g.gather(pemb, pos))
    h = _layer_norm(g, e, 1e-12)
    m = g.unsqueeze(g.unsqueeze(mask, [1]), [2])
    m = g.cast(m, 1, "f32")
    m = g.mul(g.sub(g.const(1.0, "f32"), m), g.const(float(np.finfo(np.float32).min), "f32"))
    scale = g.const(math.sqrt(hd), "f32")
    for _ in range(layers):
        q = g.transpose(g.reshape(_dense(g, h, hidden, hidden, flops), (batch, seq, heads, hd)), [0, 2, 1, 3])
        k = g.transpose(g.reshape(_dense(g, h, hidden, hidden, flops), (batch, seq, heads, hd)), [0, 2, 3, 1])
        v = g.transpose(g.reshape(_dense(g, h, hidden, hidden, flops), (batch, seq, heads, hd)), [0, 2, 1, 3])
        s = g.add(g.div(g.matmul(q, k), scale), m)
        flops[0] += 2 * batch * heads * seq * seq * hd * 2
        p = g.softmax(s, -1)
        ctx = g.reshape(g.transpose(g.matmul(p, v), [0, 2, 1, 3]), (batch, seq, hidden))
        h = _layer_norm(g, g.add(_dense(g, ctx, hidden, hidden, flops), h), 1e-12)
        f = _dense(g, h, hidden, ffn, flops)
        f = g.mul(g.mul(f, g.add(g.erf(g.div(f, g.const(1.4142135381698608, "f32"))), g.const(1.0, "f32"))),
                  g.const(0.5, "f32"))
        h = _layer_norm(g, g.add(_dense(g, f, ffn, hidden, flops), h), 1e-12)
    return SynthGraph(f"bert_tiny_s{seq}", g.finish([h]), g.args, [h.shape], 5e-4, batch, seq, flops[0])


# ---------------------------------------------------------------------------
# Llama-style decoders (configs 2 and 4)
# ---------------------------------------------------------------------------

def _rms_norm(g: GraphBuilder, x: Val, eps: float) -> Val:
    w = g.filled((x.shape[-1],), 1.0)
    ms = g.reduce_mean(g.pow(x, g.const(2.0, "f32")), [-1])
    return g.mul(g.div(x, g.sqrt(g.add(ms, g.const(eps, "f32")))), w)


def _rotate_half(g: GraphBuilder, x: Val) -> Val:
    d = x.shape[-1]
    r = len(x.shape) - 1
    x1 = g.slice(x, [0], [d // 2], [r])
    x2 = g.slice(x, [d // 2], [d], [r])
    return g.cat([g.neg(x2), x1], r)


def llama(batch: int = 1, seq: int = 256, dim: int = 288, layers: int = 6, heads: int = 6,
          kv_heads: Optional[int] = None, ffn: int = 768, vocab: int = 32000, eps: float = 1e-5,
          theta: float = 10000.0, seed: int = 42, name: str = "llama15m") -> SynthGraph:
    kv_heads = kv_heads or heads
    rep = heads // kv_heads
    hd = dim // heads
    g = GraphBuilder(f"synthetic:{name}_b{batch}_s{seq}", seed)
    flops = [0]
    ids = g.input("i64", (batch, seq), lambda: np.random.default_rng(seed + 1).integers(0, vocab, (batch, seq), dtype=np.int64))
    emb = g.normal((vocab, dim), 0.02)
    h = g.gather(emb, ids)
    # RoPE tables: positions (Range) x inv_freq, duplicated, then cos/sin.
    inv = g.const((1.0 / (theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))).astype(np.float32).reshape(1, hd // 2), "f32")
    pos = g.cast(g.unsqueeze(g.range_(0, seq, 1), [1]), 1, "f32")          # [S,1]
    freqs = g.mul(pos, inv)                                                 # [S,hd/2]
    embp = g.cat([freqs, freqs], 1)                                         # [S,hd]
    cos = g.unsqueeze(g.cos(embp), [0, 1])                                  # [1,1,S,hd]
    sin = g.unsqueeze(g.sin(embp), [0, 1])
    # causal mask: key index j <= query index i -> 0, else -inf
    r = g.range_(0, seq, 1)
    allowed = g.less_equal(g.unsqueeze(r, [0]), g.unsqueeze(r, [1]))       # [S,S]
    mask = g.where(allowed, g.const(0.0, "f32"), g.const(float("-inf"), "f32"))
    scale = g.const(math.sqrt(hd), "f32")
    for _ in range(layers):
        x = _rms_norm(g, h, eps)
        q = g.transpose(g.reshape(_dense(g, x, dim, heads * hd, flops, False), (batch, seq, heads, hd)), [0, 2, 1, 3])
        k = g.transpose(g.reshape(_dense(g, x, dim, kv_heads * hd, flops, False), (batch, seq, kv_heads, hd)), [0, 2, 1, 3])
        v = g.transpose(g.reshape(_dense(g, x, dim, kv_heads * hd, flops, False), (batch, seq, kv_heads, hd)), [0, 2, 1, 3])
        q = g.add(g.mul(q, cos), g.mul(_rotate_half(g, q), sin))
        k = g.add(g.mul(k, cos), g.mul(_rotate_half(g, k), sin))
        if rep > 1:
            k = g.reshape(g.expand(g.unsqueeze(k, [2]), (batch, kv_heads, rep, seq, hd)), (batch, heads, seq, hd))
            v = g.reshape(g.expand(g.unsqueeze(v, [2]), (batch, kv_heads, rep, seq, hd)), (batch, heads, seq, hd))
        s = g.add(g.div(g.matmul(q, g.transpose(k, [0, 1, 3, 2])), scale), mask)
        flops[0] += 2 * batch * heads * seq * seq * hd * 2
        p = g.softmax(s, -1)
        o = g.reshape(g.transpose(g.matmul(p, v), [0, 2, 1, 3]), (batch, seq, heads * hd))
        h = g.add(h, _dense(g, o, heads * hd, dim, flops, False))
        x = _rms_norm(g, h, eps)
        gate = _dense(g, x, dim, ffn, flops, False)
        up = _dense(g, x, dim, ffn, flops, False)
        act = g.mul(g.mul(gate, g.sigmoid(gate)), up)
        h = g.add(h, _dense(g, act, ffn, dim, flops, False))
    h = _rms_norm(g, h, eps)
    flops[0] += 2 * batch * seq * dim * vocab
    logits = g.matmul(h, g.transpose(emb, [1, 0]))
    return SynthGraph(f"{name}_b{batch}_s{seq}", g.finish([logits]), g.args, [logits.shape], 5e-4,
                      batch, seq, flops[0])


def llama_decode(batch: int = 1, past: int = 1, dim: int = 288, layers: int = 6, heads: int = 6,
                 kv_heads: Optional[int] = None, ffn: int = 768, vocab: int = 32000, eps: float = 1e-5,
                 theta: float = 10000.0, seed: int = 42, name: str = "llama15m_decode",
                 present: bool = True) -> SynthGraph:
    """One KV-cache decode step, with the inputs of the reference's tinyllama
    binding (eval_priority_models.py:38-54): input_ids [B, 1],
    attention_mask [B, past + 1] (1 = attend), position_ids [B, 1], then per
    layer past key and value [B, kv_heads, past, head_dim].  Each layer
    appends the new key and value to the past ones (Concat on the sequence
    axis), rotates the new query and key by position_ids (RoPE), and attends
    over all past + 1 positions; masked positions get -inf.  Outputs: logits
    [B, 1, vocab], then (present=True) each layer's present key and value
    [B, kv_heads, past + 1, head_dim], the next step's past."""
    kv_heads = kv_heads or heads
    rep = heads // kv_heads
    hd = dim // heads
    total = past + 1
    g = GraphBuilder(f"synthetic:{name}_b{batch}_p{past}", seed)
    flops = [0]
    rng = np.random.default_rng(seed + 1)
    ids_v = rng.integers(0, vocab, (batch, 1), dtype=np.int64)
    mask_v = np.ones((batch, total), np.int64)
    if past >= 2:
        mask_v[:, 0] = 0  # a padded first position: exercises the mask
    pos_v = np.full((batch, 1), past, np.int64)
    ids = g.input("i64", (batch, 1), lambda: ids_v)
    am = g.input("i64", (batch, total), lambda: mask_v)
    pid = g.input("i64", (batch, 1), lambda: pos_v)
    pasts = []
    for li in range(layers):
        kv = [np.random.default_rng(seed + 100 + 2 * li + j).standard_normal((batch, kv_heads, past, hd),
                                                                          dtype=np.float32) for j in (0, 1)]
        pasts.append((g.input("f32", (batch, kv_heads, past, hd), lambda a=kv[0]: a),
                      g.input("f32", (batch, kv_heads, past, hd), lambda a=kv[1]: a)))
    emb = g.normal((vocab, dim), 0.02)
    h = g.gather(emb, ids)                                                  # [B,1,dim]
    inv = g.const((1.0 / (theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))).astype(np.float32).reshape(1, hd // 2), "f32")
    pos = g.unsqueeze(g.cast(pid, 1, "f32"), [2])                           # [B,1,1]
    freqs = g.mul(pos, inv)                                                 # [B,1,hd/2]
    embp = g.cat([freqs, freqs], 2)                                         # [B,1,hd]
    cos = g.unsqueeze(g.cos(embp), [1])                                     # [B,1,1,hd]
    sin = g.unsqueeze(g.sin(embp), [1])
    masked = g.less_equal(am, g.const(0, "i64"))                            # [B,total]
    mask = g.unsqueeze(g.where(masked, g.const(float("-inf"), "f32"), g.const(0.0, "f32")), [1, 2])  # [B,1,1,total]
    scale = g.const(math.sqrt(hd), "f32")
    presents = []
    for li in range(layers):
        x = _rms_norm(g, h, eps)
        q = g.transpose(g.reshape(_dense(g, x, dim, heads * hd, flops, False), (batch, 1, heads, hd)), [0, 2, 1, 3])
        k = g.transpose(g.reshape(_dense(g, x, dim, kv_heads * hd, flops, False), (batch, 1, kv_heads, hd)), [0, 2, 1, 3])
        v = g.transpose(g.reshape(_dense(g, x, dim, kv_heads * hd, flops, False), (batch, 1, kv_heads, hd)), [0, 2, 1, 3])
        q = g.add(g.mul(q, cos), g.mul(_rotate_half(g, q), sin))
        k = g.add(g.mul(k, cos), g.mul(_rotate_half(g, k), sin))
        kc = g.cat([pasts[li][0], k], 2)                                    # [B,kv_heads,total,hd]
        vc = g.cat([pasts[li][1], v], 2)
        presents += [kc, vc]
        if rep > 1:
            kc = g.reshape(g.expand(g.unsqueeze(kc, [2]), (batch, kv_heads, rep, total, hd)), (batch, heads, total, hd))
            vc = g.reshape(g.expand(g.unsqueeze(vc, [2]), (batch, kv_heads, rep, total, hd)), (batch, heads, total, hd))
        s = g.add(g.div(g.matmul(q, g.transpose(kc, [0, 1, 3, 2])), scale), mask)
        flops[0] += 2 * batch * heads * total * hd * 2
        o = g.reshape(g.transpose(g.matmul(g.softmax(s, -1), vc), [0, 2, 1, 3]), (batch, 1, heads * hd))
        h = g.add(h, _dense(g, o, heads * hd, dim, flops, False))
        x = _rms_norm(g, h, eps)
        gate = _dense(g, x, dim, ffn, flops, False)
        up = _dense(g, x, dim, ffn, flops, False)
        h = g.add(h, _dense(g, g.mul(g.mul(gate, g.sigmoid(gate)), up), ffn, dim, flops, False))
    h = _rms_norm(g, h, eps)
    flops[0] += 2 * batch * dim * vocab
    logits = g.matmul(h, g.transpose(emb, [1, 0]))
    outs = [logits] + (presents if present else [])
    return SynthGraph(f"{name}_b{batch}_p{past}", g.finish(outs), g.args, [o.shape for o in outs], 5e-4,
                      batch, 1, flops[0])


def llama15m_decode(batch: int = 1, past: int = 1, **kw) -> SynthGraph:
    """Tinyllama-15M's decode step; past = 1 is the reference binding's static shape."""
    return llama_decode(batch, past, dim=288, layers=6, heads=6, ffn=768, vocab=32000, name="llama15m_decode", **kw)


def llama15m(batch: int = 1, seq: int = 256, **kw) -> SynthGraph:
    return llama(batch, seq, dim=288, layers=6, heads=6, ffn=768, vocab=32000, name="llama15m", **kw)


def smollm135m(batch: int = 64, seq: int = 512, **kw) -> SynthGraph:
    return llama(batch, seq, dim=576, layers=30, heads=9, kv_heads=3, ffn=1536, vocab=49152,
                 name="decoder135m", **kw)


CONFIGS = {
    "resnet18_b1": lambda: resnet18(1),
    "bert_tiny": lambda: bert_tiny(),
    "llama15m": lambda: llama15m(),
    "resnet18_b256": lambda: resnet18(256),
    "decoder135m": lambda: smollm135m(),
}
