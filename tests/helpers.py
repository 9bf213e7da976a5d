"""Shared helpers: single-op graph construction and CUDA-vs-oracle parity checks."""
from __future__ import annotations

from typing import Callable, List, Sequence

import numpy as np

from gawee_b200.synth import GraphBuilder, Val, _arr  # noqa: F401  (re-exported for tests)


def build(fn: Callable[[GraphBuilder], Sequence[Val]], seed: int = 0):
    """Build a graph with `fn(g)` returning the outputs; returns (mlir, args)."""
    g = GraphBuilder("synthetic:test", seed)
    outs = fn(g)
    if isinstance(outs, Val):
        outs = [outs]
    mlir = g.finish(list(outs))
    args = [np.ascontiguousarray(a.make()) for a in g.args]
    return mlir, args


def rand_input(g: GraphBuilder, shape, seed: int, scale: float = 1.0, dtype: str = "f32", lo=None, hi=None):
    shape = tuple(shape)

    def make():
        r = np.random.default_rng(seed)
        if dtype == "f32":
            return (r.standard_normal(shape, dtype=np.float32) * np.float32(scale))
        if dtype == "i64":
            return r.integers(lo if lo is not None else 0, hi if hi is not None else 10, shape, dtype=np.int64)
        if dtype == "i1":
            return r.integers(0, 2, shape).astype(np.bool_)
        raise ValueError(dtype)
    return g.input(dtype, shape, make)


def compare(got: np.ndarray, want: np.ndarray, atol: float, rtol: float, what: str = ""):
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    assert got.dtype == want.dtype, f"{what}: dtype {got.dtype} vs {want.dtype}"
    if np.issubdtype(want.dtype, np.floating):
        nan_g, nan_w = np.isnan(got), np.isnan(want)
        assert np.array_equal(nan_g, nan_w), f"{what}: NaN positions differ"
        ok = ~nan_w
        g64, w64 = got[ok].astype(np.float64), want[ok].astype(np.float64)
        with np.errstate(invalid="ignore"):
            diff = np.where(g64 == w64, 0.0, np.abs(g64 - w64))
            bound = atol + rtol * np.abs(w64)  # NaN for an infinite want with rtol 0: equality decides there
            within = (g64 == w64) | (diff <= bound)
        if diff.size:
            k = int(np.argmin(within))
            assert np.all(within), (f"{what}: max_abs_diff={diff.max():.3e} worst at flat {k}: "
                                    f"got {got[ok].ravel()[k]!r} want {want[ok].ravel()[k]!r}")
        return float(diff.max()) if diff.size else 0.0
    assert np.array_equal(got, want), f"{what}: integer/bool outputs differ at {np.argwhere(got != want)[:5]}"
    return 0.0


def parity_line(what: str, got: np.ndarray, want: np.ndarray, atol: float, rtol: float) -> str:
    """One line of the parity table (printed by the model tests under -s):
    max |got - want|, max |want|, and the worst |got - want| / (atol + rtol |want|),
    the fraction of the reference tolerance used (below 1 passes)."""
    g64, w64 = got.astype(np.float64), want.astype(np.float64)
    ok = np.isfinite(w64)
    diff = np.abs(g64[ok] - w64[ok])
    ratio = float(np.max(diff / (atol + rtol * np.abs(w64[ok])))) if diff.size else 0.0
    line = (f"PARITY {what}: max_abs_diff={float(diff.max()) if diff.size else 0.0:.3e} "
            f"max_abs_ref={float(np.max(np.abs(w64[ok]))) if diff.size else 0.0:.3e} "
            f"tolerance_used={ratio:.3f} (atol {atol:g}, rtol {rtol:g})")
    print(line)
    return line


def parity(mlir: str, args: List[np.ndarray], atol: float = 1e-5, rtol: float = 1e-5, runs: int = 1,
           graph_mode: bool = True):
    """Run the graph on the CUDA backend and on the oracle; assert they agree."""
    import oracle
    from gawee_b200.runtime import Model

    want = oracle.run(mlir, args)
    m = Model(mlir, graph_mode=graph_mode)
    try:
        for _ in range(runs):
            got = m.run(args)
            for k, (a, b) in enumerate(zip(got, want)):
                compare(a, b, atol, rtol, f"output{k}")
    finally:
        m.close()
    return got, want
