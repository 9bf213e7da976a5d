"""The drop-in boundary on the GPU: the reference's own runner ABI and tools
driving libgawee_cuda.

* `gawee_ciface_forward` / `gawee_embedded_forward` take the memref
  descriptors the reference's launcher builds (back/runtime_support.h:21-28)
  and return a malloc'ed result, as `_mlir_ciface_forward` does
  (back/gawee_aot.cpp:174-195).
* `gawee-cuda-runner` keeps the runner's file contract (argN.npy in,
  outputN.npy out; back/gawee_aot.cpp:226-289), byte-compatible with the
  oracle CLI's npy output.
* The launcher written by the reference's own `gawee-aot` (compiled from its
  sources into oracle/_ref by oracle/build_ref.py), linked with the ciface
  shim and -lgawee_cuda, runs the graph on the GPU; the reference's own
  `gawee-eval compare` checks its output against the oracle's, and
  `gawee-eval benchmark` drives it as it drives the CPU runner.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import oracle
from gawee_b200 import synth
from tests.helpers import compare

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
RUNNER = os.path.join(ROOT, "gawee_b200", "bin", "gawee-cuda-runner")

CTYPE = {np.dtype(np.float32): ctypes.c_float, np.dtype(np.int64): ctypes.c_int64,
         np.dtype(np.float64): ctypes.c_double, np.dtype(np.int32): ctypes.c_int32}


def memref_type(rank: int):
    """ctypes mirror of MemRefDescriptor<T, Rank> (back/runtime_support.h:21-28)."""
    class MemRef(ctypes.Structure):
        _fields_ = [("allocated", ctypes.c_void_p), ("aligned", ctypes.c_void_p), ("offset", ctypes.c_int64),
                    ("sizes", ctypes.c_int64 * max(rank, 1)), ("strides", ctypes.c_int64 * max(rank, 1))]
    return MemRef


def describe(a: np.ndarray, offset_elems: int = 0):
    """Descriptor of `a` as makeDescriptor builds it (dense C order); with an
    offset, `aligned` points offset_elems before the data."""
    desc = memref_type(a.ndim)()
    base = a.ctypes.data - offset_elems * a.itemsize
    desc.allocated = base
    desc.aligned = base
    desc.offset = offset_elems
    st = 1
    for d in range(a.ndim - 1, -1, -1):
        desc.sizes[d] = a.shape[d]
        desc.strides[d] = st
        st *= a.shape[d]
    return desc


def _result_array(desc, shape, dtype):
    n = int(np.prod(shape))
    ptr = desc.aligned + desc.offset * np.dtype(dtype).itemsize
    buf = (CTYPE[np.dtype(dtype)] * n).from_address(ptr)
    return np.ctypeslib.as_array(buf).reshape(shape).copy()


def test_ciface_forward_descriptors_and_malloced_result(cuda_lib):
    g = synth.resnet18(1, image=64)
    args = g.make_args()
    want = oracle.run(g.mlir, args)[0]
    libc = ctypes.CDLL(None)
    libc.free.argtypes = [ctypes.c_void_p]
    ctx = ctypes.c_void_p()
    assert cuda_lib.gawee_create(g.mlir.encode(), b"forward", 0, ctypes.byref(ctx)) == 0
    try:
        # the first argument is handed over with a non-zero descriptor offset
        padded = np.concatenate([np.full(7, np.nan, np.float32), args[0].ravel()])
        off = describe(padded[7:].reshape(args[0].shape), 7)  # aligned = padded's base, offset 7
        assert off.aligned == padded.ctypes.data
        descs = [off] + [describe(a) for a in args[1:]]
        ptrs = (ctypes.c_void_p * len(descs))(*[ctypes.addressof(d) for d in descs])
        for call in range(2):
            res = memref_type(want.ndim)()
            st = cuda_lib.gawee_ciface_forward(ctx, ctypes.addressof(res), ptrs, len(descs))
            assert st == 0, st
            assert res.offset == 0 and res.allocated == res.aligned and res.aligned
            assert tuple(res.sizes) == want.shape and tuple(res.strides) == (1000, 1)
            got = _result_array(res, want.shape, np.float32)
            libc.free(res.allocated)  # the caller owns the result, as in the reference ABI
            compare(got, want, 1e-4, 1e-4, f"ciface call {call}")
        # a descriptor that is not dense row-major is refused
        bad = describe(args[0])
        bad.strides[3] = 2
        ptrs[0] = ctypes.addressof(bad)
        res = memref_type(2)()
        assert cuda_lib.gawee_ciface_forward(ctx, ctypes.addressof(res), ptrs, len(descs)) == 1
        assert cuda_lib.gawee_ciface_forward(ctx, ctypes.addressof(res), ptrs, len(descs) - 1) == 1
    finally:
        cuda_lib.gawee_destroy(ctx)


def test_embedded_forward_plans_once_and_reports_errors(cuda_lib):
    g = synth.bert_tiny(seq=16, vocab=64, max_pos=32)
    args = g.make_args()
    want = oracle.run(g.mlir, args)[0]
    text = ctypes.create_string_buffer(g.mlir.encode())  # one address: the context cache key
    descs = [describe(a) for a in args]
    ptrs = (ctypes.c_void_p * len(descs))(*[ctypes.addressof(d) for d in descs])
    libc = ctypes.CDLL(None)
    libc.free.argtypes = [ctypes.c_void_p]
    for call in range(2):
        res = memref_type(3)()
        st = cuda_lib.gawee_embedded_forward(text, 0, ctypes.addressof(res), ptrs, len(descs))
        assert st == 0, st
        got = _result_array(res, want.shape, np.float32)
        libc.free(res.allocated)
        compare(got, want, 5e-4, 1e-4, f"embedded call {call}")
    # an out-of-range token id: the gather kernel flags it, the call fails with a message
    bad = args[0].copy()
    bad[0, 3] = 10_000
    descs[0] = describe(bad)
    ptrs[0] = ctypes.addressof(descs[0])
    res = memref_type(3)()
    st = cuda_lib.gawee_embedded_forward(text, 0, ctypes.addressof(res), ptrs, len(descs))
    assert st == 6  # GAWEE_ERR_DEVICE
    msg = ctypes.create_string_buffer(512)
    cuda_lib.gawee_last_error(None, msg, len(msg))
    assert msg.value, "no error message for the failed call"


def test_cuda_runner_file_contract(tmp_path):
    g = synth.bert_tiny(seq=16, vocab=64, max_pos=32)
    args = g.make_args()
    (tmp_path / "in").mkdir()
    for i, a in enumerate(args):
        np.save(tmp_path / "in" / f"arg{i}.npy", a)
    mlir = tmp_path / "m.mlir"
    mlir.write_text(g.mlir)
    oracle.build()
    r = subprocess.run([oracle.CLI_PATH, str(mlir), str(tmp_path / "in"), str(tmp_path / "want")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([RUNNER, str(mlir), str(tmp_path / "in"), str(tmp_path / "out")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got, want = np.load(tmp_path / "out" / "output0.npy"), np.load(tmp_path / "want" / "output0.npy")
    compare(got, want, 5e-4, 1e-4, "runner output0")
    with open(tmp_path / "out" / "output0.npy", "rb") as f1, open(tmp_path / "want" / "output0.npy", "rb") as f2:
        h1, h2 = f1.read(128), f2.read(128)
    hl = int.from_bytes(h1[8:10], "little")
    assert h1[:10 + hl] == h2[:10 + hl], "npy headers differ"
    # a missing input is an error with a non-zero exit, as in the reference runner
    os.remove(tmp_path / "in" / "arg5.npy")
    r = subprocess.run([RUNNER, str(mlir), str(tmp_path / "in"), str(tmp_path / "out2")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode != 0


def _ref_graph(name):
    import importlib.util
    spec = importlib.util.spec_from_file_location("build_ref", os.path.join(ROOT, "oracle", "build_ref.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.graph(name)


@pytest.mark.parametrize("name,atol", [("resnet18_b1_64", 1e-4), ("bert_tiny_s16", 5e-4)])
def test_reference_launcher_on_libgawee_cuda(tmp_path, name, atol):
    d = os.path.join(REF, "aot", name)
    runner = os.path.join(d, "runner")
    if not os.path.exists(runner):
        pytest.skip("oracle/_ref was not built (needs the reference's sources: python oracle/build_ref.py)")
    g = _ref_graph(name)
    with open(os.path.join(d, "forward.mlir")) as f:
        assert f.read() == g.mlir, "oracle/_ref launcher is stale: rerun python oracle/build_ref.py"
    args = g.make_args()
    (tmp_path / "in").mkdir()
    for i, a in enumerate(args):
        np.save(tmp_path / "in" / f"arg{i}.npy", a)
    oracle.build()
    r = subprocess.run([oracle.CLI_PATH, os.path.join(d, "forward.mlir"), str(tmp_path / "in"),
                        str(tmp_path / "want")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([runner, str(tmp_path / "in"), str(tmp_path / "out")], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    assert "[gawee-aot] done" in r.stderr
    # the reference's comparator (back/gawee_eval.cpp:97-128) on the two output directories
    r = subprocess.run([os.path.join(REF, "gawee-eval"), "compare", "--actual", str(tmp_path / "out"),
                        "--expected", str(tmp_path / "want"), "--atol", str(atol), "--rtol", "1e-4"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all outputs matched" in r.stdout
    compare(np.load(tmp_path / "out" / "output0.npy"), np.load(tmp_path / "want" / "output0.npy"), atol, 1e-4)
    # the reference's process-level benchmark (back/gawee_eval.cpp:130-186) drives the same runner
    r = subprocess.run([os.path.join(REF, "gawee-eval"), "benchmark", "--runner", runner, "--inputs",
                        str(tmp_path / "in"), "--outputs", str(tmp_path / "bench"), "--warmup", "1", "--iters", "2"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "p50" in r.stdout
