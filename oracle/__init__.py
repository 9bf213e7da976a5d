"""CPU oracle for gawee-dialect graphs — test infrastructure only.

`Oracle(mlir_text).run(args)` executes a graph with the C++ restatement of the
reference's lowering semantics in `gawee_oracle.cpp`.  Only the tests, the
smoke check and the CPU-baseline leg of the benchmark use it, as the checker;
the CUDA backend never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libgawee_oracle.so")
CLI_PATH = os.path.join(HERE, "_build", "gawee-oracle")

# DType numbering shared with gawee_b200/csrc/host/ir.h
NP_OF_DTYPE = {0: np.float32, 1: np.float64, 3: np.int64, 4: np.int32, 5: np.bool_, 6: np.int64}

_lock = threading.Lock()
_lib = None


def _sources() -> List[str]:
    return [os.path.join(HERE, "gawee_oracle.cpp"), os.path.join(HERE, "gawee_oracle_cli.cpp"),
            os.path.join(HERE, "..", "gawee_b200", "csrc", "host", "ir.cpp"),
            os.path.join(HERE, "..", "gawee_b200", "csrc", "host", "ir.h"),
            os.path.join(HERE, "..", "gawee_b200", "csrc", "host", "npy.h"),
            os.path.join(HERE, "Makefile")]


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile if any source is newer than the library."""
    newest = max(os.path.getmtime(p) for p in _sources())
    if not force and os.path.exists(LIB_PATH) and os.path.exists(CLI_PATH) and \
            min(os.path.getmtime(LIB_PATH), os.path.getmtime(CLI_PATH)) >= newest:
        return LIB_PATH
    subprocess.run(["make", "-s", "-C", HERE, "-j4"], check=True)
    return LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            build()
            lib = ctypes.CDLL(LIB_PATH)
            lib.gawee_oracle_load.restype = ctypes.c_void_p
            lib.gawee_oracle_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
            lib.gawee_oracle_free.argtypes = [ctypes.c_void_p]
            lib.gawee_oracle_num_args.argtypes = [ctypes.c_void_p]
            lib.gawee_oracle_num_outputs.argtypes = [ctypes.c_void_p]
            for f in (lib.gawee_oracle_arg_info, lib.gawee_oracle_output_info):
                f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                              ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64)]
            lib.gawee_oracle_run.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                             ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                             ctypes.c_char_p, ctypes.c_int]
            _lib = lib
    return _lib


class OracleError(RuntimeError):
    pass


class Oracle:
    def __init__(self, mlir_text: str, entry: str = "forward"):
        self._lib = _load()
        err = ctypes.create_string_buffer(2048)
        self._h = self._lib.gawee_oracle_load(mlir_text.encode(), entry.encode(), err, len(err))
        if not self._h:
            raise OracleError(err.value.decode())

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.gawee_oracle_free(h)
            self._h = None

    def _info(self, fn, i):
        dt, rk = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 8)()
        fn(self._h, i, ctypes.byref(dt), ctypes.byref(rk), shape)
        return NP_OF_DTYPE[dt.value], tuple(shape[k] for k in range(rk.value))

    def arg_specs(self):
        return [self._info(self._lib.gawee_oracle_arg_info, i) for i in range(self._lib.gawee_oracle_num_args(self._h))]

    def output_specs(self):
        return [self._info(self._lib.gawee_oracle_output_info, i)
                for i in range(self._lib.gawee_oracle_num_outputs(self._h))]

    def run(self, args: Sequence[np.ndarray], threads: int = 0) -> List[np.ndarray]:
        specs = self.arg_specs()
        if len(args) != len(specs):
            raise OracleError(f"expected {len(specs)} arguments, got {len(args)}")
        keep = []
        for a, (dt, shape) in zip(args, specs):
            a = np.ascontiguousarray(a)
            if a.dtype != np.dtype(dt) or tuple(a.shape) != shape:
                raise OracleError(f"argument {a.dtype}{a.shape} does not match {np.dtype(dt)}{shape}")
            keep.append(a)
        outs = [np.empty(shape, dtype=dt) for dt, shape in self.output_specs()]
        aptr = (ctypes.c_void_p * len(keep))(*[a.ctypes.data for a in keep])
        optr = (ctypes.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        err = ctypes.create_string_buffer(2048)
        rc = self._lib.gawee_oracle_run(self._h, aptr, optr, threads, err, len(err))
        if rc:
            raise OracleError(err.value.decode())
        return outs


def run(mlir_text: str, args: Sequence[np.ndarray], threads: int = 0, entry: str = "forward") -> List[np.ndarray]:
    return Oracle(mlir_text, entry).run(args, threads)
