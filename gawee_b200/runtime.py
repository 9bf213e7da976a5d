"""Python host API over the libgawee_cuda C ABI (include/gawee_cuda.h).

`Model` plays the role of the reference's generated AOT runner
(back/gawee_aot.cpp:226-289): it binds the `forward` arguments (graph inputs,
then float initializers), runs the compiled graph and returns the outputs —
on a B200 instead of the host CPU.  `run_dir` keeps the runner's file
contract (argN.npy in, outputN.npy out).

There is no CPU path: if the CUDA library cannot be loaded or no GPU is
present, creating a Model raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgawee_cuda.so")

# dtype numbering of include/gawee_cuda.h
NP_OF_DTYPE = {0: np.float32, 1: np.float64, 3: np.int64, 4: np.int32, 5: np.bool_}
STATUS = {0: "ok", 1: "invalid", 2: "parse", 3: "unsupported", 4: "cuda", 5: "oom", 6: "device", 7: "nccl"}

_lock = threading.Lock()
_lib = None


class GaweeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[{STATUS.get(status, status)}] {msg}")
        self.status = status


def load_library(path: str = LIB_PATH):
    """Load libgawee_cuda.so (building it first if missing)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            from . import build
            build.build()
        lib = ctypes.CDLL(path)
        c = ctypes
        P = c.c_void_p
        sig = {
            "gawee_create": (c.c_int, [c.c_char_p, c.c_char_p, c.c_int, c.POINTER(P)]),
            "gawee_create_from_file": (c.c_int, [c.c_char_p, c.c_char_p, c.c_int, c.POINTER(P)]),
            "gawee_destroy": (None, [P]),
            "gawee_last_error": (c.c_int, [P, c.c_char_p, c.c_size_t]),
            "gawee_num_args": (c.c_int, [P]),
            "gawee_num_outputs": (c.c_int, [P]),
            "gawee_arg_info": (c.c_int, [P, c.c_int, c.POINTER(c.c_int), c.POINTER(c.c_int), c.POINTER(c.c_int64)]),
            "gawee_output_info": (c.c_int, [P, c.c_int, c.POINTER(c.c_int), c.POINTER(c.c_int), c.POINTER(c.c_int64)]),
            "gawee_set_arg": (c.c_int, [P, c.c_int, P, c.c_size_t, P]),
            "gawee_set_arg_device": (c.c_int, [P, c.c_int, P, c.c_size_t, P]),
            "gawee_forward": (c.c_int, [P, P]),
            "gawee_get_output": (c.c_int, [P, c.c_int, P, c.c_size_t, P]),
            "gawee_output_device_ptr": (c.c_int, [P, c.c_int, c.POINTER(P)]),
            "gawee_synchronize": (c.c_int, [P, P]),
            "gawee_set_graph_mode": (c.c_int, [P, c.c_int]),
            "gawee_set_precision": (c.c_int, [P, c.c_int]),
            "gawee_probe_tf32_mma": (c.c_int, [c.c_int, c.POINTER(c.c_double)]),
            "gawee_precision": (c.c_int, [P]),
            "gawee_plan_text": (c.c_int, [c.c_char_p, c.c_char_p, c.c_char_p, c.c_size_t]),
            "gawee_num_kernels": (c.c_int, [P]),
            "gawee_num_launches": (c.c_int, [P]),
            "gawee_plan_summary": (c.c_int, [P, c.c_char_p, c.c_size_t]),
            "gawee_op_info": (c.c_int, [P, c.c_int, c.c_char_p, c.c_size_t, c.POINTER(c.c_int),
                                        c.POINTER(c.c_double)]),
            "gawee_profile_forward": (c.c_int, [P, P, c.POINTER(c.c_float), c.c_int]),
            "gawee_ciface_forward": (c.c_int, [P, P, c.POINTER(P), c.c_int]),
            "gawee_embedded_forward": (c.c_int, [c.c_char_p, c.c_int, P, c.POINTER(P), c.c_int]),
            "gawee_matmul_f32_noalloc": (c.c_int, [P, P, P, c.c_int64, c.c_int64, c.c_int64, P]),
            "gawee_dp_unique_id": (c.c_int, [P]),
            "gawee_dp_init": (c.c_int, [P, c.c_int, c.c_int, P]),
            "gawee_dp_gather_output": (c.c_int, [P, c.c_int, P, P]),
            "gawee_dp_output_bytes": (c.c_int, [P, c.c_int, c.POINTER(c.c_size_t)]),
        }
        for name, (res, args) in sig.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
        return lib


def plan_text(mlir: str, entry: str = "forward") -> str:
    """Plan a graph without a GPU and return the plan summary (raises on error)."""
    lib = load_library()
    buf = ctypes.create_string_buffer(1 << 20)
    st = lib.gawee_plan_text(mlir.encode(), entry.encode(), buf, len(buf))
    if st:
        raise GaweeError(st, buf.value.decode())
    return buf.value.decode()


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream", stream))


class Model:
    """A gawee `forward` function compiled for one B200."""

    PRECISIONS = {"fp32": 0, "tf32": 1, "bf16": 2}

    def __init__(self, mlir: str, device: int = 0, entry: str = "forward", graph_mode: bool = True,
                 precision: Optional[str] = None):
        self._lib = load_library()
        h = ctypes.c_void_p()
        st = self._lib.gawee_create(mlir.encode(), entry.encode(), device, ctypes.byref(h))
        if st:
            buf = ctypes.create_string_buffer(4096)
            self._lib.gawee_last_error(None, buf, len(buf))
            raise GaweeError(st, buf.value.decode())
        self._h = h
        self.device = device
        self._lib.gawee_set_graph_mode(h, 1 if graph_mode else 0)
        if precision is not None:
            self.set_precision(precision)
        self.arg_specs = [self._info(self._lib.gawee_arg_info, i) for i in range(self._lib.gawee_num_args(h))]
        self.output_specs = [self._info(self._lib.gawee_output_info, i)
                             for i in range(self._lib.gawee_num_outputs(h))]

    @classmethod
    def from_file(cls, path: str, **kw) -> "Model":
        with open(path) as f:
            return cls(f.read(), **kw)

    def set_precision(self, precision: str):
        """Tensor-core arithmetic: "fp32" (three TF32 passes, the default and the
        parity mode), "tf32" (one pass) or "bf16" (one bf16 pass on the TMA
        contraction kernel, single-pass TF32 elsewhere); gawee_set_precision in
        include/gawee_cuda.h states each mode's error bound."""
        if precision not in self.PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(self.PRECISIONS)}, not {precision!r}")
        self._check(self._lib.gawee_set_precision(self._h, self.PRECISIONS[precision]))

    @property
    def precision(self) -> str:
        return {v: k for k, v in self.PRECISIONS.items()}[self._lib.gawee_precision(self._h)]

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.gawee_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int):
        if st:
            buf = ctypes.create_string_buffer(4096)
            self._lib.gawee_last_error(self._h, buf, len(buf))
            raise GaweeError(st, buf.value.decode())

    def _info(self, fn, i) -> Tuple[np.dtype, Tuple[int, ...]]:
        dt, rk = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 8)()
        self._check(fn(self._h, i, ctypes.byref(dt), ctypes.byref(rk), shape))
        return np.dtype(NP_OF_DTYPE[dt.value]), tuple(shape[k] for k in range(rk.value))

    # -- staging ---------------------------------------------------------------
    def set_arg(self, i: int, arr: np.ndarray, stream=None):
        dt, shape = self.arg_specs[i]
        a = np.ascontiguousarray(arr)
        if a.dtype != dt or tuple(a.shape) != shape:
            raise GaweeError(1, f"argument {i} expects {dt}{shape}, got {a.dtype}{a.shape}")
        self._check(self._lib.gawee_set_arg(self._h, i, a.ctypes.data, a.nbytes, _stream_ptr(stream)))
        if stream is None:
            # the copy is asynchronous on the context stream; keep the array alive until it lands
            self.synchronize()

    def set_arg_device(self, i: int, ptr: int, nbytes: int, stream=None):
        self._check(self._lib.gawee_set_arg_device(self._h, i, ptr, nbytes, _stream_ptr(stream)))

    def set_args(self, arrays: Sequence[np.ndarray]):
        if len(arrays) != len(self.arg_specs):
            raise GaweeError(1, f"expected {len(self.arg_specs)} arguments, got {len(arrays)}")
        for i, a in enumerate(arrays):
            self.set_arg(i, a)

    # -- execution -------------------------------------------------------------
    def forward(self, stream=None):
        self._check(self._lib.gawee_forward(self._h, _stream_ptr(stream)))

    def synchronize(self, stream=None):
        self._check(self._lib.gawee_synchronize(self._h, _stream_ptr(stream)))

    def output(self, i: int = 0, stream=None, out: Optional[np.ndarray] = None) -> np.ndarray:
        dt, shape = self.output_specs[i]
        if out is None:
            out = np.empty(shape, dtype=dt)
        self._check(self._lib.gawee_get_output(self._h, i, out.ctypes.data, out.nbytes, _stream_ptr(stream)))
        if stream is None:
            self.synchronize()
        return out

    def output_ptr(self, i: int = 0) -> int:
        p = ctypes.c_void_p()
        self._check(self._lib.gawee_output_device_ptr(self._h, i, ctypes.byref(p)))
        return p.value

    def run(self, arrays: Sequence[np.ndarray]) -> List[np.ndarray]:
        """Stage all arguments, run one forward, return every output (synchronous)."""
        self.set_args(arrays)
        self.forward()
        self.synchronize()
        return [self.output(i) for i in range(len(self.output_specs))]

    def num_launches(self) -> int:
        """Kernel launches of one forward (split contractions add a reduce kernel)."""
        return self._lib.gawee_num_launches(self._h)

    def num_kernels(self) -> int:
        return self._lib.gawee_num_kernels(self._h)

    def kernels(self):
        """[(name, is_tensor_core, algorithmic_flops)] for each kernel of one forward."""
        out = []
        for i in range(self.num_kernels()):
            name = ctypes.create_string_buffer(512)
            tc, fl = ctypes.c_int(), ctypes.c_double()
            self._check(self._lib.gawee_op_info(self._h, i, name, len(name), ctypes.byref(tc), ctypes.byref(fl)))
            out.append((name.value.decode(), bool(tc.value), fl.value))
        return out

    def profile(self, stream=None):
        """Device milliseconds of each kernel of one eager forward."""
        n = self.num_kernels()
        ms = (ctypes.c_float * n)()
        self._check(self._lib.gawee_profile_forward(self._h, _stream_ptr(stream), ms, n))
        return list(ms)

    def plan_summary(self) -> str:
        buf = ctypes.create_string_buffer(1 << 20)
        self._check(self._lib.gawee_plan_summary(self._h, buf, len(buf)))
        return buf.value.decode()

    # -- data parallel -----------------------------------------------------------
    @staticmethod
    def dp_unique_id() -> bytes:
        lib = load_library()
        buf = ctypes.create_string_buffer(128)
        st = lib.gawee_dp_unique_id(buf)
        if st:
            raise GaweeError(st, "ncclGetUniqueId failed")
        return buf.raw

    def dp_init(self, world: int, rank: int, uid: bytes):
        buf = ctypes.create_string_buffer(uid, 128)
        self._check(self._lib.gawee_dp_init(self._h, world, rank, buf))

    def dp_output_bytes(self, i: int = 0) -> int:
        """Bytes of output i over every rank (rank 0's gather destination size)."""
        n = ctypes.c_size_t()
        self._check(self._lib.gawee_dp_output_bytes(self._h, i, ctypes.byref(n)))
        return n.value

    def dp_gather_output(self, i: int, dst_ptr: Optional[int], stream=None):
        self._check(self._lib.gawee_dp_gather_output(self._h, i, dst_ptr, _stream_ptr(stream)))


def run_dir(mlir_path: str, inputs_dir: str, outputs_dir: str, device: int = 0, entry: str = "forward"):
    """The reference runner's contract: argN.npy in, outputN.npy out."""
    m = Model.from_file(mlir_path, device=device, entry=entry)
    args = [np.load(os.path.join(inputs_dir, f"arg{i}.npy")) for i in range(len(m.arg_specs))]
    outs = m.run(args)
    os.makedirs(outputs_dir, exist_ok=True)
    for i, o in enumerate(outs):
        np.save(os.path.join(outputs_dir, f"output{i}.npy"), o)
    return outs
