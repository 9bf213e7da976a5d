"""The allocation-free matrix product, gawee_matmul_f32_noalloc.

It exists for callers that cannot allocate device memory at the moment they
need a product — code inside CUDA stream capture (cudaMalloc cannot be
captured), callers living within a fixed memory budget or their own pool, or
error-recovery paths where an allocation could fail.  They pass their own A,
B and C; the library keeps the packed B planes in its static device scratch.

The test drives the entry point through the C ABI on device buffers the test
owns, twice in a row with different operands (the second call reuses the
scratch the first one left behind), and compares each result with the
regular entry points (gawee_create / gawee_set_arg / gawee_forward /
gawee_get_output) on a graph holding the same gawee.matmul.
"""
import ctypes

import numpy as np
import pytest

from tests.helpers import build, compare

pytestmark = pytest.mark.gpu


def _matmul_graph(m, k, n):
    def g_(g):
        a = g.input("f32", (m, k), lambda: np.zeros((m, k), np.float32))
        b = g.input("f32", (k, n), lambda: np.zeros((k, n), np.float32))
        return [g.matmul(a, b)]
    return build(g_)[0]


def test_noalloc_matmul_matches_planned_graph_twice():
    import torch

    from gawee_b200 import runtime

    lib = runtime.load_library()
    m, k, n = 333, 260, 200
    mlir = _matmul_graph(m, k, n)
    model = runtime.Model(mlir)
    try:
        for seed in (1, 2):
            rng = np.random.default_rng(seed)
            a = rng.standard_normal((m, k), dtype=np.float32)
            b = rng.standard_normal((k, n), dtype=np.float32)
            want = model.run([a, b])[0]

            da = torch.from_numpy(a).cuda()
            db = torch.from_numpy(b).cuda()
            dc = torch.full((m, n), float("nan"), device="cuda")
            stream = torch.cuda.current_stream().cuda_stream
            st = lib.gawee_matmul_f32_noalloc(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, stream)
            assert st == 0, f"status {st}"
            torch.cuda.synchronize()
            got = dc.cpu().numpy()
            compare(got, want, atol=2e-4, rtol=1e-4, what=f"noalloc call {seed}")
    finally:
        model.close()


def test_noalloc_matmul_rejects_oversized_and_unaligned():
    import torch

    from gawee_b200 import runtime

    lib = runtime.load_library()
    a = torch.zeros((4, 4096), device="cuda")
    b = torch.zeros((4096, 1024), device="cuda")          # n*k = 4 Mi > 2 Mi scratch elements
    c = torch.zeros((4, 1024), device="cuda")
    st = lib.gawee_matmul_f32_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), 4, 1024, 4096, None)
    assert st == 1
    buf = ctypes.create_string_buffer(512)
    lib.gawee_last_error(None, buf, len(buf))
    assert b"exceeds" in buf.value
    st = lib.gawee_matmul_f32_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), 4, 8, 6, None)  # k % 4 != 0
    assert st == 1
