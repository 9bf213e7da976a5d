"""The allocation-free matrix product, gawee_matmul_f32_noalloc.

It exists for callers that cannot allocate device memory at the moment they
need a product: a host framework whose caching allocator owns the device
memory (an allocation behind its back can fail or fragment the pool it
manages), a caller working within a fixed memory budget, or an
error-recovery path after an allocation has already failed.  They pass
their own A, B and C; the library keeps the packed B planes in its static
device scratch and reports kernel errors through a static status word.

The test drives the entry point through the C ABI on device buffers the test
owns, two calls in a row with different operands per shape (the second call
reuses the scratch the first one left behind), and compares each result with
the oracle's sequential fp32 product and with the regular entry points
(gawee_create / gawee_set_arg / gawee_forward / gawee_get_output) on a graph
holding the same gawee.matmul.  Shapes cover both tile widths (n <= 64 takes
the 64-wide tile), n not a multiple of 4, a single row, and the largest
n * k the scratch holds.  This file is collected last on purpose.
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


# (m, k, n): the first-round shape; 1 row with the 64-wide tile; 64-wide tile;
# n not a multiple of 4 on the 128-wide tile; the scratch limit n * k = 2 Mi.
SHAPES = [(333, 260, 200), (1, 4, 3), (5, 8, 64), (130, 36, 65), (3, 2048, 1024)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_noalloc_matmul_matches_oracle_and_planned_graph_twice(m, k, n):
    import torch

    import oracle
    from gawee_b200 import runtime

    lib = runtime.load_library()
    mlir = _matmul_graph(m, k, n)
    model = runtime.Model(mlir)
    atol = 1e-4 * max(1.0, np.sqrt(k) / 8)  # the tolerance of the GEMM parity tests
    try:
        for seed in (1, 2):
            rng = np.random.default_rng(seed)
            a = rng.standard_normal((m, k), dtype=np.float32)
            b = rng.standard_normal((k, n), dtype=np.float32)
            want = oracle.run(mlir, [a, b])[0]
            planned = model.run([a, b])[0]

            da = torch.from_numpy(a).cuda()
            db = torch.from_numpy(b).cuda()
            dc = torch.full((m, n), float("nan"), device="cuda")
            stream = torch.cuda.current_stream().cuda_stream
            st = lib.gawee_matmul_f32_noalloc(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, stream)
            assert st == 0, f"status {st}"
            assert lib.gawee_synchronize(None, stream) == 0, "the kernel reported an error"
            got = dc.cpu().numpy()
            compare(got, want, atol=atol, rtol=1e-4, what=f"noalloc call {seed} vs oracle")
            compare(got, planned, atol=atol, rtol=1e-4, what=f"noalloc call {seed} vs gawee_forward")
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
    st = lib.gawee_matmul_f32_noalloc(a.data_ptr() + 4, b.data_ptr(), c.data_ptr(), 3, 8, 8, None)  # A misaligned
    assert st == 1
    assert lib.gawee_synchronize(None, None) == 0
