"""Host-side logic that runs without a GPU: MLIR parsing, planning, the C ABI
surface, the synthetic graphs, the runner file contract and data parallelism."""
import ctypes
import os
import re
import subprocess
import sys

import numpy as np
import pytest

from gawee_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The reference checkout, when one is available (GAWEE_REFERENCE_DIR); its hand-written
# MLIR inputs are read by one parser test, which is skipped otherwise.
REF_DIR = os.environ.get("GAWEE_REFERENCE_DIR", "")
REF_TESTS = os.path.join(REF_DIR, "middle", "mlir", "test") if REF_DIR else ""


# ---- parser -------------------------------------------------------------------------------

def test_parser_attribute_forms_and_payloads(oracle_mod):
    # properties <{...}> and attribute dicts {...}; hex and nested dense payloads; multi-results
    mlir = """
#map = affine_map<(d0, d1) -> (d0, d1)>
#map1 = affine_map<(d0, d1) -> (0, d1)>
module attributes {test.attr = 1 : i64} {
  // comment line
  func.func private @other(%a: tensor<2xf32>) -> tensor<2xf32> { return %a : tensor<2xf32> }
  func.func @forward(%arg0: tensor<2x3xf32>, %arg1: tensor<1x3xf32>) -> (tensor<2x3xf32>, tensor<2x3xf32>, tensor<3xi64>) attributes {gawee.onnx_source = "x.onnx"} {
    %cst = arith.constant dense<"0x010000000000000002000000000000000300000000000000"> : tensor<3xi64>
    %cst_0 = arith.constant dense<[[1.000000e+00, -2.5, 0x7F800000]]> : tensor<1x3xf32>
    %0 = "gawee.add"(%arg0, %arg1) {} : (tensor<2x3xf32>, tensor<1x3xf32>) -> tensor<2x3xf32>
    %1:2 = "gawee.split"(%0) <{axis = 0 : i64, splitSizes = array<i64: 1, 1>}> : (tensor<2x3xf32>) -> (tensor<1x3xf32>, tensor<1x3xf32>)
    %2 = tensor.empty() : tensor<2x3xf32>
    %3 = linalg.generic {indexing_maps = [#map, #map1, #map], iterator_types = [#linalg.iterator_type<parallel>, #linalg.iterator_type<parallel>]} ins(%0, %cst_0 : tensor<2x3xf32>, tensor<1x3xf32>) outs(%2 : tensor<2x3xf32>) {
    ^bb0(%in: f32, %in_1: f32, %out: f32):
      %c2 = arith.constant 2.000000e+00 : f32
      %4 = arith.mulf %in, %c2 fastmath<contract> : f32
      %5 = arith.minimumf %4, %in_1 : f32
      linalg.yield %5 : f32
    } -> tensor<2x3xf32>
    %6 = "gawee.cat"(%1#1, %1#0) {axis = 0 : i64} : (tensor<1x3xf32>, tensor<1x3xf32>) -> tensor<2x3xf32>
    return %3, %6, %cst : tensor<2x3xf32>, tensor<2x3xf32>, tensor<3xi64>
  }
}
"""
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    b = np.array([[1, -1, 0.5]], np.float32)
    o3, o6, c = oracle_mod.run(mlir, [a, b])
    s = a + b
    assert np.array_equal(o3, np.minimum(s * 2, np.array([[1, -2.5, np.inf]], np.float32)))
    assert np.array_equal(o6, np.concatenate([s[1:], s[:1]]))
    assert np.array_equal(c, np.array([1, 2, 3], np.int64))


@pytest.mark.parametrize("text,msg", [
    ("module { func.func @forward(%a: tensor<?x3xf32>) -> tensor<?x3xf32> { return %a : tensor<?x3xf32> } }",
     "dynamic"),
    ("module { func.func @forward(%a: tensor<3xf32>) -> tensor<3xf32> { return %b : tensor<3xf32> } }",
     "undefined"),
    ("module { func.func @main(%a: tensor<3xf32>) -> tensor<3xf32> { return %a : tensor<3xf32> } }",
     "not found"),
])
def test_parser_errors(oracle_mod, text, msg):
    with pytest.raises(oracle_mod.OracleError, match=msg):
        oracle_mod.Oracle(text)


@pytest.mark.skipif(not REF_TESTS or not os.path.isdir(REF_TESTS),
                    reason="GAWEE_REFERENCE_DIR does not name a reference checkout")
def test_parser_reads_reference_test_inputs(oracle_mod):
    # the reference's own hand-written inputs (no RUN lines there); matmul_test has two functions
    text = open(os.path.join(REF_TESTS, "matmul_test.mlir")).read()
    for entry, shapes in [("test_matmul_2d", [(2, 4), (4, 3)]), ("test_matmul_batched", [(1, 2, 3, 4), (1, 2, 4, 5)])]:
        o = oracle_mod.Oracle(text, entry)
        assert [s for _, s in o.arg_specs()] == shapes
    text = open(os.path.join(REF_TESTS, "simple_test.mlir")).read()
    o = oracle_mod.Oracle(text, "test_add")
    a = np.ones((2, 3), np.float32)
    assert np.array_equal(o.run([a, a])[0], a + a)


# ---- planner (no device) -------------------------------------------------------------------

def _plan(mlir):
    from gawee_b200 import runtime
    return runtime.plan_text(mlir)


@pytest.mark.parametrize("name", list(synth.CONFIGS))
def test_plan_all_configs(name):
    g = synth.CONFIGS[name]()
    s = _plan(g.mlir)
    head = s.splitlines()[0]
    kv = dict(x.split("=") for x in head.split())
    assert int(kv["main"]) > 0
    if name.startswith("resnet"):
        # every conv's bias/relu/residual is fused into its epilogue
        assert s.count("conv+add+relu") == 8 and s.count("conv+relu") == 9
        assert "relu\n" not in s.replace("conv+relu", "").replace("conv+add+relu", "")
    else:
        # each layer's scores -> scale + mask -> softmax -> P.V cluster is one fused attention op
        # (no materialised scores, no softmax pass); embeddings gathered
        layers = {"bert_tiny": 2, "llama15m": 6, "decoder135m": 30}[name]
        assert s.count("attention") == layers and "softmax" not in s and "gather" in s
        assert "reshape_copy" not in s  # GQA heads are mapped, not expanded
    if name.startswith("llama") or name.startswith("decoder"):
        assert int(kv["prologue"]) >= 6  # RoPE tables and causal mask computed once


def test_plan_fuses_attention_without_a_mask():
    # matmul(Q, K^T) -> div(c) -> softmax -> matmul(., V): the add(mask) step is optional
    from tests.helpers import build, rand_input

    def g_(g):
        q, k, v = (rand_input(g, (2, 4, 160, 64), i) for i in (1, 2, 3))
        s = g.div(g.matmul(q, g.transpose(k, [0, 1, 3, 2])), g.const(8.0, "f32"))
        return [g.matmul(g.softmax(s, -1), v)]
    s = _plan(build(g_)[0])
    assert s.count("attention") == 1 and "softmax" not in s and "matmul" not in s


def test_plan_flags_interpreter_fallbacks():
    # scalar programs without a specialised form are marked in the plan summary
    assert "[interp" not in _plan(synth.resnet18(1).mlir)
    assert "[interp" not in _plan(synth.llama15m().mlir)
    s = _plan(synth.bert_tiny().mlir)
    # BERT's GEMM epilogues (bias + GELU, bias + residual) have specialised forms; its
    # embedding sum and mask arithmetic stay on the interpreter
    assert "[interp epilogue]" not in s and s.count("[interp]") == 2, s
    from tests.helpers import build, rand_input

    def g_(g):
        y = g.matmul(rand_input(g, (37, 64), 1), rand_input(g, (64, 48), 2))
        return [g.op("tanh", [y], None, "f32", y.shape)]
    assert "matmul+tanh [interp epilogue]" in _plan(build(g_)[0])


def test_plan_matches_gelu_epilogue_exactly():
    # bias + GELU runs as a specialised epilogue only when the program is exactly
    # (t * (erf(t / c) + 1)) * 0.5, in any operand order of the commutative steps
    from tests.helpers import build, rand_input
    F = "f32"

    def gelu(form):
        def g_(g):
            t = g.add(g.matmul(rand_input(g, (37, 64), 1), rand_input(g, (64, 48), 2)), rand_input(g, (48,), 3))
            c = g.const(1.4142135381698608, F)
            if form == "standard":
                y = g.mul(g.mul(t, g.add(g.erf(g.div(t, c)), g.const(1.0, F))), g.const(0.5, F))
            elif form == "swapped":
                y = g.mul(g.const(0.5, F), g.mul(g.add(g.const(1.0, F), g.erf(g.div(t, c))), t))
            elif form == "wrong_constant":
                y = g.mul(g.mul(t, g.add(g.erf(g.div(t, c)), g.const(2.0, F))), g.const(0.5, F))
            else:  # c / t: not GELU
                y = g.mul(g.mul(t, g.add(g.erf(g.div(c, t)), g.const(1.0, F))), g.const(0.5, F))
            return [y]
        return _plan(build(g_)[0])
    for form in ("standard", "swapped"):
        s = gelu(form)
        assert "erf" in s and "[interp" not in s, (form, s)
    for form in ("wrong_constant", "divisor_swapped"):
        assert "[interp epilogue]" in gelu(form), form


def test_plan_decode_step():
    # the KV-cache decode step: concat of past and new key/value, one query row,
    # attention, RoPE and RMSNorm still fused; logits + 12 present tensors out
    g = synth.llama15m_decode(1, 255)
    s = _plan(g.mlir)
    assert s.count("attention") == 6 and "softmax" not in s
    assert s.count("rope") == 12 and s.count("rms_norm") == 13
    assert len(g.out_shapes) == 13 and g.out_shapes[1] == (1, 6, 256, 48)


def test_plan_merges_projections_that_share_their_input(monkeypatch):
    # Q, K and V projections of one input (weights are arguments, results feed
    # reshapes) run as one GEMM; a projection feeding an elementwise op keeps
    # its own GEMM so the op stays fused into its epilogue; GAWEE_MERGE_GEMMS=0
    # keeps every projection separate
    from tests.helpers import build, rand_input

    def g_(g):
        x = rand_input(g, (2, 37, 64), 1)
        q, k, v = (g.matmul(x, rand_input(g, (64, n), 2 + i)) for i, n in enumerate((96, 32, 32)))
        outs = [g.transpose(g.reshape(t, (2, 37, t.shape[-1] // 16, 16)), [0, 2, 1, 3]) for t in (q, k, v)]
        gate = g.matmul(x, rand_input(g, (64, 48), 6))
        up = g.matmul(x, rand_input(g, (64, 48), 7))
        return outs + [g.mul(g.mul(gate, g.sigmoid(gate)), up)]
    mlir = build(g_)[0]
    s = _plan(mlir)
    assert s.count("matmul3") == 1 and "reshape_copy" not in s, s
    assert s.count("matmul+sigmoid+mul+mul") == 1, s  # gate and up stay apart: the product is fused
    assert "matmul3" in _plan(synth.llama15m().mlir) and "matmul3" in _plan(synth.llama15m_decode(1, 1).mlir)
    assert "matmul3" not in _plan(synth.bert_tiny().mlir)  # its projections' bias adds are epilogues
    monkeypatch.setenv("GAWEE_MERGE_GEMMS", "0")
    s = _plan(mlir)
    assert "matmul3" not in s and s.count("matmul\n") >= 4, s


def test_plan_keeps_projections_apart_when_a_merge_would_not_hold():
    # a result returned as is needs its own dense buffer; computed weights are
    # not packed once; different left operands share nothing
    from tests.helpers import build, rand_input

    def returned(g):
        x = rand_input(g, (2, 37, 64), 1)
        q = g.matmul(x, rand_input(g, (64, 32), 2))
        k = g.matmul(x, rand_input(g, (64, 32), 3))
        return [q, g.reshape(k, (2, 37, 2, 16))]

    def computed_weight(g):
        x = rand_input(g, (2, 37, 64), 1)
        w = g.add(rand_input(g, (64, 32), 2), rand_input(g, (64, 32), 4))
        q = g.matmul(x, w)
        k = g.matmul(x, rand_input(g, (64, 32), 3))
        return [g.reshape(t, (2, 37, 2, 16)) for t in (q, k)]

    def two_inputs(g):
        x = rand_input(g, (2, 37, 64), 1)
        y = rand_input(g, (2, 37, 64), 5)
        q = g.matmul(x, rand_input(g, (64, 32), 2))
        k = g.matmul(y, rand_input(g, (64, 32), 3))
        return [g.reshape(t, (2, 37, 2, 16)) for t in (q, k)]
    for f in (returned, computed_weight, two_inputs):
        s = _plan(build(f)[0])
        ops = [ln.strip() for ln in s.splitlines()[1:]]
        assert ops.count("matmul") == 2 and not any(o.startswith("matmul2") for o in ops), (f.__name__, s)


def test_plan_memory_reuse():
    g = synth.resnet18(256)
    s = _plan(g.mlir)
    kv = dict(x.split("=") for x in s.splitlines()[0].split())
    # largest activation: 256x64x112x112 fp32 = 822 MB; liveness keeps the arena to a few of them
    assert int(kv["arena_bytes"]) < 4 * 256 * 64 * 112 * 112 * 4


def test_plan_rejects_unsupported():
    from gawee_b200 import runtime
    bad = """module { func.func @forward(%a: tensor<2x3xf32>) -> tensor<2x3xf32> {
      %0 = "gawee.mystery"(%a) : (tensor<2x3xf32>) -> tensor<2x3xf32>
      return %0 : tensor<2x3xf32> } }"""
    with pytest.raises(runtime.GaweeError, match="unsupported"):
        runtime.plan_text(bad)


# ---- C ABI -----------------------------------------------------------------------------------

def test_library_exports_every_declared_symbol():
    from gawee_b200 import runtime
    lib = runtime.load_library()
    header = open(os.path.join(ROOT, "include", "gawee_cuda.h")).read()
    names = set(re.findall(r"^\s*(?:gawee_status|int|void)\s+(gawee_\w+)\s*\(", header, re.M))
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from gawee_b200 import runtime
    with pytest.raises(runtime.GaweeError):
        runtime.Model(synth.resnet18(1, image=32).mlir)


# ---- synthetic graphs -------------------------------------------------------------------------

def test_synthetic_flops_match_cost_model():
    # per-unit algorithmic FLOPs of the benchmark configurations
    assert synth.resnet18(1).flop == 3_628_146_688
    assert synth.bert_tiny().flop == 117_440_512
    assert synth.llama15m().flop == 8_229_224_448
    d = synth.smollm135m()
    assert abs(d.flop - 9.973e12) / 9.973e12 < 1e-3
    assert d.out_shapes == [(64, 512, 49152)]


def test_emitter_argument_order():
    g = synth.bert_tiny()
    kinds = [a.kind for a in g.args]
    # graph inputs first, then float initializers (ONNXMLIREmitter.cpp:2932-2975)
    assert kinds[:3] == ["input"] * 3 and set(kinds[3:]) == {"weight"}
    assert all(a.dtype == "f32" for a in g.args[3:])


def test_runner_file_contract(tmp_path, oracle_mod):
    """oracle CLI: argN.npy in, outputN.npy out, headers byte-compatible with np.load."""
    g = synth.bert_tiny(seq=16, vocab=64, max_pos=32)
    args = g.make_args()
    (tmp_path / "in").mkdir()
    for i, a in enumerate(args):
        np.save(tmp_path / "in" / f"arg{i}.npy", a)
    mlir = tmp_path / "m.mlir"
    mlir.write_text(g.mlir)
    r = subprocess.run([oracle_mod.CLI_PATH, str(mlir), str(tmp_path / "in"), str(tmp_path / "out")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = np.load(tmp_path / "out" / "output0.npy")
    assert np.array_equal(out, oracle_mod.run(g.mlir, args)[0])
    with open(tmp_path / "out" / "output0.npy", "rb") as f:
        head = f.read(128)
    hl = int.from_bytes(head[8:10], "little")
    assert (10 + hl) % 16 == 0 and b"'descr': '<f4'" in head


# ---- data parallelism (gloo ranks on CPU) ---------------------------------------------------------

def _dp_worker(rank, world, port, result_path):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import oracle
    from gawee_b200 import dp, synth as sy
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        full = sy.resnet18(5, image=32, widths=(8, 8, 16, 16), classes=10)  # 5 over 2 ranks: 3 + 2 rows
        args = full.make_args()
        local_batch = dp.shard_range(5, world, rank)
        shard = sy.resnet18(local_batch[1] - local_batch[0], image=32, widths=(8, 8, 16, 16), classes=10)
        local_args = dp.shard_args(args, [True] + [False] * (len(args) - 1), world, rank)
        out = oracle.run(shard.mlir, local_args)[0]
        uid = dp.share_nccl_id(bytes(range(128)) if rank == 0 else bytes(128), rank)
        assert uid == bytes(range(128))
        gathered = dp.gather_rows_host(out, rank, world)
        if rank == 0:
            want = oracle.run(full.mlir, args)[0]
            np.save(result_path, np.array([float(np.max(np.abs(gathered - want)))]))
    finally:
        dist.destroy_process_group()


def test_dp_sharded_matches_full_batch(tmp_path):
    import multiprocessing as mp
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    res = str(tmp_path / "r.npy")
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, res)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs)
    # batch rows are independent: sharded outputs equal the full-batch output exactly
    assert np.load(res)[0] == 0.0


def test_shard_range():
    from gawee_b200 import dp
    assert [dp.shard_range(256, 8, r) for r in (0, 7)] == [(0, 32), (224, 256)]
    assert [dp.shard_range(5, 2, r) for r in (0, 1)] == [(0, 3), (3, 5)]
    assert dp.gather_offsets([3, 2]) == [0, 3]
    assert dp.gather_offsets([32] * 8) == list(range(0, 256, 32))
    with pytest.raises(ValueError):
        dp.gather_offsets([1, -1])


# ---- AOT boundary without MLIR ---------------------------------------------------------------

PRINTED_MODULE = """#map = affine_map<(d0, d1) -> (d0, d1)>
#map1 = affine_map<(d0, d1) -> (0, d1)>
module attributes {gawee.source = "printed by --gawee-to-cuda's module.print"} {
  func.func @forward(%arg0: tensor<4x8xf32>, %arg1: tensor<8x6xf32>, %arg2: tensor<1x6xf32>) -> tensor<4x6xf32> attributes {gawee.onnx_source = "m.onnx"} {
    %0 = "gawee.matmul"(%arg0, %arg1) : (tensor<4x8xf32>, tensor<8x6xf32>) -> tensor<4x6xf32>
    %1 = tensor.empty() : tensor<4x6xf32>
    %2 = linalg.generic {indexing_maps = [#map, #map1, #map], iterator_types = ["parallel", "parallel"]} ins(%0, %arg2 : tensor<4x6xf32>, tensor<1x6xf32>) outs(%1 : tensor<4x6xf32>) {
    ^bb0(%in: f32, %in_0: f32, %out: f32):
      %3 = arith.addf %in, %in_0 : f32
      linalg.yield %3 : f32
    } -> tensor<4x6xf32>
    %4 = "gawee.relu"(%2) : (tensor<4x6xf32>) -> tensor<4x6xf32>
    return %4 : tensor<4x6xf32>
  }
}
"""


def test_planner_reads_the_form_the_mlir_pass_embeds():
    """--gawee-to-cuda prints the module with default flags: gawee ops in the
    generic form (they declare no assembly), func/linalg/arith in their custom
    forms, #map aliases on top.  The planner must accept exactly that text."""
    summary = _plan(PRINTED_MODULE)
    assert "tc" in summary.lower() or "matmul" in summary.lower(), summary


def test_aot_shim_and_abi_source(tmp_path):
    from gawee_b200 import aot
    g = synth.bert_tiny(seq=16, vocab=64, max_pos=32)
    abi = aot.abi_source(g.mlir)
    assert "tensor<" not in abi and abi.count("memref<") == len(g.args) + 1
    shim = tmp_path / "shim.c"
    shim.write_text(aot.emit_ciface_shim(g.mlir))
    obj = tmp_path / "shim.o"
    r = subprocess.run(["gcc", "-O2", "-Wall", "-c", str(shim), "-o", str(obj)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    syms = subprocess.run(["nm", str(obj)], capture_output=True, text=True).stdout
    assert re.search(r"\bT _mlir_ciface_forward\b", syms)
    assert re.search(r"\bU gawee_embedded_forward\b", syms)
    # the embedded text is the graph itself, byte for byte
    r = subprocess.run(["gcc", "-x", "c", "-E", "-P", str(shim)], capture_output=True, text=True)
    assert r.returncode == 0
    # the reference's own launcher generator accepts the ABI source (when built from its sources)
    gen = os.path.join(ROOT, "oracle", "_ref", "gawee-aot")
    if os.path.exists(gen):
        (tmp_path / "abi.mlir").write_text(abi)
        subprocess.run([gen, "build", "--abi-source", str(tmp_path / "abi.mlir"), "--input", str(tmp_path / "x.ll"),
                        "--output", str(tmp_path / "runner"), "--llvm-bin", str(tmp_path / "none"),
                        "--dump-launcher", str(tmp_path / "launcher.cpp")], capture_output=True, text=True)
        launcher = (tmp_path / "launcher.cpp").read_text()
        proto = launcher.split('extern "C" void _mlir_ciface_forward(')[1].split(");")[0]
        assert proto.count("MemRefDescriptor<") == len(g.args) + 1
        assert "loadNpy<int64_t>" in launcher and "saveReturnedMemRef" in launcher
