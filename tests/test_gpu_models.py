"""Whole-graph parity of the CUDA backend against the oracle on the benchmark
architectures, at the tolerances the reference uses for its own parity check
(back/eval_priority_models.py:67-70: atol 1e-4 for ResNet, 5e-4 for the NLP
models; rtol 1e-4)."""
import numpy as np
import pytest

from gawee_b200 import synth
from tests.helpers import compare, parity_line

pytestmark = pytest.mark.gpu


def _check(graph, runs=2):
    import oracle
    from gawee_b200.runtime import Model

    args = graph.make_args()
    want = oracle.run(graph.mlir, args)
    m = Model(graph.mlir)
    try:
        for _ in range(runs):  # second run replays the captured CUDA graph
            got = m.run(args)
            for k, (a, b) in enumerate(zip(got, want)):
                compare(a, b, graph.atol, 1e-4, f"{graph.name} output{k}")
        for k, (a, b) in enumerate(zip(got, want)):
            parity_line(f"{graph.name} output{k}", a, b, graph.atol, 1e-4)
    finally:
        m.close()


def test_resnet18_b1():
    _check(synth.resnet18(1))


def test_resnet18_b2_small_image():
    _check(synth.resnet18(2, image=96))


def test_resnet18_full_batch_rows_match_oracle():
    """The bench workload at its full size: ResNet-18, batch 256 of 3x224x224.
    Batch rows are independent, so rows of the full-batch GPU forward (two
    runs: eager, then the replayed CUDA graph) must match the oracle's
    forward of those single images with the same weights; the first, a
    middle and the last row are checked at the reference ResNet tolerance."""
    import os

    import oracle
    from gawee_b200.runtime import Model

    big = synth.resnet18(256)
    args = big.make_args()
    m = Model(big.mlir)
    try:
        got = [m.run(args)[0] for _ in range(2)]
    finally:
        m.close()
    one = synth.resnet18(1)  # same weights: they do not depend on the batch size
    o = oracle.Oracle(one.mlir)
    for r in (0, 129, 255):
        a1 = [np.ascontiguousarray(args[0][r:r + 1])] + list(args[1:])
        want = o.run(a1, threads=os.cpu_count() or 1)[0]
        for k, g in enumerate(got):
            compare(g[r:r + 1], want, big.atol, 1e-4, f"resnet18 b256 row {r} run {k}")
        parity_line(f"resnet18 b256 row {r}", got[-1][r:r + 1], want, big.atol, 1e-4)


def test_bert_tiny_s128():
    _check(synth.bert_tiny())


def test_llama15m_s256():
    _check(synth.llama15m())


def test_gqa_decoder_reduced():
    # the 135M GQA architecture (hidden 576, 9 q / 3 kv heads of 64, SwiGLU 1536)
    # with 2 layers, batch 2 and sequence 64 so the oracle finishes in seconds
    _check(synth.llama(2, 64, dim=576, layers=2, heads=9, kv_heads=3, ffn=1536, vocab=4096, name="decoder135m_l2"))


@pytest.mark.parametrize("decode", [False, True])
def test_merged_qkv_projection_matches_oracle_merged_and_not(decode, monkeypatch):
    """The Q, K and V projections of each layer as one GEMM over the
    concatenated weights (6 query and 2 key/value heads of 16: N = 96 + 32 +
    32 = 160, a ragged second tile; K and V read as column slices by RoPE,
    the KV-cache concat and attention): the oracle's values with the merge
    and without it (GAWEE_MERGE_GEMMS=0)."""
    kw = dict(dim=96, layers=2, heads=6, kv_heads=2, ffn=128, vocab=300)
    g = synth.llama_decode(2, 37, name="gqa_small_decode", **kw) if decode else \
        synth.llama(2, 40, name="gqa_small", **kw)
    from gawee_b200.runtime import plan_text
    assert plan_text(g.mlir).count("matmul3") == 2
    _check(g)
    monkeypatch.setenv("GAWEE_MERGE_GEMMS", "0")
    assert "matmul3" not in plan_text(g.mlir)
    _check(g)


@pytest.mark.parametrize("past", [1, 255])
def test_llama15m_decode_step(past):
    """A KV-cache decode step with the reference tinyllama binding's inputs
    (input_ids [1, 1], attention_mask, position_ids, past key/value per layer;
    eval_priority_models.py:38-54): logits and every layer's present key and
    value against the oracle.  past = 1 is the binding's static shape; at 255
    the first position is masked out."""
    _check(synth.llama15m_decode(1, past))


def test_gqa_decoder_decode_step():
    """Decode with grouped KV heads (9 query heads over 3 key/value heads) and
    batch 2: the concatenated cache is read through the head mapping."""
    _check(synth.llama_decode(2, 63, dim=576, layers=2, heads=9, kv_heads=3, ffn=1536, vocab=4096,
                              name="decoder135m_l2_decode"))


def test_decoder135m_full_size_sampled_sequences_match_oracle():
    """Configuration 4 at its full size: the 135M GQA decoder (30 layers,
    hidden 576, 9 / 3 heads) prefilling batch 64 x 512 tokens.  Sequences
    are independent, so the logits of the first and the last sequence of the
    full-batch GPU forward must match the oracle's forward of those single
    sequences, at the reference's transformer tolerance (5e-4 absolute,
    1e-4 relative).  Only those rows are copied back (the full logits are
    6.4 GB)."""
    import os

    import torch

    import oracle
    from gawee_b200.runtime import Model

    big = synth.smollm135m(64, 512)
    args = big.make_args()
    rows = (0, 63)
    m = Model(big.mlir)
    try:
        m.set_args(args)
        got = []
        for _ in range(2):  # eager, then the replayed CUDA graph
            m.forward()
            m.synchronize()
            base = m.output_ptr(0)
            row_elems = 512 * 49152
            per = []
            from cuda.bindings import runtime as cudart
            for r in rows:
                t = torch.empty(row_elems, dtype=torch.float32, device="cuda")
                err, = cudart.cudaMemcpy(t.data_ptr(), base + r * row_elems * 4, row_elems * 4,
                                         cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
                assert err == cudart.cudaError_t.cudaSuccess
                per.append(t.cpu().numpy().reshape(1, 512, 49152))
            got.append(per)
    finally:
        m.close()
    one = synth.smollm135m(1, 512)  # same weights: they do not depend on the batch size
    o = oracle.Oracle(one.mlir)
    for i, r in enumerate(rows):
        a1 = [np.ascontiguousarray(args[0][r:r + 1])] + list(args[1:])
        want = o.run(a1, threads=os.cpu_count() or 1)[0]
        for k in range(2):
            compare(got[k][i], want, 5e-4, 1e-4, f"decoder135m b64 sequence {r} run {k}")
        parity_line(f"decoder135m b64x512 sequence {r}", got[-1][i], want, 5e-4, 1e-4)
