"""Whole-graph parity of the CUDA backend against the oracle on the benchmark
architectures, at the tolerances the reference uses for its own parity check
(back/eval_priority_models.py:67-70: atol 1e-4 for ResNet, 5e-4 for the NLP
models; rtol 1e-4)."""
import numpy as np
import pytest

from gawee_b200 import synth
from tests.helpers import compare

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
    finally:
        m.close()


def test_resnet18_b1():
    _check(synth.resnet18(1))


def test_resnet18_b2_small_image():
    _check(synth.resnet18(2, image=96))


def test_bert_tiny_s128():
    _check(synth.bert_tiny())


def test_llama15m_s256():
    _check(synth.llama15m())


def test_gqa_decoder_reduced():
    # the 135M GQA architecture (hidden 576, 9 q / 3 kv heads of 64, SwiGLU 1536)
    # with 2 layers, batch 2 and sequence 64 so the oracle finishes in seconds
    _check(synth.llama(2, 64, dim=576, layers=2, heads=9, kv_heads=3, ffn=1536, vocab=4096, name="decoder135m_l2"))
