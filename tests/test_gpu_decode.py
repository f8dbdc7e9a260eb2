"""Whole decode step on the B200 (all hot-path kernels, CUDA graph) vs the CPU oracle
decoder: greedy-token agreement >= 99% (teacher-forced) and logits within 1e-2 rel-L2."""
import pytest

from tests.decode_check import run_agreement

pytestmark = pytest.mark.gpu


def test_decode_step_agreement_graph():
    frac, errs = run_agreement(layers=4, steps=24, batch=4, prompt=8, graph=True, return_logits=True)
    assert frac >= 0.99, frac
    assert max(errs) < 1e-2, errs


def test_decode_step_agreement_eager_batch16():
    frac = run_agreement(layers=2, steps=8, batch=16, prompt=4, graph=False)
    assert frac >= 0.99, frac
