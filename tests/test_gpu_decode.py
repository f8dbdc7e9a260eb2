"""Whole decode step on the B200 (all hot-path kernels, CUDA graph) vs the CPU oracle
decoder (teacher-forced greedy decode).  Decisive-token agreement >= 99%; raw agreement
>= 90% (near-tied logits of a random-init model flip under last-bit differences, see
tests/decode_check.py); logits within 5e-2 rel-L2."""
import pytest

from tests.decode_check import run_agreement

pytestmark = pytest.mark.gpu


def test_decode_step_agreement_graph():
    raw, decisive, errs = run_agreement(layers=4, steps=64, batch=4, prompt=8, graph=True, return_logits=True)
    assert decisive >= 0.99, (raw, decisive)
    assert raw >= 0.90, (raw, decisive)
    assert max(errs) < 5e-2, errs


def test_decode_step_agreement_eager_batch16():
    raw, decisive = run_agreement(layers=2, steps=8, batch=16, prompt=4, graph=False)
    assert decisive >= 0.99 and raw >= 0.90, (raw, decisive)
