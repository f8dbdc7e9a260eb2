"""This package inside the reference runtime on the B200 (tests/dropin_harness.py, in its own
process): install(), then the reference's ModelRunner loads a synthetic NVFP4 checkpoint
(4 layers of the Qwen3-8B widths, vocab 151936), captures its decode CUDA graphs and runs a
fresh prefill, a prefix-cache prefill and 24 teacher-forced decode steps of three sequences
scheduled by its BlockManager (page 256).  Every logits row is compared with the CPU oracle.

Pass criteria: logits within 5e-2 relative L2 of the exact oracle in every phase and no worse
than 1.25x the reference-numerics emulation's deviation on average; greedy agreement with the
exact oracle at least the emulation's less 2.5 standard errors; every NVFP4 weight prepacked at
load (the install()-hooked post-load step); graphs captured for every batch size."""
import json
import math
import os
import subprocess
import sys

import pytest

from tests.dropin_harness import reference_available

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LAYERS = 4


def _run(*args, timeout=1500):
    ok, why = reference_available()
    if not ok:
        pytest.skip(why)
    import torch
    torch.cuda.empty_cache()  # the child sizes its KV pool from the device's free memory
    r = subprocess.run([sys.executable, "-m", "tests.dropin_harness", *args], cwd=ROOT, capture_output=True,
                       text=True, timeout=timeout)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("DROPIN ")]
    assert r.returncode == 0 and lines, (r.returncode, r.stdout[-3000:], r.stderr[-5000:])
    out = json.loads(lines[-1][len("DROPIN "):])
    print(json.dumps(out))
    path = os.environ.get("ADA_AGREEMENT_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"test": "dropin_" + "_".join(args[:1] + [a.strip("-") for a in args if a == "--per-op"]), **out}) + "\n")
    return out


@pytest.mark.parametrize("path", ["fused_layers", "per_op"])
def test_dropin_inside_reference_model_runner(path):
    """Both install() decode paths: the reference's Qwen3DecoderLayer as nine fused kernels
    (the default) and the per-op replacements under the reference's own layer forward."""
    r = _run("check", "--layers", str(LAYERS), "--steps", "24", *(["--per-op"] if path == "per_op" else []))
    assert r["prepacked_weights"] == 4 * LAYERS, r
    assert r["graphs"] == [1, 2, 4, 8], r
    if path == "fused_layers":
        assert r["fused_layer_calls"] >= LAYERS * len(r["graphs"]), r  # every captured decode layer
    else:
        assert r["fused_layer_calls"] == 0, r
    assert r["rel_l2_max"] < 5e-2, r
    assert r["rel_l2_mean"] <= 1.25 * max(r["ref_rel_l2_mean"], 1e-3), r
    p = min(max(r["raw_reference"], 0.5), 1.0)
    margin = 2.5 * math.sqrt(2.0 * max(p * (1 - p), 1.0 / r["tokens"]) / r["tokens"])
    assert r["raw"] >= min(0.99, r["raw_reference"] - margin), r


def test_flash_attn_on_this_gpu_is_recorded():
    """Whether the reference's own prefill without a prefix cache (flash-attn 2) runs here; the
    install() default routes that prefill to this package's kernel where it does not."""
    r = _run("flash-attn", timeout=300)
    assert r["flash_attn"] in ("runs", "fails", "not importable"), r
