"""The tensor-core lm_head with the fused greedy pick (ada_lm_head_argmax) through the C ABI.

* logits: within one bf16 ulp (plus 2^-11 for the fp32 accumulation over k) of x . W^T in fp64
  (the reference's F.linear, adallm/ops/embed_head.py:56-66, accumulates in fp32 and rounds once);
* the pick: exactly torch.argmax over the kernel's own bf16 logits (first maximum), and the
  returned value is that logit; planted ties (duplicated weight rows, in one tile and across
  tiles) go to the lower row; idx_base offsets the index (a vocabulary shard);
* shapes: Qwen3-8B (vocab 151936 = 1187 tiles of 128), Gemma3 (vocab 262208, a partial last
  tile, k 5376), a tensor-parallel shard, 1..64 tokens, two calls in a row on one workspace."""
import pytest
import torch

from adallm_b200 import _native as N
from tests.gpu_util import dev

pytestmark = pytest.mark.gpu


def _call(x, w, idx_base=0, logits=True):
    m, k = x.shape
    v = w.shape[0]
    d = x.device
    lg = torch.full((m, v), float("nan"), dtype=torch.bfloat16, device=d) if logits else None
    idx = torch.full((m,), -1, dtype=torch.int64, device=d)
    val = torch.full((m,), float("nan"), dtype=torch.float32, device=d)
    ws = torch.zeros(int(N.lib().ada_lm_head_workspace_size(m, v)), dtype=torch.uint8, device=d)
    st = N.lib().ada_lm_head_argmax(x.data_ptr(), x.stride(0), m, k, w.data_ptr(), w.stride(0), v, idx_base,
                                    N.ptr(lg), v, idx.data_ptr(), val.data_ptr(), ws.data_ptr(), ws.numel(),
                                    torch.cuda.current_stream().cuda_stream)
    N.check(st, "lm_head")
    return lg, idx, val, ws


@pytest.mark.parametrize("m,v,k", [(16, 151936, 4096), (4, 262208, 5376), (64, 4160, 1024), (1, 1000, 64),
                                   (33, 75968, 4096), (16, 128, 4096)])
def test_lm_head_logits_and_pick(m, v, k):
    d = dev()
    g = torch.Generator(device="cpu").manual_seed(m + v)
    x = torch.randn((m, k), generator=g).to(torch.bfloat16).to(d)
    w = (torch.randn((v, k), generator=g) * 0.02).to(torch.bfloat16).to(d)
    lg, idx, val, ws = _call(x, w)
    torch.cuda.synchronize()
    # fp64 product on the host; the kernel's fp32 accumulation over k terms of mean magnitude
    # ~0.013 adds up to ~1e-4 absolute, the bf16 rounding half an ulp
    ref = (x.double().cpu() @ w.double().cpu().t())
    ulp = torch.clamp(ref.abs(), min=2.0 ** -100).log2().floor().exp2() * 2.0 ** -7
    assert bool(((lg.double().cpu() - ref).abs() <= ulp + 2.0 ** -11).all())
    assert torch.equal(idx, lg.float().argmax(dim=1))
    assert torch.equal(val, lg.float().max(dim=1).values)
    assert int(ws[:4].view(torch.int32).item()) == 0


def test_lm_head_ties_shard_offset_and_repeat():
    d = dev()
    m, v, k = 8, 151936, 4096
    g = torch.Generator(device="cpu").manual_seed(4)
    x = torch.randn((m, k), generator=g).to(torch.bfloat16)
    w = (torch.randn((v, k), generator=g) * 0.02).to(torch.bfloat16)
    # a dominant row for token 0 duplicated later in the same tile and in a later tile; token 1's
    # dominant row duplicated in an earlier position of another tile
    w[300] = x[0] * 0.05
    w[301] = w[300]
    w[90000] = w[300]
    w[70000] = x[1] * 0.05
    w[5] = w[70000]
    x, w = x.to(d), w.to(d)
    for rep in range(2):
        lg, idx, val, _ = _call(x, w, idx_base=1000)
        torch.cuda.synchronize()
        assert int(idx[0]) == 1000 + 300 and int(idx[1]) == 1000 + 5, idx[:2]
        assert torch.equal(idx - 1000, lg.float().argmax(dim=1))
    _, idx2, val2, _ = _call(x, w, logits=False)
    torch.cuda.synchronize()
    assert torch.equal(idx2 + 1000, idx) and torch.equal(val2, val)


def test_lm_head_rejects_unsupported():
    d = dev()
    x = torch.zeros((65, 64), dtype=torch.bfloat16, device=d)
    w = torch.zeros((128, 64), dtype=torch.bfloat16, device=d)
    out = torch.empty(65, dtype=torch.int64, device=d)
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device=d)
    s = torch.cuda.current_stream().cuda_stream
    assert N.lib().ada_lm_head_argmax(x.data_ptr(), 64, 65, 64, w.data_ptr(), 64, 128, 0, None, 0, out.data_ptr(),
                                      None, ws.data_ptr(), ws.numel(), s) == N.ADA_ERR_UNSUPPORTED
    assert N.lib().ada_lm_head_argmax(x.data_ptr(), 64, 4, 48, w.data_ptr(), 64, 128, 0, None, 0, out.data_ptr(),
                                      None, ws.data_ptr(), ws.numel(), s) == N.ADA_ERR_UNSUPPORTED
    assert N.lib().ada_lm_head_argmax(x.data_ptr(), 64, 4, 64, w.data_ptr(), 64, 128, 0, None, 0, out.data_ptr(),
                                      None, ws.data_ptr(), 8, s) == N.ADA_ERR_WORKSPACE
