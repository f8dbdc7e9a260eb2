"""Tensor parallelism over peer memory, with the ranks emulated on one GPU.

The row-parallel GEMM of each emulated rank writes its split-K partials, tagged with the step,
into every rank's inbox (ada_nvfp4_gemm_partials_peer); each rank's RMSNorm+quant polls the
words until they carry this step's tag and sums all ranks' planes (ada_rmsnorm_quant_peer).
The ranks run one after another on one stream, producers first, so every word is already
current when the consumer starts (nothing here has kernels waiting on one another).
Checks: the inbox holds exactly each rank's local partial planes with this step's tag, every
rank computes the same operand, bit-identical to the partial-plane RMSNorm over the same
values, a second step (epoch 1) is told from the first by its tags, and words whose tag never
arrives end the wait with the error code instead of hanging."""
import ctypes as C

import pytest
import torch

from adallm_b200 import _native as N
from tests.gpu_util import dev
from tests.test_gpu_fused import _rand_weight, act_quant, qbufs

pytestmark = pytest.mark.gpu

M, H, K_FULL, TERMS, W = 16, 4096, 4096, 4, 2
TAG_MUL, TAG_ADD = 4, 3


def _peer_gemm(rank, xq, sfx, gx, w, k, ks, inboxes, epoch, ws, terms=TERMS):
    st = N.lib().ada_nvfp4_gemm_partials_peer(
        xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), M, terms, 16, w[0].data_ptr(), w[0].stride(0),
        w[1].data_ptr(), w[2].data_ptr(), H, k, H, M * H, ks, W, rank,
        C.cast(N.ptr_array([b.data_ptr() for b in inboxes]), C.c_void_p), epoch.data_ptr(), TAG_MUL, TAG_ADD,
        ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    N.check(st, "peer gemm")


def _consume(inbox, ks, epoch, res, wn, err, terms=TERMS):
    q = qbufs(M, H, terms, 16, dev())
    st = N.lib().ada_rmsnorm_quant_peer(
        inbox.data_ptr(), W * ks, M * H, H, res.data_ptr(), H, res.data_ptr(), H, wn.data_ptr(), None, 0, M, H, 1e-6,
        0, 0, terms, 16, q[0].data_ptr(), q[1].data_ptr(), q[2].data_ptr(), epoch.data_ptr(), TAG_MUL, TAG_ADD,
        err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    N.check(st, "rms peer")
    return q


@pytest.mark.parametrize("terms", [TERMS, 1])
def test_peer_partials_and_consumer_emulated_ranks(terms):
    """terms 1 (W4A4) also writes the operand's block scale factors, which must match too."""
    d = dev()
    k = K_FULL // W
    ks = int(N.lib().ada_nvfp4_gemm_splits(M, H, k, terms))
    g = torch.Generator(device="cpu").manual_seed(3)
    xs = [torch.randn((M, k), generator=g).to(torch.bfloat16).to(d) for _ in range(W)]
    ops = [act_quant(x, terms, 16) for x in xs]
    ws_ = [_rand_weight(H, k, d, 100 + r) for r in range(W)]
    inboxes = [torch.zeros((W * ks, M, H), dtype=torch.int64, device=d) for _ in range(W)]
    epochs = [torch.zeros(1, dtype=torch.int32, device=d) for _ in range(W)]
    errs = [torch.zeros(1, dtype=torch.int32, device=d) for _ in range(W)]
    gws = [torch.zeros(256, dtype=torch.uint8, device=d) for _ in range(W)]
    res0 = torch.randn((M, H), generator=g).to(torch.bfloat16).to(d)
    wn = (torch.randn(H, generator=g) * 0.1 + 1).to(torch.bfloat16).to(d)
    s = torch.cuda.current_stream().cuda_stream

    for step in range(2):  # the second step is told from the first by its tags (epoch 1)
        for r in range(W):
            _peer_gemm(r, *ops[r], ws_[r], k, ks, inboxes, epochs[r], gws[r], terms)
        outs, res = [], []
        for r in range(W):
            rr = res0.clone()
            outs.append(_consume(inboxes[r], ks, epochs[r], rr, wn, errs[r], terms))
            res.append(rr)
        torch.cuda.synchronize()
        # the inboxes hold each rank's local partial planes, in rank-major order, with this step's tag
        tag = step * TAG_MUL + TAG_ADD
        vals = []
        for r in range(W):
            local = torch.full((ks, M, H), float("nan"), dtype=torch.float32, device=d)
            ws = torch.zeros(256, dtype=torch.uint8, device=d)
            xq, sfx, gx = ops[r]
            N.check(N.lib().ada_nvfp4_gemm_partials(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), M, terms, 16,
                                                    ws_[r][0].data_ptr(), ws_[r][0].stride(0), ws_[r][1].data_ptr(),
                                                    ws_[r][2].data_ptr(), H, k, local.data_ptr(), H, M * H, ks,
                                                    ws.data_ptr(), 256, s), "local partials")
            torch.cuda.synchronize()
            vals.append(local)
            for dst in range(W):
                words = inboxes[dst][r * ks:(r + 1) * ks]
                assert torch.equal((words >> 32) & 0xffffffff, torch.full_like(words, tag))
                assert torch.equal((words & 0xffffffff).to(torch.int32).view(torch.float32), local)
        # every rank computes the same rows, exactly as the local partial-plane RMSNorm
        planes = torch.cat(vals, 0).contiguous()
        ref = qbufs(M, H, terms, 16, d)
        rr = res0.clone()
        N.check(N.lib().ada_rmsnorm_quant_parts(planes.data_ptr(), W * ks, M * H, H, rr.data_ptr(), H,
                                                rr.data_ptr(), H, wn.data_ptr(), None, 0, M, H, 1e-6, 0, 0, terms, 16,
                                                ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr(), s),
                "rms parts")
        for r in range(W):
            N.check(N.lib().ada_tp_epoch_advance(epochs[r].data_ptr(), s), "epoch")
        torch.cuda.synchronize()
        for r in range(W):
            assert int(errs[r].item()) == 0
            assert int(epochs[r].item()) == step + 1
            assert torch.equal(res[r], rr)
            assert torch.equal(outs[r][0], ref[0]) and torch.equal(outs[r][2], ref[2])
            assert torch.equal(outs[r][1], ref[1])  # block scale factors (written for terms == 1)


def test_peer_wait_times_out_with_error_code():
    """Words whose tag never arrives: the consumer gives up after its bound (~2 s), records 0x50
    in the error word, and the context stays usable."""
    d = dev()
    inbox = torch.zeros((W, M, H), dtype=torch.int64, device=d)
    epoch = torch.zeros(1, dtype=torch.int32, device=d)
    err = torch.zeros(1, dtype=torch.int32, device=d)
    res = torch.zeros((M, H), dtype=torch.bfloat16, device=d)
    wn = torch.ones(H, dtype=torch.bfloat16, device=d)
    _consume(inbox, 1, epoch, res, wn, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0x50
    assert torch.equal(torch.ones(2, device=d) * 2, torch.ones(2, device=d) + 1)  # still usable
