"""ada_argmax_noalloc (library-internal scratch, no caller workspace) vs ada_argmax (caller
workspace) through the C ABI: identical indices on two consecutive calls, bf16 and fp16,
including ties (first maximum) and a row longer than one chunk; oversized requests are
rejected before any launch.  Collected last (file name) so it also runs after other tests."""
import pytest
import torch

from adallm_b200 import _native as N
from tests.gpu_util import dev

pytestmark = pytest.mark.gpu


def _with_workspace(logits):
    d = logits.device
    rows, cols = logits.shape
    out = torch.empty(rows, dtype=torch.int64, device=d)
    ws = torch.empty(int(N.lib().ada_argmax_workspace_size(rows, cols)), dtype=torch.uint8, device=d)
    N.check(N.lib().ada_argmax(logits.data_ptr(), logits.stride(0), rows, cols, N.DT[logits.dtype], out.data_ptr(),
                               ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream), "argmax")
    return out


def _no_alloc(logits):
    rows, cols = logits.shape
    out = torch.full((rows,), -7, dtype=torch.int64, device=logits.device)
    N.check(N.lib().ada_argmax_noalloc(logits.data_ptr(), logits.stride(0), rows, cols, N.DT[logits.dtype],
                                       out.data_ptr(), torch.cuda.current_stream().cuda_stream), "argmax_noalloc")
    return out


@pytest.mark.parametrize("dtype,rows,cols", [(torch.bfloat16, 16, 151936), (torch.float16, 37, 4099),
                                             (torch.bfloat16, 291, 151936)])
def test_noalloc_matches_workspace_entry(dtype, rows, cols):
    d = dev()
    g = torch.Generator(device="cpu").manual_seed(rows + cols)
    logits = torch.randn((rows, cols), generator=g).to(dtype).to(d)
    logits[0, 5] = 30.0
    logits[0, cols - 3] = 30.0          # tie: the first maximum wins
    logits[1, cols - 1] = 40.0          # maximum in the last chunk
    ref = _with_workspace(logits)
    first = _no_alloc(logits)
    second = _no_alloc(logits)
    torch.cuda.synchronize()
    assert torch.equal(first, ref) and torch.equal(second, ref)
    assert torch.equal(ref.cpu(), logits.float().argmax(dim=1).cpu())
    assert first[0].item() == 5 and first[1].item() == cols - 1


def test_noalloc_setup_call_then_two_calls():
    """rows == 0 performs only the per-device scratch look-up (the call a recording runtime makes
    first); the calls after it still match the workspace entry."""
    d = dev()
    st = N.lib().ada_argmax_noalloc(None, 8, 0, 8, 0, None, torch.cuda.current_stream().cuda_stream)
    assert st == N.ADA_OK
    logits = torch.randn((4, 1000), device=d, dtype=torch.bfloat16)
    ref = _with_workspace(logits)
    assert torch.equal(_no_alloc(logits), ref) and torch.equal(_no_alloc(logits), ref)


def test_noalloc_rejects_rows_beyond_scratch():
    d = dev()
    logits = torch.zeros((292, 151936), dtype=torch.bfloat16, device=d)
    out = torch.empty(292, dtype=torch.int64, device=d)
    st = N.lib().ada_argmax_noalloc(logits.data_ptr(), 151936, 292, 151936, 0, out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    assert st == N.ADA_ERR_WORKSPACE
