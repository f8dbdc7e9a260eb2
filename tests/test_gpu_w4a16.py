"""NVFP4 linear in the reference's W4A16 arithmetic on SM-pair tensor-core tiles
(ada_nvfp4_linear_w4a16, tcgen05.mma.cta_group::2.kind::f16) vs dequantise-then-matmul.

The weights are widened to fp16 exactly (e2m1 value x e4m3 block scale), the activations are
cast to fp16 as the reference's kernel casts them (adallm/ops/nvfp4_gemm.py:100-105), and the products
accumulate in fp32, so against an fp64 matmul of the same fp16 operands the only error is fp32
summation order and the output rounding: rel-L2 <= 2e-3 for bf16 outputs, <= 5e-4 for fp16."""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as nv
from adallm_b200.nvfp4_gemm import nvfp4_linear_w4a16, prepack_scales
from tests.gpu_util import dev, rel_l2
from tests.test_gpu_nvfp4 import random_weight

pytestmark = pytest.mark.gpu


def ref_w4a16(x, packed, scale16, s2, bias):
    """fp64 x.half() @ (lut x block scale)^T x scale_2 (+ bias): oracle.nvfp4.linear_w4a16_ref."""
    return nv.linear_w4a16_ref(x, packed, scale16.astype(np.float32), s2, bias)


@pytest.mark.parametrize("m,n,k,with_bias,dtype", [
    (2048, 6144, 4096, False, torch.bfloat16),
    (300, 512, 256, True, torch.float16),      # ragged last tile (rows 300..511 never stored)
    (17, 256, 64, False, torch.bfloat16),      # one K stage, one tile
    (1100, 4096, 1024, True, torch.bfloat16),
])
def test_w4a16_matches_dequant_matmul(m, n, k, with_bias, dtype):
    d = dev()
    packed, sbits, scale16, s2 = random_weight(n, k, seed=31, realistic=False)
    g = torch.Generator().manual_seed(31)
    x = torch.randn((m, k), generator=g).to(dtype)
    bias = (torch.randn((n,), generator=g) * 0.1).to(dtype) if with_bias else None
    y = nvfp4_linear_w4a16(x.to(d), torch.from_numpy(packed).to(d), torch.from_numpy(scale16).to(d),
                           torch.tensor(s2, device=d), None if bias is None else bias.to(d))
    torch.cuda.synchronize()
    assert y.dtype == dtype and y.shape == (m, n)
    ref = ref_w4a16(x, packed, scale16, s2, bias)
    tol = 2e-3 if dtype == torch.bfloat16 else 5e-4
    err = rel_l2(y.double().cpu(), ref)
    assert err < tol, f"rel-L2 {err:.2e}"
    # against the reference's own formula (fp32 dequantised weights incl. scale_2): same bar
    w = nv.dequant_nvfp4_torch(packed, scale16.astype(np.float32), s2)
    ref2 = x.half().float() @ w.t() + (bias.float() if bias is not None else 0.0)
    assert rel_l2(y.float().cpu(), ref2) < tol


def test_w4a16_in_cuda_graph_and_strided_io():
    """Replays from a CUDA graph with the eager result; a strided input view (ldx > K) and an
    output slice of a wider buffer (ldy > N) give the same values as contiguous ones."""
    d = dev()
    m, n, k = 1024, 2048, 1024
    packed, sbits, scale16, s2 = random_weight(n, k, seed=32, realistic=False)
    pk, sc, s2t = torch.from_numpy(packed).to(d), torch.from_numpy(scale16).to(d), torch.tensor(s2, device=d)
    sf = prepack_scales(sc, n, k)
    xw = torch.randn((m, k + 64), generator=torch.Generator().manual_seed(32)).to(torch.bfloat16).to(d)
    x = xw[:, :k]
    y_eager = nvfp4_linear_w4a16(x.contiguous(), pk, sc, s2t, sf=sf)
    wide = torch.zeros((m, n + 256), dtype=torch.bfloat16, device=d)
    y_strided = nvfp4_linear_w4a16(x, pk, sc, s2t, sf=sf, out=wide[:, :n])
    torch.cuda.synchronize()
    assert torch.equal(y_strided, y_eager)
    assert torch.count_nonzero(wide[:, n:]) == 0
    y_graph = torch.empty_like(y_eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            nvfp4_linear_w4a16(x, pk, sc, s2t, sf=sf, out=y_graph)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_graph, y_eager)
    del graph


def test_w4a16_rejects_unsupported_shapes():
    d = dev()
    packed, sbits, scale16, s2 = random_weight(128, 256, seed=33, realistic=False)
    x = torch.randn((64, 256), dtype=torch.bfloat16, device=d)
    with pytest.raises(Exception):  # N % 256 != 0
        nvfp4_linear_w4a16(x, torch.from_numpy(packed).to(d), torch.from_numpy(scale16).to(d),
                           torch.tensor(s2, device=d))


def test_w4a16_full_code_and_scale_range():
    """Every e2m1 code pair and block scales over the whole finite e4m3 range (subnormal 2^-9 to
    448): code value x block scale is exact in fp16 across it (2^-10 .. 2688), so the bar is the
    same as for moderate scales."""
    d = dev()
    m, n, k = 256, 256, 512
    g = torch.Generator().manual_seed(34)
    packed = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8).numpy()
    packed[0, :] = np.arange(256, dtype=np.uint8)  # row 0 holds every byte once
    sbits = torch.randint(0x01, 0x7F, (n, k // 16), generator=g, dtype=torch.int32).to(torch.uint8).numpy()
    scale16 = nv.e4m3_decode(sbits).astype(np.float16)
    s2 = np.float32(0.01)
    x = torch.randn((m, k), generator=g).to(torch.float16)
    y = nvfp4_linear_w4a16(x.to(d), torch.from_numpy(packed).to(d), torch.from_numpy(scale16).to(d),
                           torch.tensor(s2, device=d))
    torch.cuda.synchronize()
    ref = ref_w4a16(x, packed, scale16, s2, None)
    assert rel_l2(y.double().cpu(), ref) < 5e-4
    assert rel_l2(y[:, 0].double().cpu(), ref[:, 0]) < 5e-4


def test_nvfp4_linear_routes_prefill_size_to_w4a16(monkeypatch):
    """nvfp4_linear with the default terms runs the W4A16 kernel from W4A16_MIN_M (256) tokens
    (identical to nvfp4_linear_w4a16) and the multi-term operand below it (identical to terms=4);
    an explicit terms or W4A16_MIN_M = 0 keeps the multi-term operand at any size."""
    from adallm_b200 import nvfp4_gemm
    from adallm_b200.nvfp4_gemm import nvfp4_linear
    d = dev()
    n, k = 1024, 1024
    packed, sbits, scale16, s2 = random_weight(n, k, seed=35, realistic=False)
    args = (torch.from_numpy(packed).to(d), torch.from_numpy(scale16).to(d), torch.tensor(s2, device=d))
    g = torch.Generator().manual_seed(35)
    x_big = torch.randn((3, 200, k), generator=g).to(torch.bfloat16).to(d)   # 600 tokens, leading dims
    x_small = torch.randn((100, k), generator=g).to(torch.bfloat16).to(d)
    y = nvfp4_linear(x_big, *args, None, None, 16)
    assert y.shape == (3, 200, n)
    assert torch.equal(y, nvfp4_linear_w4a16(x_big, *args))
    assert not torch.equal(y, nvfp4_linear(x_big, *args, None, None, 16, terms=4))
    assert torch.equal(nvfp4_linear(x_small, *args, None, None, 16), nvfp4_linear(x_small, *args, None, None, 16, terms=4))
    monkeypatch.setattr(nvfp4_gemm, "W4A16_MIN_M", 0)
    assert torch.equal(nvfp4_linear(x_big, *args, None, None, 16), nvfp4_linear(x_big, *args, None, None, 16, terms=4))
