"""CPU-side checks of the C ABI: the library builds for sm_100a, loads, and
exports every entry point declared in include/adallm_b200.h.  No kernel runs."""
import ctypes
import subprocess

import pytest

from adallm_b200 import _native as N
from adallm_b200 import build as B


@pytest.fixture(scope="module")
def built():
    return B.build()


def test_library_exports_every_declared_symbol(built):
    declared = N.declared_symbols()
    assert len(declared) >= 10
    h = ctypes.CDLL(built)
    for name in declared:
        assert hasattr(h, name), f"{name} declared in include/adallm_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    ada = {s for s in exported if s.startswith("ada_")}
    assert ada == set(declared), f"exported but undeclared: {sorted(ada - set(declared))}"


def test_binding_signatures_cover_header(built):
    assert set(N._SIGS) == set(N.declared_symbols())


def test_status_strings_and_version(built):
    lib = N.lib()
    assert lib.ada_abi_version() >= 1
    assert lib.ada_status_string(0) == b"ok"
    assert b"workspace" in lib.ada_status_string(N.ADA_ERR_WORKSPACE)


def test_argument_errors_are_reported_before_any_launch(built):
    lib = N.lib()
    # head_dim 64 is not implemented -> UNSUPPORTED, without touching the (null) pointers' memory
    st = lib.ada_fp8_paged_decode(16, 0, 0, 0, 16, 16, 0, 0, 0, 4, 16, 4, 4, 16, 1, 8, 2, 64, 16, 1.0, 1.0, 1.0, 0,
                                  16, 0, 16, 1 << 20, None)
    assert st == N.ADA_ERR_UNSUPPORTED
    st = lib.ada_rmsnorm(None, 0, None, 0, None, 0, None, None, 0, 4, 128, 1e-6, 0, 0, None)
    assert st == N.ADA_ERR_INVALID_ARG
    # unknown attention launch flags are rejected
    st = lib.ada_fp8_paged_decode_quant_ex(16, 0, 0, 0, 16, 16, 0, 0, 0, 4, 16, 4, 4, 16, 1, 32, 8, 128, 16, 1.0,
                                           1.0, 1.0, 0, None, 0, 4, 16, 16, None, 16, 16, 1 << 20, 2, None)
    assert st == N.ADA_ERR_INVALID_ARG
    with pytest.raises(ValueError):
        N.check(N.ADA_ERR_ALIGNMENT, "x")
    with pytest.raises(RuntimeError, match="no fallback"):
        N.check(N.ADA_ERR_LAUNCH, "x")


def test_prefill_and_expert_parallel_argument_errors(built):
    """The entries added for the prefill attention and expert parallelism validate their
    arguments before any CUDA call (pointers are placeholders, never dereferenced)."""
    lib = N.lib()
    P = 1 << 20  # 16-byte aligned placeholder address

    def prefill(**kw):
        a = dict(q=P, q_dtype=0, q_st=32 * 128, q_sh=128, k=P, v=P, s_page=16 * 8 * 128, s_tok=8 * 128, s_head=128,
                 num_pages=64, bt=P, bt_stride=8, max_pages=8, cu_q=P, cu_k=P, batch=2, max_q=40, hq=32, hkv=8,
                 d=128, page=16, scale=0.088, k_scale=1.0, v_scale=1.0, window=0, out=P, out_dtype=0,
                 o_st=32 * 128, o_sh=128, err=None, stream=None)
        a.update(kw)
        return lib.ada_fp8_paged_prefill(*a.values())

    assert prefill(d=64) == N.ADA_ERR_UNSUPPORTED            # head_dim 128 only
    assert prefill(page=24) == N.ADA_ERR_UNSUPPORTED          # pages of whole 16-key tiles
    assert prefill(hq=30) == N.ADA_ERR_INVALID_ARG            # GQA groups must divide
    assert prefill(hq=512, hkv=1) == N.ADA_ERR_UNSUPPORTED    # at most 256 rows of a KV head per CTA
    assert prefill(scale=0.0) == N.ADA_ERR_INVALID_ARG        # the row max is taken on unscaled scores
    assert prefill(window=-1) == N.ADA_ERR_INVALID_ARG
    assert prefill(q=P + 8) == N.ADA_ERR_ALIGNMENT
    assert prefill(o_sh=100) == N.ADA_ERR_ALIGNMENT
    assert prefill(batch=0) == 0 and prefill(max_q=0) == 0    # nothing to do
    assert prefill(cu_q=None) == N.ADA_ERR_INVALID_ARG
    # expert parallelism
    st = lib.ada_moe_combine_ep(P, 0, 64, P, None, 0, 4, 2, 2, 64, P, 64, None)
    assert st == N.ADA_ERR_INVALID_ARG                        # expert ids are required
    st = lib.ada_moe_combine_ep(P, 0, 64, P, P, -1, 4, 2, 2, 64, P, 64, None)
    assert st == N.ADA_ERR_INVALID_ARG
    st = lib.ada_nvfp4_linear_grouped_ep(P, 0, 256, 8, 256, P, 128, P, P, 4, -1, 128, P, P, 0, 128, 4, P, 1 << 20,
                                         None)
    assert st == N.ADA_ERR_INVALID_ARG                        # negative expert base


def test_prepack_model_skips_modules_off_the_gpu():
    """prepack_model only touches NVFP4 weights on a GPU; CPU modules and other layouts are
    skipped without any CUDA call."""
    import torch
    from adallm_b200.nvfp4_gemm import prepack_model
    lin = torch.nn.Module()
    lin.weight = torch.nn.Parameter(torch.zeros((128, 256), dtype=torch.uint8), requires_grad=False)
    lin.weight_scale = torch.nn.Parameter(torch.zeros((128, 32), dtype=torch.float16), requires_grad=False)
    model = torch.nn.Sequential(lin, torch.nn.Linear(4, 4))
    assert prepack_model(model) == 0
    assert not hasattr(lin.weight_scale, "_ada_sf")


def test_w4a16_linear_argument_errors(built):
    """ada_nvfp4_linear_w4a16 (the reference's W4A16 arithmetic at prefill size) validates shapes,
    dtypes, workspace size and alignment before any CUDA call (placeholder pointers)."""
    lib = N.lib()
    P = 1 << 20
    m, n, k = 512, 1024, 2048
    ws = int(lib.ada_nvfp4_linear_w4a16_workspace_size(m, k))
    assert ws == 256 + m * k * 2 and lib.ada_nvfp4_linear_w4a16_workspace_size(0, k) == 0

    def call(**kw):
        a = dict(x=P, x_dt=0, ldx=k, m=m, k=k, w=P, ldw=k // 2, sf=P, s2=P, n=n, bias=None, y=P, y_dt=0, ldy=n,
                 ws=P, ws_bytes=ws, stream=None)
        a.update(kw)
        return lib.ada_nvfp4_linear_w4a16(*a.values())

    assert call(m=0) == 0                                     # nothing to do
    assert call(x=None) == N.ADA_ERR_INVALID_ARG
    assert call(m=-1) == N.ADA_ERR_INVALID_ARG
    assert call(x_dt=7) == N.ADA_ERR_INVALID_ARG
    assert call(ldx=k - 8) == N.ADA_ERR_INVALID_ARG
    assert call(n=n - 128, ldy=n) == N.ADA_ERR_UNSUPPORTED    # 256 weight rows per pair tile
    assert call(k=k - 32, ldx=k) == N.ADA_ERR_UNSUPPORTED     # 64-wide K stages
    # a pair may walk every tile: more than 2^31 K steps in all is refused (counters would wrap)
    big = dict(m=1 << 24, k=1 << 16, ldx=1 << 16, ldw=1 << 15, n=1 << 14, ldy=1 << 14, ws_bytes=1 << 62)
    assert call(**big) == N.ADA_ERR_UNSUPPORTED                   # 2^32 K steps
    assert call(**dict(big, m=1 << 22, x=P + 8)) == N.ADA_ERR_ALIGNMENT  # 2^30: past the bound
    assert call(ws_bytes=ws - 1) == N.ADA_ERR_WORKSPACE
    assert call(x=P + 8) == N.ADA_ERR_ALIGNMENT
    assert call(ldy=n + 4) == N.ADA_ERR_ALIGNMENT
    assert call(bias=P + 2) == N.ADA_ERR_ALIGNMENT
    assert call(ldw=k // 2 + 8) == N.ADA_ERR_ALIGNMENT        # weight rows 16-byte aligned
    assert call(ws=P + 16) == N.ADA_ERR_ALIGNMENT             # workspace 256-byte aligned


def test_w4a16_route_eligibility(monkeypatch):
    """nvfp4_linear sends a default-terms call to the W4A16 kernel only from W4A16_MIN_M tokens,
    for shapes and output views that kernel takes, and never with an explicit split-K."""
    import torch
    from adallm_b200 import nvfp4_gemm as G
    w = torch.zeros((512, 1024), dtype=torch.uint8)
    assert G._w4a16_eligible(256, 512, 2048, w, None, 0)
    assert not G._w4a16_eligible(255, 512, 2048, w, None, 0)
    assert not G._w4a16_eligible(4096, 512, 2048, w, None, 2)          # explicit split-K
    assert not G._w4a16_eligible(4096, 384, 2048, w[:384], None, 0)     # N % 256
    assert not G._w4a16_eligible(4096, 512, 2016, w[:, :1008], None, 0)  # K % 64
    wide = torch.zeros((4096, 520), dtype=torch.bfloat16)
    assert G._w4a16_eligible(4096, 512, 2048, w, wide[:, :512], 0)
    odd = torch.zeros((4096, 516), dtype=torch.bfloat16)
    assert not G._w4a16_eligible(4096, 512, 2048, w, odd[:, :512], 0)   # row stride not 16 bytes
    monkeypatch.setattr(G, "W4A16_MIN_M", 0)
    assert not G._w4a16_eligible(4096, 512, 2048, w, None, 0)
