"""The reference's own Triton kernels, run on this GPU, against the oracle's restatements of
their arithmetic -- pinning the "reference numerics" emulation the agreement tests compare with,
and the W4A8 restatement.  Runs in its own process (``python -m tests.ref_triton_check MODE``),
since the reference reads NVFP4_FP8 when its module is imported (nvfp4_gemm.py:23-40).

  gemm     nvfp4_linear (nvfp4_gemm.py:460-564) on BASELINE config 0 (x bf16 [16, 4096],
           W [12288, 4096] quantised from N(0, 0.02)): with NVFP4_FP8=0 the fp16 kernel
           (:58-136) against oracle.decode's "reference" linear; with NVFP4_FP8=1 the W4A8 kernel
           (:252-360) against oracle.nvfp4.linear_w4a8_ref.  Also reports how far each, and this
           package's nvfp4_linear (4 activation terms), sit from the exact W4A16 product.
  attn     fp8_kv_decode_group_kernel (attention.py:126-233) through Attention.forward's decode
           branch at page 256 (the page size the reference's engine requires, settings.py:152;
           its kernel walks pages in 64-token steps, so smaller pages are outside its contract)
           against oracle.attention.paged_decode_fp16_kernel and the fp64 paged_decode.

  prefill  the prefix-cache prefill branch of Attention.forward (attention.py:335-358: its
           _gather_kv_from_blocks of the e4m3 pages to fp16, then flash_attn_varlen_func with
           causal=True and window (W, 0)) against oracle.attention.paged_prefill -- the
           restatement of flash-attn's bottom-right causal mask and window -- and against this
           package's paged prefill kernel, on ragged cached/new lengths with and without a window.

One JSON line ("REFTRITON {...}").  Test infrastructure only (tests/test_gpu_reference_triton.py)."""
from __future__ import annotations

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.environ.get("ADALLM_REF", os.path.join(ROOT, "baseline", "_ref"))


def _path():
    for p in (ROOT, REF_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)


def gemm() -> dict:
    _path()
    import numpy as np
    import torch
    import adallm.ops.nvfp4_gemm as rg
    from oracle import nvfp4 as nv
    from adallm_b200.nvfp4_gemm import nvfp4_linear
    d = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    w = (torch.randn((12288, 4096), generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    packed, sbits, s2 = nv.quantize_weight(w)
    scale16 = nv.e4m3_decode(sbits).astype(np.float16)
    x = torch.randn((16, 4096), generator=g).to(torch.bfloat16)
    pk, sc = torch.from_numpy(packed), torch.from_numpy(scale16)
    exact = nv.linear_ref(x.float().numpy(), packed, scale16.astype(np.float32), s2)
    tri = rg.nvfp4_linear(x.to(d), pk.to(d), sc.to(d), torch.tensor(s2, device=d), None, None, 16)
    torch.cuda.synchronize()
    tri = tri.float().cpu().numpy()
    if rg._FP8_ENABLED:
        oracle = nv.linear_w4a8_ref(x.float().numpy(), pk, sc, s2).float().numpy()
        mode = "w4a8"
    else:
        w16 = nv.dequant_nvfp4_kernel_fp16(pk, sc, s2).float()
        oracle = (x.to(torch.float16).float() @ w16.t()).to(torch.float16).to(torch.bfloat16).float().numpy()
        mode = "w4a16"
    ours = nvfp4_linear(x.to(d), pk.to(d), sc.to(d), torch.tensor(s2, device=d), None, None, 16)
    torch.cuda.synchronize()
    return {"mode": mode, "triton_vs_oracle": nv.rel_l2(tri, oracle), "triton_vs_exact": nv.rel_l2(tri, exact),
            "oracle_vs_exact": nv.rel_l2(oracle, exact), "ours_vs_exact": nv.rel_l2(ours.float().cpu().numpy(), exact)}


def gemm_prefill() -> dict:
    """The reference's fp16 NVFP4 GEMM (NVFP4_FP8=0) at prefill size (1024 tokens) against this
    package's W4A16 kernel, called directly and through nvfp4_linear's route from 256 tokens:
    the same fp16 operands and fp32 accumulation; the reference folds scale_2 into its fp16
    weights (one more rounding), this package applies it in fp32 after the sum."""
    _path()
    import numpy as np
    import torch
    import adallm.ops.nvfp4_gemm as rg
    from oracle import nvfp4 as nv
    from adallm_b200.nvfp4_gemm import nvfp4_linear, nvfp4_linear_w4a16
    d = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(1)
    w = (torch.randn((4096, 4096), generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    packed, sbits, s2 = nv.quantize_weight(w)
    scale16 = nv.e4m3_decode(sbits).astype(np.float16)
    x = torch.randn((1024, 4096), generator=g).to(torch.bfloat16)
    pk, sc, s2t = torch.from_numpy(packed).to(d), torch.from_numpy(scale16).to(d), torch.tensor(s2, device=d)
    exact = nv.linear_ref(x.float().numpy(), packed, scale16.astype(np.float32), s2)
    tri = rg.nvfp4_linear(x.to(d), pk, sc, s2t, None, None, 16)
    ours = nvfp4_linear(x.to(d), pk, sc, s2t, None, None, 16)
    direct = nvfp4_linear_w4a16(x.to(d), pk, sc, s2t)
    torch.cuda.synchronize()
    tri_np, ours_np = tri.float().cpu().numpy(), ours.float().cpu().numpy()
    return {"mode": "w4a8" if rg._FP8_ENABLED else "w4a16", "routed_equals_direct": bool(torch.equal(ours, direct)),
            "ours_vs_triton": nv.rel_l2(ours_np, tri_np), "triton_vs_exact": nv.rel_l2(tri_np, exact),
            "ours_vs_exact": nv.rel_l2(ours_np, exact)}


def attn() -> dict:
    _path()
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    import numpy as np
    import torch
    import torch.distributed as dist
    import adallm.infra.context as rc
    import adallm.ops.attention as ra
    from adallm.infra.quant import get_quant_config
    from oracle import attention as oa
    from oracle.nvfp4 import rel_l2
    d = torch.device("cuda", 0)
    get_quant_config().fp8_decode_kernel_enabled = True
    case = oa.make_paged_case(11, batch=4, hq=32, hkv=8, d=128, page=256, ctx_lo=300, ctx_hi=2000)
    m = ra.Attention(32, 128, float(case["scale"]), 8)
    m.k_cache = torch.from_numpy(case["k"]).to(d).view(torch.float8_e4m3fn)
    m.v_cache = torch.from_numpy(case["v"]).to(d).view(torch.float8_e4m3fn)
    q = torch.from_numpy(case["q"]).to(torch.bfloat16).to(d)
    rc.set_context(False, slot_mapping=torch.full((4,), -1, dtype=torch.int32, device=d),
                   context_lens=torch.from_numpy(case["context_lens"]).to(d),
                   block_tables=torch.from_numpy(case["block_tables"]).to(d), max_seqlen_k=2000)
    kv = torch.zeros((4, 8, 128), dtype=torch.bfloat16, device=d)
    out = m.forward(q, kv, kv)  # slot -1: nothing stored, the cache is read as built
    torch.cuda.synchronize()
    rc.reset_context()
    tri = out.float().cpu().numpy()
    emul = oa.paged_decode_fp16_kernel(case["q"], case["k"], case["v"], case["block_tables"], case["context_lens"],
                                       case["scale"])
    emul = torch.from_numpy(emul).to(torch.bfloat16).float().numpy()
    exact = oa.paged_decode(case["q"], case["k"], case["v"], case["block_tables"], case["context_lens"],
                            case["scale"])
    return {"triton_vs_emulation": rel_l2(tri, emul), "triton_vs_exact": rel_l2(tri, exact),
            "emulation_vs_exact": rel_l2(emul, exact), "page": 256}


def prefill() -> dict:
    _path()
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    import numpy as np
    import torch
    import adallm.infra.context as rc
    import adallm.ops.attention as ra
    from oracle import attention as oa
    from oracle.nvfp4 import rel_l2
    from adallm_b200.attention import paged_prefill
    d = torch.device("cuda", 0)
    cases = [  # cached, new, hq, hkv, page, window
        ([0, 37, 300, 5], [50, 1, 129, 3], 32, 8, 16, 0),
        ([0, 37, 300, 5], [50, 1, 129, 3], 32, 8, 16, 40),
        ([100, 0], [77, 200], 32, 4, 64, 0),
        ([3, 250], [130, 60], 4, 4, 16, 17),
    ]
    res = []
    for i, (cached, new, hq, hkv, page, window) in enumerate(cases):
        c = oa.make_prefill_case(100 + i, cached, new, hq, hkv, 128, page, extra_pages=3)
        m = ra.Attention(hq, 128, float(c["scale"]), hkv, sliding_window=window or None)
        m.k_cache = torch.from_numpy(c["k"]).to(d).view(torch.float8_e4m3fn)
        m.v_cache = torch.from_numpy(c["v"]).to(d).view(torch.float8_e4m3fn)
        q = torch.from_numpy(c["q"]).to(torch.bfloat16).to(d)
        tq = q.shape[0]
        len_k = np.diff(c["cu_k"])
        rc.set_context(True, cu_seqlens_q=torch.from_numpy(c["cu_q"]).to(d),
                       cu_seqlens_k=torch.from_numpy(c["cu_k"]).to(d), max_seqlen_q=int(c["max_seqlen_q"]),
                       max_seqlen_k=int(len_k.max()), slot_mapping=torch.full((tq,), -1, dtype=torch.int32, device=d),
                       block_tables=torch.from_numpy(c["block_tables"]).to(d))
        kv = torch.zeros((tq, hkv, 128), dtype=torch.bfloat16, device=d)
        ref_out = m.forward(q, kv, kv)  # slot -1: nothing stored, the cache is read as built
        torch.cuda.synchronize()
        rc.reset_context()
        ref_out = ref_out.float().cpu().numpy().reshape(tq, hq, 128)
        oracle = oa.paged_prefill(c["q"], c["k"], c["v"], c["block_tables"], c["cu_q"], c["cu_k"], c["scale"],
                                  window)
        ours = paged_prefill(q, m.k_cache, m.v_cache, torch.from_numpy(c["block_tables"]).to(d),
                             torch.from_numpy(c["cu_q"]).to(d), torch.from_numpy(c["cu_k"]).to(d),
                             int(c["max_seqlen_q"]), float(c["scale"]), window)
        torch.cuda.synchronize()
        ours = ours.float().cpu().numpy().reshape(tq, hq, 128)
        res.append({"case": i, "window": window, "reference_vs_oracle": rel_l2(ref_out, oracle),
                    "ours_vs_reference": rel_l2(ours, ref_out), "ours_vs_oracle": rel_l2(ours, oracle)})
    return {"cases": res, "reference_vs_oracle_max": max(r["reference_vs_oracle"] for r in res),
            "ours_vs_reference_max": max(r["ours_vs_reference"] for r in res)}


def main():
    if not os.path.isdir(os.path.join(REF_DIR, "adallm")):
        print("REFTRITON " + json.dumps({"unavailable": f"reference package not found in {REF_DIR}"}))
        return
    r = {"gemm": gemm, "gemm_prefill": gemm_prefill, "attn": attn, "prefill": prefill}[sys.argv[1]]()
    print("REFTRITON " + json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
