"""Generate the golden fixtures in this directory by running the REFERENCE's own
Python functions (package ``adallm`` of Kukuskas/AdaLLMv2) on seeded inputs.

Run from the repository root with a checkout of the reference available:

    ADALLM_REF=<path to the reference checkout> python tests/golden/make_golden.py

The reference's ``torch.compile`` decorators are bypassed with
TORCHDYNAMO_DISABLE=1 so the eager code runs on CPU.  Its Triton kernels need
a GPU and are not run here; what is recorded is the reference's CPU-runnable
arithmetic:

  golden_nvfp4.npz   e2m1 table (adallm/infra/nvfp4.py:7-18), dequant_nvfp4
                     (adallm/infra/nvfp4.py:36-77) and the "dequant"-mode
                     linear (adallm/infra/loader.py:92-102 -> F.linear at
                     adallm/ops/linear.py:74)
  golden_kv.npz      _gather_kv_from_blocks (adallm/ops/attention.py:254-286)
                     on an fp8 paged cache, and the fp8 cast the reference's
                     torch store fallback applies (adallm/ops/attention.py:245-251)
  golden_layers.npz  RMSNorm / GemmaRMSNorm (adallm/ops/layernorm.py),
                     RotaryEmbedding (adallm/ops/rotary_embedding.py),
                     SiluAndMul / GeluAndMul (adallm/ops/activation.py)
"""
from __future__ import annotations

import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ref = os.environ.get("ADALLM_REF")
    if not ref or not os.path.isdir(os.path.join(ref, "adallm")):
        raise SystemExit("set ADALLM_REF to a checkout of the reference (directory holding adallm/)")
    sys.path.insert(0, ref)
    from adallm.infra import nvfp4 as ref_nvfp4
    from adallm.ops import attention as ref_attn
    from adallm.ops import layernorm as ref_ln
    from adallm.ops import rotary_embedding as ref_rope
    from adallm.ops import activation as ref_act

    g = torch.Generator().manual_seed(1234)

    # ---- NVFP4 -------------------------------------------------------------
    lut = ref_nvfp4._FP4_E2M1_LUT.numpy().astype(np.float32)
    n, k = 96, 256
    packed = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8)
    # e4m3 scale values stored in fp16 params, as the loader does (adallm/ops/linear.py:38-41)
    sbits = torch.randint(0, 0x7F, (n, k // 16), generator=g, dtype=torch.int32).to(torch.uint8)
    scale = sbits.view(torch.float8_e4m3fn).to(torch.float16)
    scale_2 = torch.tensor(0.0123, dtype=torch.float32)
    deq = ref_nvfp4.dequant_nvfp4(packed, scale, scale_2, 16, torch.float32)
    x = torch.randn((8, k), generator=g).to(torch.bfloat16)
    w_bf16 = ref_nvfp4.dequant_nvfp4(packed, scale, scale_2, 16, torch.bfloat16)
    y = torch.nn.functional.linear(x, w_bf16)
    np.savez_compressed(
        os.path.join(HERE, "golden_nvfp4.npz"),
        lut=lut, packed=packed.numpy(), scale_bits=sbits.numpy(), scale_fp16=scale.numpy(),
        scale_2=scale_2.numpy(), dequant=deq.numpy(), x_bf16=_bf16_bits(x), y_bf16=_bf16_bits(y),
    )

    # ---- paged KV ----------------------------------------------------------
    pages, page, hkv, d = 24, 16, 2, 32
    kc = torch.randn((pages, page, hkv, d), generator=g).to(torch.float8_e4m3fn)
    vc = torch.randn((pages, page, hkv, d), generator=g).to(torch.float8_e4m3fn)
    ctx = torch.tensor([5, 33, 0, 16, 47], dtype=torch.int32)
    perm = torch.randperm(pages, generator=g).to(torch.int32)
    bt = torch.full((5, 4), -1, dtype=torch.int32)
    off = 0
    for i, c in enumerate(ctx.tolist()):
        nb = (c + page - 1) // page
        bt[i, :nb] = perm[off: off + nb]
        off += nb
    k_out, v_out, cu = ref_attn._gather_kv_from_blocks(kc, vc, bt, ctx)
    # fp8 cast used by the reference's torch store fallback; every bf16 value in [-448, 448]
    allbits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    allf = allbits.float()
    inrange = allbits[(allf.abs() <= 448) & torch.isfinite(allf)]
    cast = inrange.to(torch.float8_e4m3fn).view(torch.uint8)
    np.savez_compressed(
        os.path.join(HERE, "golden_kv.npz"),
        k_cache=kc.view(torch.uint8).numpy(), v_cache=vc.view(torch.uint8).numpy(),
        block_tables=bt.numpy(), context_lens=ctx.numpy(),
        k_out=k_out.numpy(), v_out=v_out.numpy(), cu=cu.numpy(),
        cast_in_bf16=_bf16_bits(inrange), cast_out_e4m3=cast.numpy(),
    )

    # ---- norms / rope / activations ----------------------------------------
    t, hid = 6, 256
    xb = (torch.randn((t, hid), generator=g) * 3).to(torch.bfloat16)
    rb = torch.randn((t, hid), generator=g).to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn((hid,), generator=g)).to(torch.bfloat16)
    wg = (0.1 * torch.randn((hid,), generator=g)).to(torch.bfloat16)
    rms = ref_ln.RMSNorm(hid, eps=1e-6).to(torch.bfloat16)
    rms.weight.data.copy_(wq)
    y_rms = rms(xb)
    y_add, r_add = rms(xb, rb)
    gem = ref_ln.GemmaRMSNorm(hid, eps=1e-6).to(torch.bfloat16)
    gem.weight.data.copy_(wg)
    y_g = gem(xb)
    y_gadd, r_gadd = gem(xb, rb)

    hq, hk, hd = 4, 2, 64
    rope = ref_rope.RotaryEmbedding(hd, hd, 512, 1e6, None)
    rope_lin = ref_rope.RotaryEmbedding(hd, hd, 512, 1e4, {"rope_type": "linear", "factor": 8.0})
    pos = torch.tensor([0, 1, 7, 100, 511, 300], dtype=torch.long)
    q = torch.randn((t, hq, hd), generator=g).to(torch.bfloat16)
    kk = torch.randn((t, hk, hd), generator=g).to(torch.bfloat16)
    q1, k1 = rope(pos, q, kk)
    q2, k2 = rope_lin(pos, q, kk)

    a = torch.randn((t, 2 * hid), generator=g).to(torch.bfloat16)
    y_silu = ref_act.SiluAndMul()(a)
    y_gelu = ref_act.GeluAndMul("tanh")(a)
    np.savez_compressed(
        os.path.join(HERE, "golden_layers.npz"),
        x=_bf16_bits(xb), r=_bf16_bits(rb), w=_bf16_bits(wq), wg=_bf16_bits(wg),
        y_rms=_bf16_bits(y_rms), y_add=_bf16_bits(y_add), r_add=_bf16_bits(r_add),
        y_g=_bf16_bits(y_g), y_gadd=_bf16_bits(y_gadd), r_gadd=_bf16_bits(r_gadd),
        pos=pos.numpy(), q=_bf16_bits(q), k=_bf16_bits(kk),
        cache=rope.cos_sin_cache.numpy(), cache_lin=rope_lin.cos_sin_cache.numpy(),
        q1=_bf16_bits(q1), k1=_bf16_bits(k1), q2=_bf16_bits(q2), k2=_bf16_bits(k2),
        a=_bf16_bits(a), y_silu=_bf16_bits(y_silu), y_gelu=_bf16_bits(y_gelu),
    )
    print("wrote golden fixtures to", HERE)


if __name__ == "__main__":
    main()
