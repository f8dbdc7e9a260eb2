"""NVFP4 linear on the B200 tensor cores (adallm_b200 C ABI ``ada_nvfp4_linear``).

Drop-in for the reference's functional API in adallm/ops/nvfp4_gemm.py:
  * nvfp4_linear(x, w_packed, w_scale, w_scale_2, w_scale_col, bias, group_size)   (:460-564)
  * nvfp4_linear_dual(x, w1_packed, w1_scale, w1_scale_2, w2_packed, w2_scale,
                      w2_scale_2, bias1, bias2, group_size)                          (:567-654)
  * nvfp4_linear_gather(x, w_packed, w_scale, w_scale_2, expert_ids, group_size)     (:657-714)
Weights keep the reference parameter layout (adallm/ops/linear.py:31-43).  The fp16
scale tensor is re-laid out once into the tensor-core scale-factor layout
(``prepack_scales``) and cached on the scale tensor.

Activation precision: ``terms`` e2m1 terms per activation row.  1 = NVFP4 activations
with per-16 block scales (W4A4, ~0.1 relative deviation from the reference); 2..8 =
row-scaled terms whose sum approximates the bf16 activation (4 terms, the default:
~5e-4 relative L2 for Gaussian rows; 6 terms: ~1e-5).  Set with the environment
variable ADALLM_B200_NVFP4_TERMS or per call.

Prefill-size calls (M >= W4A16_MIN_M = 256 tokens, N % 256 == 0, K % 64 == 0) that leave
``terms`` at its default run the reference's own W4A16 arithmetic instead
(``nvfp4_linear_w4a16``: fp16 activations, e2m1 weights widened exactly to fp16 on chip, fp32
accumulation on SM-pair tensor-core tiles), which at these sizes is also the faster form.
ADALLM_B200_W4A16_MIN_M=0 turns this off.
"""
from __future__ import annotations

import os

import torch

from . import _native as N

DEFAULT_TERMS = int(os.environ.get("ADALLM_B200_NVFP4_TERMS", "4"))
W4A16_MIN_M = int(os.environ.get("ADALLM_B200_W4A16_MIN_M", "256"))


def sf_bytes(n: int, k: int) -> int:
    return int(N.lib().ada_nvfp4_sf_bytes(n, k))


def prepack_scales(w_scale: torch.Tensor, n: int, k: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """[N, K/16] e4m3 scales (fp16 values as the reference loader stores them, or
    float8_e4m3fn / uint8 bytes) -> uint8 [sf_bytes(N, K)] in the MMA scale-factor layout."""
    N.require_cuda(w_scale, what="prepack_scales")
    if w_scale.dim() != 2 or w_scale.shape[0] != n or w_scale.shape[1] * 16 != k:
        raise ValueError("weight_scale shape does not match packed_weight")
    if w_scale.stride(-1) != 1:
        w_scale = w_scale.contiguous()
    if w_scale.dtype == torch.float16:
        is_fp16 = 1
    elif w_scale.dtype in (torch.float8_e4m3fn, torch.uint8):
        is_fp16 = 0
    else:
        w_scale = w_scale.to(torch.float16)
        is_fp16 = 1
    nbytes = sf_bytes(n, k)
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=w_scale.device)
    st = N.lib().ada_nvfp4_prepack_scales(w_scale.data_ptr(), is_fp16, w_scale.stride(0), n, k, out.data_ptr(),
                                          N.stream_ptr(w_scale.device))
    N.check(st, "nvfp4 prepack")
    return out


def _cached_sf(w_scale: torch.Tensor, n: int, k: int, owner: torch.Tensor | None = None) -> torch.Tensor:
    """Prepacked scales of w_scale ([n, k/16]), cached on `owner` (default: w_scale itself)."""
    owner = w_scale if owner is None else owner
    key = (w_scale.data_ptr(), owner._version, n, k)
    cached = getattr(owner, "_ada_sf", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    sf = prepack_scales(w_scale, n, k)
    try:
        owner._ada_sf = (key, sf)
    except Exception:
        pass
    return sf


def prepack_model(model) -> int:
    """Load-time scale prepack for a loaded model (the reference's post-load step,
    adallm/infra/loader.py:129-162, where weight_scale_col is derived): for every module whose
    `weight` is NVFP4 (uint8 [N, K/2] on a GPU) with `weight_scale` [N, K/16], derive the MMA
    scale-factor layout once and cache it on `weight_scale`, where nvfp4_linear looks it up, so
    no forward pays for it.  Modules on the CPU or in another layout are skipped.  Returns the
    number of weights prepacked."""
    done = 0
    for mod in model.modules():
        w = getattr(mod, "weight", None)
        s = getattr(mod, "weight_scale", None)
        if not isinstance(w, torch.Tensor) or not isinstance(s, torch.Tensor):
            continue
        if w.dtype != torch.uint8 or w.dim() != 2 or s.dim() != 2 or not w.is_cuda or not s.is_cuda:
            continue
        n, k = int(w.shape[0]), int(w.shape[1]) * 2
        if tuple(s.shape) != (n, k // 16) or k % 64:
            continue
        _cached_sf(s, n, k)
        done += 1
    return done


def workspace_bytes(m: int, n: int, k: int, terms: int) -> int:
    return int(N.lib().ada_nvfp4_linear_workspace_size(m, n, k, terms))


_WS: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised workspace reused per (device, stream); kernels leave it ready for reuse.
    Inside CUDA-graph capture a fresh buffer (zeroed by a captured memset) is used."""
    if torch.cuda.is_current_stream_capturing():
        return torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def check_device_errors() -> None:
    """Raise RuntimeError if an eager nvfp4 call of this process reported a failed bounded wait
    (the error word at the start of each cached workspace; synchronises).  Calls captured into a
    CUDA graph use workspaces from the graph's memory pool, which this does not read."""
    for buf in list(_WS.values()):
        N.raise_on_error_word(int(buf[:4].view(torch.int32).item()), "nvfp4_linear")


def _as_fp32_scalar(s: torch.Tensor | float, device) -> torch.Tensor:
    if isinstance(s, torch.Tensor):
        if s.dtype == torch.float32 and s.is_cuda and s.numel() == 1:
            return s
        return s.detach().to(device=device, dtype=torch.float32).reshape(())
    return torch.tensor(float(s), dtype=torch.float32, device=device)


def nvfp4_linear(x: torch.Tensor, w_packed: torch.Tensor, w_scale: torch.Tensor, w_scale_2: torch.Tensor,
                 w_scale_col: torch.Tensor | None = None, bias: torch.Tensor | None = None, group_size: int = 16,
                 terms: int | None = None, sf: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None, ksplit: int = 0) -> torch.Tensor:
    """y = x @ dequant(W)^T (+ bias) with the reference's signature.  ``w_scale_col``
    (the reference's FP8-path column scale) is accepted and unused."""
    if not x.is_cuda:
        raise RuntimeError("nvfp4_linear requires CUDA tensors")
    if group_size != 16:
        raise ValueError("adallm_b200 implements NVFP4 group size 16")
    out_dtype = x.dtype
    if x.dtype not in (torch.float16, torch.bfloat16):
        x = x.to(torch.float16)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) % 8) or (x2.data_ptr() % 16):
        x2 = x2.contiguous()
    m, k = x2.shape
    n = w_packed.shape[0]
    if w_packed.shape[1] * 2 != k:
        raise ValueError("Packed weight shape does not match input features")
    if terms is None and _w4a16_eligible(m, n, k, w_packed, out, ksplit):
        return nvfp4_linear_w4a16(x, w_packed, w_scale, w_scale_2, bias, sf, out).to(out_dtype)
    t = DEFAULT_TERMS if terms is None else int(terms)
    if sf is None:
        sf = _cached_sf(w_scale, n, k)
    g2 = _as_fp32_scalar(w_scale_2, x.device)
    ydt = x2.dtype
    y = out if out is not None else torch.empty((m, n), dtype=ydt, device=x.device)
    b = None if bias is None else bias.to(ydt).contiguous()
    if m == 0:
        return y.to(out_dtype).view(*x.shape[:-1], n)
    need = workspace_bytes(m, n, k, t)
    if need == 0:
        raise ValueError(f"nvfp4_linear: unsupported shape M={m} N={n} K={k} (needs N%128==0, K%256==0)")
    ws = workspace if workspace is not None else _workspace(x.device, need)
    st = N.lib().ada_nvfp4_linear_ex(x2.data_ptr(), N.DT[ydt], x2.stride(0), m, k, w_packed.data_ptr(),
                                     w_packed.stride(0), sf.data_ptr(), g2.data_ptr(), n, N.ptr(b), y.data_ptr(),
                                     N.DT[ydt], y.stride(0), t, int(ksplit), ws.data_ptr(), ws.numel(),
                                     N.stream_ptr(x.device))
    N.check(st, "NVFP4 kernel")
    return y.to(out_dtype).view(*x.shape[:-1], n)


def _w4a16_eligible(m: int, n: int, k: int, w_packed: torch.Tensor, out: torch.Tensor | None, ksplit: int) -> bool:
    if W4A16_MIN_M <= 0 or m < W4A16_MIN_M or ksplit or n % 256 or k % 64:
        return False
    if w_packed.stride(-1) != 1 or w_packed.stride(0) % 16 or w_packed.data_ptr() % 16:
        return False
    return out is None or (out.stride(-1) == 1 and out.stride(0) % 8 == 0 and out.data_ptr() % 16 == 0)


def nvfp4_linear_w4a16(x: torch.Tensor, w_packed: torch.Tensor, w_scale: torch.Tensor, w_scale_2: torch.Tensor,
                       bias: torch.Tensor | None = None, sf: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ dequant(W)^T (+ bias) in the reference's W4A16 arithmetic (fp16 activations,
    fp16-exact dequantised weights, fp32 accumulation; adallm/ops/nvfp4_gemm.py:460-564) on
    SM-pair tensor-core tiles, for prefill-size M.  Needs N % 256 == 0 and K % 64 == 0."""
    if not x.is_cuda:
        raise RuntimeError("nvfp4_linear_w4a16 requires CUDA tensors")
    out_dtype = x.dtype
    if x.dtype not in (torch.float16, torch.bfloat16):
        x = x.to(torch.float16)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) % 8) or (x2.data_ptr() % 16):
        x2 = x2.contiguous()
    m, k = x2.shape
    n = w_packed.shape[0]
    if w_packed.shape[1] * 2 != k:
        raise ValueError("Packed weight shape does not match input features")
    if sf is None:
        sf = _cached_sf(w_scale, n, k)
    g2 = _as_fp32_scalar(w_scale_2, x.device)
    ydt = x2.dtype
    y = out if out is not None else torch.empty((m, n), dtype=ydt, device=x.device)
    b = None if bias is None else bias.to(ydt).contiguous()
    if m == 0:
        return y.to(out_dtype).view(*x.shape[:-1], n)
    ws = _workspace(x.device, int(N.lib().ada_nvfp4_linear_w4a16_workspace_size(m, k)))
    st = N.lib().ada_nvfp4_linear_w4a16(x2.data_ptr(), N.DT[ydt], x2.stride(0), m, k, w_packed.data_ptr(),
                                        w_packed.stride(0), sf.data_ptr(), g2.data_ptr(), n, N.ptr(b), y.data_ptr(),
                                        N.DT[ydt], y.stride(0), ws.data_ptr(), ws.numel(), N.stream_ptr(x.device))
    N.check(st, "NVFP4 W4A16 kernel")
    return y.to(out_dtype).view(*x.shape[:-1], n)


def nvfp4_linear_dual(x, w1_packed, w1_scale, w1_scale_2, w2_packed, w2_scale, w2_scale_2, bias1, bias2,
                      group_size, terms: int | None = None):
    """gate and up projections sharing one activation (adallm/ops/nvfp4_gemm.py:567-654)."""
    if w1_packed.shape[0] != w2_packed.shape[0]:
        raise ValueError("Dual NVFP4 expects matching output sizes")
    y1 = nvfp4_linear(x, w1_packed, w1_scale, w1_scale_2, None, bias1, group_size, terms)
    y2 = nvfp4_linear(x, w2_packed, w2_scale, w2_scale_2, None, bias2, group_size, terms)
    return y1, y2


def nvfp4_linear_gather(x, w_packed, w_scale, w_scale_2, expert_ids, group_size, terms: int | None = None,
                        expert_base: int | None = None):
    """Row m uses expert expert_ids[m] (adallm/ops/nvfp4_gemm.py:657-714).  One grouped
    tensor-core GEMM on the device (ada_nvfp4_linear_grouped): a routing kernel gives every
    expert whole 16-row operand tiles, the quantiser gathers the rows into them and the GEMM
    streams only the weights of the experts in use.  No host synchronisation: graph-capturable.

    expert_base (expert parallelism): w_packed / w_scale / w_scale_2 hold this rank's experts
    [expert_base, expert_base + E); rows routed elsewhere are skipped and their output rows are
    left unwritten (ada_nvfp4_linear_grouped_ep)."""
    if not x.is_cuda:
        raise RuntimeError("nvfp4_linear_gather requires CUDA tensors")
    if group_size != 16:
        raise ValueError("adallm_b200 implements NVFP4 group size 16")
    x2 = x.reshape(-1, x.shape[-1])
    m, k = x2.shape
    e, n, khalf = w_packed.shape
    if khalf * 2 != k:
        raise ValueError("Packed weight shape does not match input features")
    if expert_ids.numel() != m:
        raise ValueError("expert_ids must have one entry per row in x")
    if w_scale_2 is None:
        w_scale_2 = torch.ones((e,), device=x.device, dtype=torch.float32)
    dt = x2.dtype if x2.dtype in (torch.float16, torch.bfloat16) else torch.float16
    x2 = x2.to(dt)
    if x2.stride(-1) != 1 or (x2.stride(0) % 8) or (x2.data_ptr() % 16):
        x2 = x2.contiguous()
    wp = w_packed if w_packed.is_contiguous() else w_packed.contiguous()
    sf = _cached_sf(w_scale.reshape(e * n, k // 16), e * n, k, owner=w_scale)
    g2 = w_scale_2.detach().to(device=x.device, dtype=torch.float32).reshape(e).contiguous()
    ids = expert_ids.to(device=x.device, dtype=torch.int32).reshape(m).contiguous()
    t = DEFAULT_TERMS if terms is None else int(terms)
    y = torch.empty((m, n), dtype=dt, device=x.device)
    if m == 0:
        return y.to(x.dtype).view(*x.shape[:-1], n)
    need = int(N.lib().ada_nvfp4_linear_grouped_workspace_size(m, n, k, t, e))
    if need == 0:
        raise ValueError(f"nvfp4_linear_gather: unsupported shape M={m} N={n} K={k} E={e}")
    ws = _workspace(x.device, need)
    if expert_base is None:
        st = N.lib().ada_nvfp4_linear_grouped(x2.data_ptr(), N.DT[dt], x2.stride(0), m, k, wp.data_ptr(),
                                              wp.stride(1), sf.data_ptr(), g2.data_ptr(), e, n, ids.data_ptr(),
                                              y.data_ptr(), N.DT[dt], y.stride(0), t, ws.data_ptr(), ws.numel(),
                                              N.stream_ptr(x.device))
    else:
        st = N.lib().ada_nvfp4_linear_grouped_ep(x2.data_ptr(), N.DT[dt], x2.stride(0), m, k, wp.data_ptr(),
                                                 wp.stride(1), sf.data_ptr(), g2.data_ptr(), e, int(expert_base), n,
                                                 ids.data_ptr(), y.data_ptr(), N.DT[dt], y.stride(0), t,
                                                 ws.data_ptr(), ws.numel(), N.stream_ptr(x.device))
    N.check(st, "NVFP4 grouped kernel")
    return y.to(x.dtype).view(*x.shape[:-1], n)
