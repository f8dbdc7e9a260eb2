"""ctypes binding of the adallm_b200 C ABI (include/adallm_b200.h).

The CUDA library is built in-tree (``python -m adallm_b200.build``) and loaded
from ``adallm_b200/_lib``.  There is no CPU or PyTorch fallback: if the library
is missing, every op raises.  Status codes map to the reference's exception
types: shape / argument problems raise ValueError (as adallm/ops/nvfp4_gemm.py:477-478
does), launch and device failures raise RuntimeError with "no fallback" wording
(as adallm/ops/nvfp4_gemm.py:532-535 and adallm/ops/attention.py:409-414 do).
"""
from __future__ import annotations

import ctypes as C
import os
import re

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libadallm_b200.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "adallm_b200.h")

ADA_OK = 0
ADA_ERR_INVALID_ARG = 1
ADA_ERR_UNSUPPORTED = 2
ADA_ERR_ALIGNMENT = 3
ADA_ERR_WORKSPACE = 4
ADA_ERR_LAUNCH = 5
ADA_ERR_TIMEOUT = 6
ADA_ERR_CUDA = 7

DT = {torch.bfloat16: 0, torch.float16: 1}

P, I32, I64, F32, INT, SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_int, C.c_size_t
PP, U32 = C.POINTER(C.c_void_p), C.c_uint32

# name -> (restype, argtypes)
_SIGS = {
    "ada_status_string": (C.c_char_p, [INT]),
    "ada_abi_version": (INT, []),
    "ada_set_pdl": (INT, [INT]),
    "ada_set_pair_gemm": (INT, [INT]),
    "ada_fp8_paged_decode_workspace_size": (SZ, [I32, I32, I32, I32, I32]),
    "ada_fp8_paged_decode": (INT, [P, INT, I64, I64, P, P, I64, I64, I64, I64, P, I64, I32, P, I32, I32, I32, I32, I32,
                                   F32, F32, F32, I32, P, INT, P, SZ, P]),
    "ada_fp8_paged_decode_quant": (INT, [P, INT, I64, I64, P, P, I64, I64, I64, I64, P, I64, I32, P, I32, I32, I32,
                                         I32, I32, F32, F32, F32, I32, P, INT, INT, INT, P, P, P, P, SZ, P]),
    "ada_fp8_paged_decode_quant_ex": (INT, [P, INT, I64, I64, P, P, I64, I64, I64, I64, P, I64, I32, P, I32, I32, I32,
                                            I32, I32, F32, F32, F32, I32, P, INT, INT, INT, P, P, P, P, SZ, I32, P]),
    "ada_fp8_paged_prefill": (INT, [P, INT, I64, I64, P, P, I64, I64, I64, I64, P, I64, I32, P, P, I32, I32, I32,
                                    I32, I32, I32, F32, F32, F32, I32, P, INT, I64, I64, P, P]),
    "ada_rmsnorm_quant": (INT, [P, I64, P, I64, P, I64, P, P, I64, I64, I32, F32, INT, INT, INT, INT, P, P, P, P]),
    "ada_gated_act_quant": (INT, [P, I64, P, I64, I64, I32, INT, INT, INT, INT, P, P, P, P]),
    "ada_store_kvcache_fp8": (INT, [P, P, INT, I64, I32, I32, I64, I64, P, P, P, I64, F32, F32, P]),
    "ada_rmsnorm": (INT, [P, I64, P, I64, P, I64, P, P, I64, I64, I32, F32, INT, INT, P]),
    "ada_rope": (INT, [P, P, I64, P, I64, P, P, I64, I32, I32, I32, P, I64, INT, P]),
    "ada_gated_act": (INT, [P, I64, P, I64, I64, I32, INT, INT, P]),
    "ada_qk_norm_rope_store": (INT, [P, I64, I64, I32, I32, I32, P, P, F32, P, P, I64, P, P, P, F32, F32, P, P,
                                     INT, P]),
    "ada_embedding": (INT, [P, I64, P, I64, I64, I32, P, INT, P]),
    "ada_gemma_norm2_quant_parts": (INT, [P, I32, I64, I64, P, P, I64, P, I64, P, P, I64, I64, I32, F32, INT, INT,
                                         INT, P, P, P, P]),
    "ada_qk_norm_rope_store_parts_ex": (INT, [P, I32, I64, I64, I64, I32, I32, I32, P, P, F32, INT, P, P, I64, P, P,
                                             P, F32, F32, P, P, INT, P]),
    "ada_qk_norm_rope_store_ex": (INT, [P, I64, I64, I32, I32, I32, P, P, F32, INT, P, P, I64, P, P, P, F32, F32, P, P,
                                       INT, P]),
    "ada_lm_head_workspace_size": (SZ, [I64, I64]),
    "ada_lm_head_argmax": (INT, [P, I64, I64, I64, P, I64, I64, I64, P, I64, P, P, P, SZ, P]),
    "ada_nvfp4_gemm_partials_pf": (INT, [P, P, P, I64, INT, INT, P, I64, P, P, I64, I64, P, I64, I64, INT, P, SZ, P,
                                        SZ, P, SZ, P]),
    "ada_argmax_workspace_size": (SZ, [I64, I64]),
    "ada_argmax": (INT, [P, I64, I64, I64, INT, P, P, SZ, P]),
    "ada_argmax_noalloc": (INT, [P, I64, I64, I64, INT, P, P]),
    "ada_nvfp4_sf_bytes": (SZ, [I64, I64]),
    "ada_nvfp4_prepack_scales": (INT, [P, INT, I64, I64, I64, P, P]),
    "ada_nvfp4_linear_workspace_size": (SZ, [I64, I64, I64, INT]),
    "ada_nvfp4_linear": (INT, [P, INT, I64, I64, I64, P, I64, P, P, I64, P, P, INT, I64, INT, P, SZ, P]),
    "ada_nvfp4_linear_w4a16_workspace_size": (SZ, [I64, I64]),
    "ada_nvfp4_linear_w4a16": (INT, [P, INT, I64, I64, I64, P, I64, P, P, I64, P, P, INT, I64, P, SZ, P]),
    "ada_nvfp4_linear_ex": (INT, [P, INT, I64, I64, I64, P, I64, P, P, I64, P, P, INT, I64, INT, INT, P, SZ, P]),
    "ada_nvfp4_workspace_status": (INT, [P, I64, I64, I64, INT, P, P]),
    "ada_nvfp4_act_quant": (INT, [P, INT, I64, I64, I64, INT, INT, P, P, P, P]),
    "ada_nvfp4_block_n": (INT, [I64, INT]),
    "ada_nvfp4_gemm_workspace_size": (SZ, [I64, I64, I64, INT]),
    "ada_nvfp4_gemm": (INT, [P, P, P, I64, INT, INT, P, I64, P, P, I64, I64, P, P, INT, I64, INT, P, SZ, P]),
    "ada_nvfp4_gemm_splits": (INT, [I64, I64, I64, INT]),
    "ada_moe_route_topk": (INT, [P, INT, I64, I64, I32, I32, I32, P, P, P]),
    "ada_moe_combine": (INT, [P, INT, I64, P, I64, I32, I32, P, I64, P]),
    "ada_moe_combine_ep": (INT, [P, INT, I64, P, P, I32, I32, I64, I32, I32, P, I64, P]),
    "ada_moe_experts_workspace_size": (SZ, [I64, I32, I64, I64, INT, I32]),
    "ada_moe_experts": (INT, [P, INT, I64, I64, I32, P, I32, I32, I32, P, I64, P, P, P, I64, P, P, I64, I64, INT, P,
                              I64, INT, P, SZ, P]),
    "ada_moe_router_topk": (INT, [P, INT, I64, I64, P, I64, I32, I32, I32, I32, P, P, P, P]),
    "ada_moe_combine_ep_f32": (INT, [P, INT, I64, P, P, I32, I32, I64, I32, I32, P, I64, P]),
    "ada_nvfp4_linear_grouped_ep": (INT, [P, INT, I64, I64, I64, P, I64, P, P, I32, I32, I64, P, P, INT, I64, INT,
                                          P, SZ, P]),
    "ada_nvfp4_linear_grouped_workspace_size": (SZ, [I64, I64, I64, INT, I32]),
    "ada_nvfp4_linear_grouped": (INT, [P, INT, I64, I64, I64, P, I64, P, P, I32, I64, P, P, INT, I64, INT, P, SZ,
                                       P]),
    "ada_nvfp4_gemm_partials": (INT, [P, P, P, I64, INT, INT, P, I64, P, P, I64, I64, P, I64, I64, INT, P, SZ, P]),
    "ada_rmsnorm_quant_parts": (INT, [P, I32, I64, I64, P, I64, P, I64, P, P, I64, I64, I32, F32, INT, INT, INT, INT,
                                      P, P, P, P]),
    "ada_rmsnorm_quant_combine": (INT, [P, I64, P, I32, P, I64, P, I64, P, P, I64, I64, I32, F32, INT, INT, INT, INT,
                                        P, P, P, P]),
    "ada_peer_alloc": (INT, [SZ, PP, P]),
    "ada_peer_open": (INT, [P, PP]),
    "ada_peer_close": (INT, [P]),
    "ada_peer_free": (INT, [P]),
    "ada_tp_epoch_advance": (INT, [P, P]),
    "ada_nvfp4_gemm_ctas": (INT, [I64, I64, I64, INT, INT]),
    "ada_nvfp4_gemm_partials_peer": (INT, [P, P, P, I64, INT, INT, P, I64, P, P, I64, I64, I64, I64, INT, I32, I32, P,
                                           P, U32, U32, P, SZ, P]),
    "ada_rmsnorm_quant_peer": (INT, [P, I32, I64, I64, P, I64, P, I64, P, P, I64, I64, I32, F32, INT, INT, INT, INT,
                                     P, P, P, P, U32, U32, P, P]),
    "ada_gated_act_quant_parts": (INT, [P, I32, I64, I64, P, I64, I64, I32, INT, INT, INT, INT, P, P, P, P]),
    "ada_qk_norm_rope_store_parts": (INT, [P, I32, I64, I64, I64, I32, I32, I32, P, P, F32, P, P, I64, P, P, P, F32,
                                           F32, P, P, INT, P]),
}

_lib = None


class NativeLibraryMissing(RuntimeError):
    pass


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"adallm_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -m adallm_b200.build`. There is no CPU/PyTorch fallback.")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        if os.environ.get("ADALLM_B200_PDL", "1") == "0":
            h.ada_set_pdl(0)
        if os.environ.get("ADALLM_B200_PAIR_GEMM", "1") == "0":
            h.ada_set_pair_gemm(0)
        _lib = h
    return _lib


def declared_symbols() -> list[str]:
    """Entry points declared in include/adallm_b200.h."""
    with open(HEADER, "r", encoding="utf-8") as f:
        text = f.read()
    return sorted(set(re.findall(r"^ADA_API\s+(?:const\s+)?\w+\*?\s+\**(ada_\w+)\s*\(", text, flags=re.M)))


def check(status: int, what: str) -> None:
    if status == ADA_OK:
        return
    msg = lib().ada_status_string(status).decode()
    if status in (ADA_ERR_INVALID_ARG, ADA_ERR_UNSUPPORTED, ADA_ERR_ALIGNMENT, ADA_ERR_WORKSPACE):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({msg}); no fallback is allowed in this runtime.")


# Codes the kernels OR into a device error word (a workspace's first 4 bytes) when a bounded
# wait runs out (~2 s) or an input is out of range; the word stays set until the caller clears it.
_ERROR_BITS = [(0x1, "GEMM producer waited for a free pipeline stage"),
               (0x2, "GEMM MMA issuer waited for a loaded stage"),
               (0x4, "GEMM epilogue waited for the accumulator"),
               (0x8, "GEMM MMA issuer waited for a free accumulator")]
_ERROR_CODES = {0x50: "a peer's partial planes never arrived (tensor-parallel inbox wait)",
                0x60: "an expert id outside [0, num_experts)",
                0x70: "a prefill attention tile load never completed",
                0x80: "a router logit never arrived (fused MoE router wait)"}


def describe_error_word(code: int) -> str:
    parts = [txt for bit, txt in _ERROR_BITS if code & bit]
    hi = code & ~0xF
    if hi:
        parts.append(_ERROR_CODES.get(hi, f"code 0x{hi:x}"))
    return "; ".join(parts) or "ok"


def raise_on_error_word(code: int, what: str) -> None:
    """Raise RuntimeError when a device error word is nonzero (the results it guards are not valid)."""
    if code:
        raise RuntimeError(f"{what}: device error word 0x{code:x} ({describe_error_word(code)}); "
                           "the results of this call are not valid; no fallback is allowed in this runtime.")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def ptr_array(addrs: list[int]) -> C.Array:
    """A host array of device pointers (for the entry points that take `T* const*`)."""
    return (C.c_void_p * len(addrs))(*addrs)


def require_cuda(*tensors: torch.Tensor, what: str) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{what} requires CUDA tensors")
