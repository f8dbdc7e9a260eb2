#!/usr/bin/env python
"""Decode throughput of the adallm_b200 hot path on B200.

Metric: decode tok/s of a Qwen3-8B-shape model at batch 16 -- 36 layers,
hidden 4096, 32 query / 8 KV heads of 128, SwiGLU 12288, vocab 151936, random-init NVFP4
weights, FP8 paged KV (page 16), greedy decode after a 16-token random prompt.

One "step" = one full decode step for the 16 sequences (all layers, lm_head, greedy pick),
replayed from a CUDA graph.  The weights (~5.2 GB per step at TP=1) are far larger than the
126 MB L2, so every step streams them from HBM; no L2 flush is needed.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

N > 1 runs tensor parallelism over N ranks (launched with torch.distributed.run, NCCL
all-reduce after the row-parallel projections), so `scaling` is "strong": the batch of 16
is fixed and split by heads / columns across the GPUs.

`--impl reference` times the reference's own CPU decode path on the host cores: the reference
package (installed beside the repository in baseline/_ref) building its Qwen3ForCausalLM with
bf16-dequantised weights, F.linear and its page gather + SDPA (oracle/reference_cpu.py); only
rank 0 runs it.  The cpu_baseline leg of our arm times the same code on a few steps.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (Qwen3-8B shape, bs16)"
WORKLOAD = ("Qwen3-8B-shape decode step: 36 layers, hidden 4096, 32q/8kv heads x128, SwiGLU 12288, "
            "vocab 151936, random-init NVFP4 weights, FP8 paged KV page 16, batch 16, 16-token prompt, greedy")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--layers", type=int, default=36, help="decoder layers (36 = the Qwen3-8B shape)")
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--terms", type=int, default=4, help="activation e2m1 terms (1 = W4A4 NVFP4, 2..8 row-scaled)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel and other-config lines")
    ap.add_argument("--cpu-reps", type=int, default=3)
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def measured_bf16():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return None


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one captured launch of the decode
# GEMM in partial-plane mode divided by its algorithmic bytes: 28,746,752 / 28,835,840 (ncu
# --set full on the down projection, M 16 N 4096 K 12288; the planes stay in L2, no writes).
# Every projection of the mix is dominated by the same weight stream, so the mix's per-launch
# traffic is this ratio times its algorithmic bytes.
GEMM_DRAM_PER_ALG_BYTE = 28746752 / 28835840


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    def __init__(self, index: int, period_s: float = 0.01):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in names.items():
                    if mask & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def seq_len(args) -> int:
    """Context length at the end of our arm's timed steps: the prompt, then warm-up + timed steps
    of the device loop and again of the host-fed loop."""
    return args.prompt + 2 * (args.warmup + args.steps)


def bench_config(args, world: int) -> dict:
    """The workload both arms report (identical dicts, so the runs compare like for like)."""
    return {"workload": WORKLOAD, "global_batch": args.batch, "seq_len": seq_len(args),
            "parallelism": f"tp{world}", "layers": args.layers, "nvfp4_act_terms": args.terms,
            "l2": "inputs larger than L2 (every step streams ~5.2 GB of weights at tp1)"}


class CpuReference:
    """The reference's decode step on the host cores, one code path for both CPU legs: the
    reference package's own Qwen3ForCausalLM with dequantised bf16 weights, F.linear, its page
    gather and SDPA (oracle/reference_cpu.py), all layers, at context seq_len(args).  Falls back
    to the oracle's restatement (one full-size layer scaled to all layers, kind "port") only when
    the reference package is not importable."""

    def __init__(self, args):
        from oracle import reference_cpu
        ok, why = reference_cpu.available()
        self.kind = "reference" if ok else "port"
        self.why = why
        self.ctx = seq_len(args)
        self.layers = args.layers
        t0 = time.perf_counter()
        if ok:
            self.r = reference_cpu.ReferenceCpuDecode(layers=args.layers, batch=args.batch, ctx=self.ctx)
            self.threads = self.r.threads
        else:
            from oracle.baseline import CpuDecodeSample
            self.r = CpuDecodeSample(args.layers, 4096, 32, 8, 128, 12288, 151936, args.batch, self.ctx)
            self.threads = self.r.threads
        self.setup_s = time.perf_counter() - t0

    def step(self) -> float:
        if self.kind == "reference":
            return self.r.step()
        t1 = self.r.one_step()
        th = self.r.lm_head_time()
        return th + self.layers * max(t1 - th, 0.0)

    def sample(self, steps: int, warmup: int) -> str:
        if self.kind == "reference":
            return (f"{steps} full decode steps (all {self.layers} layers, lm_head, greedy) after {warmup} warm-up "
                    f"steps at context {self.ctx}, the reference package's Qwen3ForCausalLM on the host cores: "
                    f"weights dequantised to bf16 by its dequant_nvfp4 (setup {self.setup_s:.0f} s, untimed), "
                    f"F.linear, its _gather_kv_from_blocks + SDPA")
        return (f"{steps} steps of one full-size layer + lm_head scaled to {self.layers} layers "
                f"(oracle restatement; reference not importable: {self.why})")


def cpu_baseline(args):
    """Bounded sample of the reference's CPU decode step (rank 0, N = 1)."""
    ref = CpuReference(args)
    ref.step()
    steps = max(1, args.cpu_reps)
    ts = [ref.step() for _ in range(steps)]
    return {"value": args.batch * steps / sum(ts), "unit": "tok/s", "cores": ref.threads, "kind": ref.kind,
            "sample": ref.sample(steps, 1)}


def kernel_benches(dev, peak):
    """The two kernels BASELINE's metric quotes besides the decode step, each on its own, two
    ways, CUDA events on the launching stream:
      * cold: one call after a 256 MiB buffer was written (L2 flushed; only the call timed);
      * steady: calls back to back in a CUDA graph, rotating over copies of the weights / KV
        pools that together exceed L2, so every call streams cold operands (the way the op
        runs inside a model); per-call time.
      * config 0: NVFP4 linear x bf16 [16, 4096] . W [12288, 4096] (act-quant + GEMM, the
        drop-in nvfp4_linear) -- algorithmic bytes W 25,165,824 + e4m3 scales 3,145,728 +
        x 131,072 + y 393,216 + 4;
      * config 1: FP8 paged decode attention B16 Hq32 Hkv8 D128, ctx ~ U[512, 8192], page 16,
        seeded random page permutation (split + merge kernels) -- algorithmic bytes
        2*sum(ctx)*Hkv*D (e4m3 K and V) + q + out + 4*sum(pages) + 4*B."""
    import torch
    from adallm_b200.attention import paged_decode, paged_decode_workspace_bytes
    from adallm_b200.decode_step import random_nvfp4
    from adallm_b200.nvfp4_gemm import nvfp4_linear, nvfp4_linear_w4a16, prepack_scales, workspace_bytes

    st = torch.cuda.current_stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(reps):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            fn()
            b.record(st)
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts) * 1e3  # us

    def steady(calls, reps=5):
        """Per-call time of `calls` (closures) launched back to back, captured in one graph."""
        for fn in calls:
            fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for fn in calls:
                fn()
        gr.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(reps):
            gr.replay()
        b.record(st)
        b.synchronize()
        del gr
        return a.elapsed_time(b) * 1e3 / (reps * len(calls))

    def line(us, nb, extra):
        d = {"us": round(us, 2), "alg_bytes": nb, "gbs": round(nb / us / 1e3, 1), "frac": round(nb / us / 1e3 / peak, 4)}
        d.update(extra)
        return d

    out = {}
    m, n, k = 16, 12288, 4096
    copies = []
    for i in range(8):  # 8 x 28.8 MB of weights > L2
        packed, scale, s2 = random_nvfp4(n, k, 4242 + i, dev)
        copies.append((packed, scale, prepack_scales(scale, n, k), torch.tensor(s2, dtype=torch.float32, device=dev)))
    x = torch.randn((m, k), device=dev, dtype=torch.bfloat16)
    y = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
    ws = torch.zeros(workspace_bytes(m, n, k, 4), dtype=torch.uint8, device=dev)

    def lin(cp):
        return lambda: nvfp4_linear(x, cp[0], cp[1], cp[3], None, None, 16, terms=4, sf=cp[2], out=y, workspace=ws)

    nb = n * k // 2 + n * k // 16 + m * k * 2 + m * n * 2 + 4
    us_cold = timed(lin(copies[0]))
    us = steady([lin(cp) for cp in copies])
    out["gemm_config0"] = line(us, nb, {"mode": "steady", "tflops": round(2 * m * n * k / us / 1e6, 2),
                                        "cold_us": round(us_cold, 2), "launches": 2})
    del copies, x, y, ws

    g = torch.Generator().manual_seed(0)
    B, hq, hkv, D, page = 16, 32, 8, 128, 16
    ctx = torch.randint(512, 8193, (B,), generator=g, dtype=torch.int32)
    pages = [(int(c) + page - 1) // page for c in ctx]
    pool = sum(pages)
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    bt = torch.full((B, max(pages)), -1, dtype=torch.int32)
    o = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[o:o + pages[b]]
        o += pages[b]
    pools = []
    for _ in range(2):  # 2 x 150 MB KV pools > L2
        kc = torch.randn((pool, page, hkv, D), device=dev, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
        vc = torch.randn((pool, page, hkv, D), device=dev, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
        pools.append((kc, vc))
    q = torch.randn((B, hq, D), device=dev, dtype=torch.bfloat16)
    bt_d, ctx_d = bt.to(dev), ctx.to(dev)
    o_buf = torch.empty_like(q)
    aws = torch.empty(paged_decode_workspace_bytes(B, hq, bt.shape[1], page, D), dtype=torch.uint8, device=dev)

    def att(pl):
        return lambda: paged_decode(q, pl[0], pl[1], bt_d, ctx_d, D ** -0.5, out=o_buf, workspace=aws)

    sctx = int(ctx.sum())
    nb = 2 * sctx * hkv * D + 2 * q.numel() * 2 + 4 * pool + 4 * B
    us_cold = timed(att(pools[0]))
    us = steady([att(pl) for pl in pools] * 2)
    out["attention_config1"] = line(us, nb, {"mode": "steady", "cold_us": round(us_cold, 2), "launches": 2,
                                             "sum_ctx": sctx})
    del pools

    # config 4 shape (Qwen3-30B-A3B MoE): the experts' gate+up projection [128][1536][2048] for 16
    # tokens routed top-8 (128 rows) -- the grouped GEMM (routing + gathering quantiser + one GEMM);
    # algorithmic bytes: the touched experts' weights and scales + x + y + ids
    from adallm_b200.nvfp4_gemm import nvfp4_linear_gather
    E, hid, n_e, tokens, topk = 128, 2048, 1536, 16, 8
    mm = tokens * topk
    ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(tokens)]).flatten().to(torch.int32)
    touched = int(ids.unique().numel())
    ids = ids.to(dev)
    sets = []
    for i in range(2):  # 2 x 226 MB of expert weights > L2
        packed, scale, s2 = random_nvfp4(E * n_e, hid, 777 + i, dev)
        sets.append((packed.view(E, n_e, hid // 2), scale.view(E, n_e, hid // 16),
                     torch.full((E,), s2, dtype=torch.float32, device=dev)))
    xm = torch.randn((mm, hid), device=dev, dtype=torch.bfloat16)

    def moe(sv):
        return lambda: nvfp4_linear_gather(xm, sv[0], sv[1], sv[2], ids, 16, terms=4)

    nb = touched * (n_e * hid // 2 + n_e * hid // 16) + mm * hid * 2 + mm * n_e * 2 + 4 * mm
    us_cold = timed(moe(sets[0]))
    us = steady([moe(sv) for sv in sets] * 2)
    out["moe_grouped_config4"] = line(us, nb, {"mode": "steady", "cold_us": round(us_cold, 2), "launches": 3,
                                               "rows": mm, "experts_touched": touched})
    del sets, xm

    # prefill-size GEMM (tensor-core bound): M 8192 tokens x gate_up N 24576 K 4096, W4A4 operand
    # (terms 1); FLOPs 2MNK against spec dense FP4 (9 PFLOP/s) and 4x the measured bf16 burst
    mp, npf, kpf = 8192, 24576, 4096
    packed, scale, s2 = random_nvfp4(npf, kpf, 4711, dev)
    sfp, s2t = prepack_scales(scale, npf, kpf), torch.tensor(s2, dtype=torch.float32, device=dev)
    xp = torch.randn((mp, kpf), device=dev, dtype=torch.bfloat16)
    yp = torch.empty((mp, npf), device=dev, dtype=torch.bfloat16)
    wsp = torch.zeros(workspace_bytes(mp, npf, kpf, 1), dtype=torch.uint8, device=dev)
    pf = lambda: nvfp4_linear(xp, packed, scale, s2t, None, None, 16, terms=1, sf=sfp, out=yp, workspace=wsp)
    us = steady([pf] * 4, reps=3)
    tf = 2 * mp * npf * kpf / us / 1e6
    bf16_burst = measured_bf16()
    out["gemm_prefill_w4a4"] = {"us": round(us, 1), "tflops": round(tf, 1), "m": mp, "n": npf, "k": kpf, "terms": 1,
                                "frac_fp4_spec": round(tf / 9000.0, 4),
                                "frac_4x_bf16_measured": round(tf / (4 * bf16_burst), 4) if bf16_burst else None,
                                "mode": "steady", "launches": 2}
    # the same GEMM in the reference's W4A16 arithmetic (fp16 activations, weights widened to
    # fp16 on chip, tcgen05 kind::f16 on SM pairs): what nvfp4_linear runs from 256 tokens
    yp16 = torch.empty((mp, npf), device=dev, dtype=torch.bfloat16)
    pf16 = lambda: nvfp4_linear_w4a16(xp, packed, scale, s2t, sf=sfp, out=yp16)
    us = steady([pf16] * 4, reps=3)
    tf = 2 * mp * npf * kpf / us / 1e6
    out["gemm_prefill_w4a16"] = {"us": round(us, 1), "tflops": round(tf, 1), "m": mp, "n": npf, "k": kpf,
                                 "frac_bf16_measured": round(tf / bf16_burst, 4) if bf16_burst else None,
                                 "mode": "steady", "launches": 2}
    del xp, yp, yp16, wsp, packed, scale, flush
    torch.cuda.empty_cache()

    # prefix-cache prefill attention on the e4m3 pages (Qwen3-8B heads): 4 sequences with 2048
    # cached tokens and 2048 new ones; FLOPs = 4 * D * (visible keys summed over query rows and
    # heads), the causal half of the new block included, masked work not counted
    from adallm_b200.attention import paged_prefill
    nseq, cached, new = 4, 2048, 2048
    lk = cached + new
    npg = lk // page
    bt_p = torch.arange(nseq * npg, dtype=torch.int32).view(nseq, npg)
    bt_p = bt_p.flatten()[torch.randperm(nseq * npg, generator=g)].view(nseq, npg).to(dev)
    kc = torch.randn((nseq * npg, page, hkv, D), device=dev, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    vc = torch.randn((nseq * npg, page, hkv, D), device=dev, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    qp = torch.randn((nseq * new, hq, D), device=dev, dtype=torch.bfloat16)
    op = torch.empty_like(qp)
    cu_q = torch.arange(0, (nseq + 1) * new, new, dtype=torch.int32, device=dev)
    cu_k = torch.arange(0, (nseq + 1) * lk, lk, dtype=torch.int32, device=dev)
    pa = lambda: paged_prefill(qp, kc, vc, bt_p, cu_q, cu_k, new, D ** -0.5, out=op)
    us = steady([pa] * 4, reps=3)
    vis = nseq * hq * (cached * new + new * (new + 1) // 2)
    tf = 4 * D * vis / us / 1e6
    bf16_burst = measured_bf16()
    out["prefill_attention_fp8"] = {"us": round(us, 1), "tflops": round(tf, 1), "seqs": nseq, "cached": cached,
                                    "new": new, "heads": [hq, hkv], "page": page,
                                    "frac_bf16_measured": round(tf / bf16_burst, 4) if bf16_burst else None,
                                    "mode": "steady", "launches": 1}
    del kc, vc, qp, op
    torch.cuda.empty_cache()
    return out


def _graph_steps(eng, sess, steps, warmup, prompt, toks):
    """Device-resident graph steps (forward + on-device advance) after `prompt` + `warmup`
    untimed ones; (ms per timed step, context lengths when timing starts)."""
    import torch
    gr = eng.capture(with_advance=True)
    sess.prepare(toks)
    sess.upload()
    for _ in range(prompt + warmup):
        gr.replay()
    torch.cuda.synchronize()
    ctx_start = sess.lens + prompt + warmup + 1
    st = torch.cuda.current_stream(eng.device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        gr.replay()
    e1.record(st)
    e1.synchronize()
    eng.check_errors()
    del gr
    return e0.elapsed_time(e1) / steps, ctx_start


def gemma3_bench(dev, peak, steps=32, warmup=3):
    """the Gemma3-27B-shape decode step (62 layers, hidden 5376, 32/16 heads,
    GeGLU 21504, vocab 262208 tied lm_head, 5:1 local/global with window 1024) at batch 4 on
    sequences whose FP8 paged caches already hold U[4096, 16384] tokens (random e4m3), after a
    16-token prompt; device-resident graph steps, CUDA events.  Algorithmic bytes per step: NVFP4
    weights + e4m3 scales of every layer, the bf16 lm_head, and the K/V bytes the attention reads
    (all cached tokens on global layers, the last 1024 on local ones)."""
    import torch
    from adallm_b200.decode_step import DecodeSession
    from adallm_b200.gemma3_step import Gemma3Config, Gemma3DecodeEngine
    cfg = Gemma3Config()
    B, prompt = 4, 16
    g = torch.Generator().manual_seed(0)
    ctx0 = torch.randint(4096, 16385, (B,), generator=g)
    eng = Gemma3DecodeEngine(cfg, dev, B, max_ctx=int(ctx0.max()) + prompt + warmup + steps + 8, seed=0)
    kv = eng.kv_cache.view(torch.uint8)
    for li in range(cfg.num_layers):  # finite random e4m3 bytes (magnitude codes < 0x7e, random sign)
        blk = kv[:, li]
        blk.copy_(torch.randint(0, 0x7e, blk.shape, device=dev, dtype=torch.int16).to(torch.uint8)
                  | (torch.randint(0, 2, blk.shape, device=dev, dtype=torch.int16).to(torch.uint8) << 7))
    sess = DecodeSession(eng, seed=0)
    sess.lens[:] = ctx0
    ms, ctx_start = _graph_steps(eng, sess, steps, warmup, prompt, torch.randint(0, cfg.vocab, (B,), generator=g))
    w_bytes = sum(w.n * w.k // 2 + w.n * w.k // 16 for L in eng.layers for w in (L["qkv"], L["o"], L["gate_up"],
                                                                                 L["down"]))
    head = cfg.vocab * cfg.hidden * 2
    per_tok = 2 * cfg.num_kv_heads * cfg.head_dim
    ctx_mid = (ctx_start + steps // 2).double()
    kv_bytes = sum(float((ctx_mid if not cfg.is_sliding(li) else ctx_mid.clamp(max=cfg.sliding_window)).sum())
                   * per_tok for li in range(cfg.num_layers))
    nb = w_bytes + head + kv_bytes
    out = {"tok_s": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 4), "layers": cfg.num_layers, "batch": B,
           "ctx_start": [int(c) for c in ctx_start], "window": cfg.sliding_window, "alg_bytes_per_step": int(nb),
           "gbs": round(nb / ms / 1e6, 1), "frac": round(nb / ms / 1e6 / peak, 4),
           "launches_per_step": eng.kernels_per_step(), "mode": "device-resident graph steps"}
    del eng, sess, kv
    torch.cuda.empty_cache()
    return out


def moe_bench(dev, peak, steps=32, warmup=3):
    """the Qwen3-30B-A3B-shape MoE decode step (48 layers, hidden 2048, 32/4
    heads, 128 experts top-8 of intermediate 768, vocab 151936) at batch 16 after a 16-token
    prompt, TP = 1; device-resident graph steps, CUDA events.  Algorithmic bytes per step: the
    attention NVFP4 weights + scales, every expert touched in the step (counted from the routing
    of one timed step, the same in every layer's estimate) x its gate, up and down weights +
    scales, the bf16 router and lm_head, the K/V read."""
    import torch
    from adallm_b200.decode_step import DecodeSession
    from adallm_b200.moe_step import MoEConfig, Qwen3MoeDecodeEngine
    cfg = MoEConfig()
    B, prompt = 16, 16
    g = torch.Generator().manual_seed(0)
    eng = Qwen3MoeDecodeEngine(cfg, dev, B, max_ctx=prompt + warmup + steps + 8, seed=0)
    sess = DecodeSession(eng, seed=0)
    ms, ctx_start = _graph_steps(eng, sess, steps, warmup, prompt, torch.randint(0, cfg.vocab, (B,), generator=g))
    touched = int(eng.route_ids.unique().numel())  # the last layer's routing of the last step
    ex = eng.layers[0]["experts_gate_up"], eng.layers[0]["experts_down"]
    per_expert = sum(w.n * w.k // 2 + w.n * w.k // 16 for w in ex)
    attn = sum(w.n * w.k // 2 + w.n * w.k // 16 for w in (eng.layers[0]["qkv"], eng.layers[0]["o"]))
    kv = 2 * cfg.num_kv_heads * cfg.head_dim * float((ctx_start + steps // 2).sum())
    nb = cfg.num_layers * (attn + touched * per_expert + cfg.num_experts * cfg.hidden * 2 + kv) \
        + cfg.vocab * cfg.hidden * 2
    out = {"tok_s": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 4), "layers": cfg.num_layers, "batch": B,
           "experts_touched_per_layer": touched, "alg_bytes_per_step": int(nb), "gbs": round(nb / ms / 1e6, 1),
           "frac": round(nb / ms / 1e6 / peak, 4), "launches_per_step": eng.kernels_per_step(),
           "mode": "device-resident graph steps, TP 1"}
    del eng, sess
    torch.cuda.empty_cache()
    return out


def dropin_bench(layers=36, batch=16, ctx=64):
    """The reference runtime's own decode graph (its Qwen3ForCausalLM, KV allocation and graph
    capture) with this package installed, in a child process (tests/dropin_harness.py)."""
    import subprocess
    r = subprocess.run([sys.executable, "-m", "tests.dropin_harness", "bench", "--layers", str(layers), "--batch",
                        str(batch), "--ctx", str(ctx), "--reps", "20"], cwd=ROOT, capture_output=True, text=True,
                       timeout=900)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("DROPIN ")]
    if r.returncode != 0 or not lines:
        return {"error": (r.stderr or r.stdout)[-400:]}
    out = json.loads(lines[-1][len("DROPIN "):])
    out["what"] = ("reference Qwen3ForCausalLM + ModelRunner.capture_cudagraph/run_model with adallm_b200.install() "
                   "(decode layers as nine fused kernels on the reference's parameters, KV cache and context; "
                   "page 256); run_model_ms includes the eager lm_head and static-buffer copies")
    return out


def run_reference(args, rank):
    """The reference's own CPU decode path on the host cores (rank 0 only; other ranks exit):
    W warm-up steps, then K timed full decode steps, wall time per step."""
    if rank != 0:
        return
    ref = CpuReference(args)
    for _ in range(args.warmup):
        ref.step()
    ts = [ref.step() for _ in range(args.steps)]
    total = sum(ts)
    value = args.batch * args.steps / total
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 (dequantised NVFP4 weights)", "data": "synthetic",
            "impl": "reference",
            "config": bench_config(args, args.gpus),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": ref.threads, "kind": ref.kind,
                             "sample": ref.sample(args.steps, args.warmup)},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from adallm_b200 import _native as N
    from adallm_b200.decode_step import DecodeConfig, Qwen3DecodeEngine, DecodeSession

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    group = dist.group.WORLD if world > 1 else None
    cfg = DecodeConfig(num_layers=args.layers, terms=args.terms, tp_size=world, tp_rank=rank)
    B = args.batch
    total_steps = args.prompt + 2 * (args.warmup + args.steps) + 8
    engine = Qwen3DecodeEngine(cfg, dev, B, max_ctx=total_steps + 16, seed=0, group=group)
    sess = DecodeSession(engine, seed=0)
    g_plain = engine.capture(with_advance=False)
    g_adv = engine.capture(with_advance=True)

    # prompt (16 random ids per sequence) fed through the decode step token by token
    gen = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (B, args.prompt), generator=gen)
    toks = None
    for i in range(args.prompt):
        sess.prepare(prompt[:, i])
        sess.upload()
        g_plain.replay()
        toks = sess.download()
        sess.commit()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(ms: float) -> float:
        if world == 1:
            return ms
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)
    # ---------------- value: device-resident step loop (graph = forward + on-device advance)
    sess.prepare(toks)
    sess.upload()
    for _ in range(args.warmup):
        g_adv.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            g_adv.replay()
        e1.record(stream)
        e1.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = B * args.steps / (ms / 1e3)
    engine.check_errors()  # a failed bounded wait anywhere in the timed steps voids them
    # sync host bookkeeping with the device-side advance (warmup + steps tokens were generated)
    sess.lens += args.warmup + args.steps
    toks = engine.input_ids.cpu()

    # ---------------- e2e: host-fed steps through the session: every step fills the pinned
    # inputs on the host, replays one graph (H2D copies of the inputs, forward, D2H copy of the
    # tokens) and waits for the tokens
    g_step = sess.capture_step()
    for _ in range(args.warmup):
        toks = sess.step(toks)
        sess.commit()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        toks = sess.step(toks)
        sess.commit()
    f1.record(stream)
    f1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1))
    e2e = B * args.steps / (e2e_ms / 1e3)

    # ---------------- roofline of the dominant kernel: the NVFP4 tensor-core GEMM, timed alone over
    # every projection of every layer (cold weights: 36 layers x 108 MB >> L2)
    m = B
    bn = N.lib().ada_nvfp4_block_n(m, cfg.terms)
    lin = [(L[name]) for L in engine.layers for name in ("qkv", "o", "gate_up", "down")]
    kmax = max(w.k for w in lin)
    xq = torch.zeros(cfg.terms * bn * kmax // 2, dtype=torch.uint8, device=dev)
    sfx = torch.zeros((kmax // 64) * 512, dtype=torch.uint8, device=dev)
    gx = torch.zeros(bn, dtype=torch.float32, device=dev)
    xin = torch.randn((m, kmax), device=dev, dtype=torch.bfloat16)
    ys = {w.n: torch.empty((m, w.n), device=dev, dtype=torch.bfloat16) for w in lin}
    wsb = max(int(N.lib().ada_nvfp4_gemm_workspace_size(m, w.n, w.k, cfg.terms)) for w in lin)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
    sp = stream.cuda_stream
    quant = {}
    for kk in sorted({w.k for w in lin}):
        N.check(N.lib().ada_nvfp4_act_quant(xin.data_ptr(), 0, kmax, m, kk, cfg.terms, bn, xq.data_ptr(),
                                            sfx.data_ptr(), gx.data_ptr(), sp), "act_quant")
        quant[kk] = (xq.clone(), sfx.clone(), gx.clone())

    # the GEMM exactly as the decode step runs it: split-K partial planes when the engine uses
    # them (TP1), else the reduced bf16 output
    part_buf = torch.empty(max(8 * m * w.n for w in lin), dtype=torch.float32, device=dev)

    def gemm_launch(w):
        a, b, c_ = quant[w.k]
        st = torch.cuda.current_stream(dev).cuda_stream
        if engine.use_parts:
            ns = int(N.lib().ada_nvfp4_gemm_splits(m, w.n, w.k, cfg.terms))
            N.check(N.lib().ada_nvfp4_gemm_partials(a.data_ptr(), b.data_ptr(), c_.data_ptr(), m, cfg.terms, bn,
                                                    w.packed.data_ptr(), w.packed.stride(0), w.sf.data_ptr(),
                                                    w.scale_2.data_ptr(), w.n, w.k, part_buf.data_ptr(), w.n,
                                                    m * w.n, ns, ws.data_ptr(), ws.numel(), st), "gemm")
        else:
            N.check(N.lib().ada_nvfp4_gemm(a.data_ptr(), b.data_ptr(), c_.data_ptr(), m, cfg.terms, bn,
                                           w.packed.data_ptr(), w.packed.stride(0), w.sf.data_ptr(),
                                           w.scale_2.data_ptr(), w.n, w.k, None, ys[w.n].data_ptr(), 0, w.n, 0,
                                           ws.data_ptr(), ws.numel(), st), "gemm")

    def graph_of(ws_list):
        """GEMM launches captured once, so the timing has no host launch overhead."""
        for w in ws_list:  # eager warm-up (kernel attributes)
            gemm_launch(w)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for w in ws_list:
                gemm_launch(w)
        return gr

    def time_graph(gr, reps):
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(reps):
            gr.replay()
        t1.record(stream)
        t1.synchronize()
        return t0.elapsed_time(t1)

    reps = 3
    g_all = graph_of(lin)
    launches = reps * len(lin)
    gemm_ms = time_graph(g_all, reps) / launches
    per_shape = {}
    for name in ("qkv", "o", "gate_up", "down"):
        ws_ = [L[name] for L in engine.layers]
        w0 = ws_[0]
        gr = graph_of(ws_)
        us = time_graph(gr, reps) / (reps * len(ws_)) * 1e3
        nb = w0.n * w0.k // 2 + w0.n * w0.k // 16 + m * w0.k * 2 + m * w0.n * 2
        per_shape[name] = {"n": w0.n, "k": w0.k, "us": round(us, 2), "gbs": round(nb / us / 1e3, 1)}
        del gr
    del g_all
    alg_bytes = sum(w.n * w.k // 2 + w.n * w.k // 16 + m * w.k * 2 + m * w.n * 2 for w in lin) / len(lin)
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (gemm_ms / 1e3) / 1e9
    traffic = int(GEMM_DRAM_PER_ALG_BYTE * alg_bytes)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_kind,
                "kernel": "adallm_b200 nvfp4 gemm_kernel (tcgen05 mxf4nvf4)" +
                          (", split-K partial planes as in the step" if engine.use_parts else ""),
                "alg_bytes_per_launch": int(alg_bytes), "us_per_launch": round(gemm_ms * 1e3, 3),
                "launch_mix": "qkv/o/gate_up/down of all layers, batch 16", "per_shape": per_shape}

    kernels = kernel_benches(dev, peak) if rank == 0 and world == 1 and not args.no_kernels else None
    if kernels is not None and args.layers == 36 and B == 16:
        for name, fn in (("gemma3_config2", gemma3_bench), ("moe_config4", moe_bench)):
            try:
                kernels[name] = fn(dev, peak)
            except Exception as exc:  # recorded; the headline line still prints
                kernels[name] = {"error": f"{type(exc).__name__}: {exc}"[:400]}
        kernels["dropin_decode_step"] = dropin_bench(batch=B, ctx=seq_len(args))

    ctx_end = int(sess.lens.max().item())
    assert ctx_end == seq_len(args), (ctx_end, seq_len(args))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args)

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4", "data": "synthetic",
                "config": bench_config(args, world),
                "roofline": roofline,
                "kernels": kernels,
                "cpu_baseline": cpu,
                "e2e": {"value": round(e2e, 2), "unit": "tok/s",
                        "h2d_bytes_per_step": sess.H2D_BYTES_PER_STEP, "d2h_bytes_per_step": sess.D2H_BYTES_PER_STEP,
                        "ms_per_step": round(e2e_ms / args.steps, 4)},
                "gpu_launches": engine.kernels_per_step() * args.steps,
                "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    del g_plain, g_adv, g_step  # graphs holding NCCL work go before the process group
    sess._step_graph = None
    engine.close()  # peer mappings (TP) are released by every rank before the group goes


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world != 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import torch.distributed as dist
    if world > 1:
        import torch
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
