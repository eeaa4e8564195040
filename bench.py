#!/usr/bin/env python
"""Benchmark: fused SunShape decode attention (batched GQA decode, 16 x 8192 tokens).

Workload (per GPU): batch 16, 32 query heads / 8 kv heads, head_dim 128,
T_kv = 8192 cached tokens per sequence; keys 1-bit SunShape block-VQ
(block_dim 8, 256 centroids, 16 B/token/kv-head) from a codec fit on 4096
anisotropic keys + 2048 queries; fp16 values; one new query token per step.
Synthetic seeded data. Multi-GPU: one process per GPU (torchrun), each rank
owns its own 16-sequence shard of a global batch of 16*N (weak scaling, no
collective on the data path).

  value : device throughput of the fused kernel with everything resident,
          queries/s summed over ranks (max-over-ranks step time).
  e2e   : the same metric through the public API per step with page-locked
          host buffers: one host->device copy of the step's query and new K/V
          token, cache.append (deferred: the next sunshape_sdpa's table launch
          quantizes and stores the token), sunshape_sdpa writing its output
          into page-locked host memory (the device->host transfer).

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

python bench.py --config 3 | 5 times the other two decode configurations
(config 3: B=64, T_kv=32768, 2-bit TurboQuant-style values with fp16 per-group
scales; config 5: B=1, 64q/8kv, T_kv=524288 mixed-precision keys, split-KV
across the torchrun ranks with an NCCL all-gather + log-sum-exp merge).

python bench.py --assign [--assign-path tensor|simt] prints a second kind of
line: the config-2 cache fill (16 x 8 x 8192 fp16 keys through codec.quantize's
nearest-centroid assignment, ss_vq_assign), token-heads/s, with the oracle's
CPU quantize beside it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, HQ, HKV, D, T, BD, KC = 16, 32, 8, 128, 8192, 8, 256
NB = D // BD
BYTES_PER_TOKEN_HEAD = NB + 2 * D  # 16 B indices + 256 B fp16 values
METRIC = "fused decode-attn queries/s"
WORKLOAD = ("cfg2: batched GQA decode, B=16/GPU, 32q/8kv heads, head_dim 128, T_kv 8192, "
            "SunShape 1-bit keys (bd 8, 256 centroids) + fp16 values, 1 query token/step")


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic():
    """DRAM bytes per launch of the decode kernel from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "decode_attn_cfg2_traffic.json")) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except Exception:
        return None


def _channel_sigma(seed=1):
    return np.exp(np.random.default_rng(seed).normal(0.0, 0.5, size=D)).astype(np.float32)


def _calibration():
    """2048 calibration queries and 4096 keys, anisotropic N(0, sigma_d^2)."""
    sig = _channel_sigma()
    rng = np.random.default_rng(3)
    q = (rng.standard_normal((2048, D)).astype(np.float32) * sig).astype(np.float16)
    k = (rng.standard_normal((4096, D)).astype(np.float32) * sig).astype(np.float16)
    return q, k, sig


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle sampling (200 ms) while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.gpu_id = gpu_id
        self.proc = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "200"]
        if self.gpu_id is not None:
            cmd += ["-i", self.gpu_id]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _gpu_id(dev_index: int) -> str | None:
    import torch

    try:
        u = str(torch.cuda.get_device_properties(dev_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


# ---------------------------------------------------------------------- workload
def build_workload(rank: int, device):
    import torch
    import sunshape_mlx_b200 as ss

    qc, kc, sig = _calibration()
    codec = ss.SunShapeBlockCodec(head_dim=D, block_dim=BD, n_centroids=KC, device=device)
    codec.fit(qc, kc, kmeans_iters=25, seed=0)
    cache = ss.create_kv_cache(codec, n_kv_heads=HKV)
    g = torch.Generator(device=device)
    sig_t = torch.tensor(sig, device=device)
    for b in range(B):  # per sequence to bound temporaries
        g.manual_seed(1000 * rank + b)
        k = (torch.randn((1, HKV, T, D), generator=g, device=device) * sig_t).half()
        v = torch.randn((1, HKV, T, D), generator=g, device=device).half()
        if b == 0:
            keys = torch.empty((B, HKV, T, D), dtype=torch.float16, device=device)
            vals = torch.empty_like(keys)
        keys[b:b + 1] = k
        vals[b:b + 1] = v
    cache.append(keys, vals)
    del keys, vals
    g.manual_seed(777 + rank)
    q = torch.randn((B, HQ, 1, D), generator=g, device=device).half()
    return codec, cache, q


def cpu_baseline(codec, cache, q, budget_s: float = 8.0):
    """Oracle (NumPy restatement of the reference's CPU path) on a bounded
    sample: batch row 0 (8 kv-heads x 4 q-heads x 8192 tokens) repeated."""
    import oracle as O

    st = codec.state_dict()
    state = {"mode": "profileperm_baseline", "head_dim": D, "block_dim": BD, "n_blocks": NB,
             "n_centroids": KC, "centroids": st["centroids"].numpy(),
             "permutation": st["permutation"].numpy(), "heavy": np.zeros(NB, bool)}
    idx = cache.key_indices[:1].cpu().numpy()
    vals = cache.values[:1].cpu().numpy()
    qn = q[:1].cpu().numpy()
    O.sdpa(qn, state, idx, vals, 1 / math.sqrt(D))  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        O.sdpa(qn, state, idx, vals, 1 / math.sqrt(D))
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": HQ * n / dt, "unit": "queries/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} x decode of batch row 0 ({HQ} queries over {HKV} kv-heads x {T} tokens), "
                      "oracle NumPy 2-pass path, all host cores"}


# ---------------------------------------------------------------------- our arm
def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from sunshape_mlx_b200.attention import PreparedDecode
    import sunshape_mlx_b200 as ss

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    codec, cache, q = build_workload(rank, device)
    scale = 1 / math.sqrt(D)
    prep = PreparedDecode(q, cache, scale)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        prep.run()
    # clock soak: keep the kernel running ~1.5 s so clocks settle, sampled
    # together with the timed region
    sampler = ClockSampler(_gpu_id(local))
    sampler.start()
    t_end = time.perf_counter() + 1.5
    while time.perf_counter() < t_end:
        for _ in range(200):
            prep.run()
        torch.cuda.synchronize()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        prep.run()
    e1.record(st)
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t)

    # ---- e2e through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # one page-locked host buffer holding each step's query and new K/V
        # token, and a page-locked output
        g = torch.Generator().manual_seed(99 + rank)
        nq, nkv = q.numel(), B * HKV * D
        hin = torch.empty(nq + 2 * nkv, dtype=torch.float16).pin_memory()
        hin[:nq] = q.cpu().reshape(-1)
        hin[nq:] = torch.randn(2 * nkv, generator=g).half()
        qh, kh, vh = hin[:nq], hin[nq:nq + nkv], hin[nq + nkv:]
        oh = torch.empty((B, HQ, 1, D), dtype=torch.float16).pin_memory()
        din = torch.empty(hin.numel(), dtype=torch.float16, device=device)
        qd = din[:nq].view(B, HQ, 1, D)
        kd = din[nq:nq + nkv].view(B, HKV, 1, D)
        vd = din[nq + nkv:].view(B, HKV, 1, D)

        # One copy brings the step's query and new K/V token to the device;
        # the append is deferred into the attention's table launch, and the
        # decode kernel writes the output straight into the page-locked host
        # buffer (out=), so no separate device-to-host copy follows it.
        # (Measured alternatives: the query copied on a side stream beside the
        # token's copy, and the output copied back after the kernel, were
        # slower: 93 and 87 against 84 us per step before the append fix.)
        def e2e_step():
            din.copy_(hin, non_blocking=True)
            cache.append(kd, vd)
            ss.sunshape_sdpa(qd, cache, scale, out=oh)
            cache.trim(1)

        for _ in range(max(3, args.warmup)):
            e2e_step()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(st)
        for _ in range(args.steps):
            e2e_step()
        f1.record(st)
        barrier()
        ems = f0.elapsed_time(f1) / args.steps
        et = torch.tensor([ems], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        ems = float(et)
        e2e = {"value": world * B * HQ / (ems / 1e3), "unit": "queries/s",
               "h2d_bytes_per_step": qh.numel() * 2 + kh.numel() * 2 + vh.numel() * 2,
               "d2h_bytes_per_step": oh.numel() * 2, "ms_per_step": ems,
               "gpu_launches_per_step": 2}  # table kernel (with the fused append) + decode

    if rank != 0:
        return None
    peak, peak_kind = _peaks()
    alg_bytes = B * HKV * T * BYTES_PER_TOKEN_HEAD + 2 * B * HQ * D * 2
    achieved = alg_bytes / (ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": world * B * HQ / (ms / 1e3), "unit": "queries/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded anisotropic keys, N(0,1) fp16 values/queries)",
        "config": {"workload": WORKLOAD, "global_batch": B * world, "seq_len": T,
                   "parallelism": f"dp{world} (batch shards, no collective)",
                   "l2": "inputs larger than L2 (285 MB streamed per step vs 126 MB L2)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "frac_of_8TBs_nominal": achieved / 8000.0,
                     "traffic": _traffic(), "algorithmic_bytes_per_launch": alg_bytes},
        "gpu_launches": 2 * args.steps,  # table kernel + decode kernel per step
        "clocks": clocks,
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(codec, cache, q)
    return line


# ---------------------------------------------------------------------- configs 3 and 5
CFG3 = dict(B=64, HQ=32, HKV=8, T=32768, bytes_per_th=NB + 32 + 8,
            workload="cfg3: hybrid-cache decode, B=64/GPU, 32q/8kv heads, head_dim 128, T_kv 32768, "
                     "SunShape 1-bit keys + 2-bit TurboQuant-style values (rotated, Lloyd-Max levels, "
                     "fp16 scale per 32 channels), buffer_size 0, 1 query token/step")
CFG5 = dict(B=1, HQ=64, HKV=8, T=524288, bytes_per_th=12 + 4 * BD * 2 + 2 * D,
            workload="cfg5: long-context decode, B=1, 64q/8kv heads, head_dim 128, T_kv 524288, "
                     "profileperm_mixed_precision keys (4 of 16 blocks fp16, 12 VQ'd), fp16 values, "
                     "prefill-quantised in 32768-token chunks, T_kv split across ranks")


def _build_cfg3(device):
    import torch
    import sunshape_mlx_b200 as ss

    c = CFG3
    qc, kc, sig = _calibration()
    codec = ss.SunShapeBlockCodec(head_dim=D, block_dim=BD, n_centroids=KC, device=device)
    codec.fit(qc, kc, kmeans_iters=25, seed=0)
    cache = ss.create_kv_cache(codec, n_kv_heads=c["HKV"], value_backend="turboquant",
                               value_bits=2, tq_group_size=32, buffer_size=0)
    g = torch.Generator(device=device).manual_seed(31)
    sig_t = torch.tensor(sig, device=device)
    for _ in range(c["T"] // 2048):
        k = (torch.randn((c["B"], c["HKV"], 2048, D), generator=g, device=device) * sig_t).half()
        v = torch.randn((c["B"], c["HKV"], 2048, D), generator=g, device=device).half()
        cache.append(k, v)
    del k, v
    q = torch.randn((c["B"], c["HQ"], 1, D), generator=g, device=device).half()
    return codec, cache, q


def _build_cfg5(device, rank, world):
    """This rank's contiguous token range of the config-5 sequence."""
    import torch
    import sunshape_mlx_b200 as ss
    from sunshape_mlx_b200 import splitkv

    c = CFG5
    qc, kc, sig = _calibration()
    codec = ss.SunShapeBlockCodec(head_dim=D, block_dim=BD, n_centroids=KC, device=device,
                                  mode="profileperm_mixed_precision", n_heavy=4)
    codec.fit(qc, kc, kmeans_iters=25, seed=0)
    cache = ss.create_kv_cache(codec, n_kv_heads=c["HKV"])
    lo, hi = splitkv.shard_range(c["T"], rank, world)
    sig_t = torch.tensor(sig, device=device)
    chunk = 32768
    for a in range(0, c["T"], chunk):  # the same sequence on every rank; keep this shard
        if a + chunk <= lo or a >= hi:
            continue
        g = torch.Generator(device=device).manual_seed(5000 + a // chunk)
        k = (torch.randn((1, c["HKV"], chunk, D), generator=g, device=device) * sig_t).half()
        v = torch.randn((1, c["HKV"], chunk, D), generator=g, device=device).half()
        s0, s1 = max(lo, a) - a, min(hi, a + chunk) - a
        cache.append(k[:, :, s0:s1].contiguous(), v[:, :, s0:s1].contiguous())
    g = torch.Generator(device=device).manual_seed(777)
    q = torch.randn((1, c["HQ"], 1, D), generator=g, device=device).half()
    return codec, cache, q

CFG4 = dict(B=32, HQ=32, HKV=8, T=4096, LAYERS=32, bytes_per_th=32 + 32,
            workload="cfg4 attention: 32 layers of decode attention, B=32/GPU, 32q/8kv heads, "
                     "head_dim 128, T_kv 4096, block-VQ keys AND values (block_dim 4, 256 centroids, "
                     "32 blocks; value_backend 'sunshape'), buffer_size 0, 1 query token/step/layer")


def _build_cfg4(device):
    """32 layers of (B, 8, 4096) caches with block-VQ keys and values. One key
    codec and one value codec (fit once) serve every layer; each layer holds
    its own seeded tokens."""
    import torch
    import sunshape_mlx_b200 as ss

    c = CFG4
    qc, kc, sig = _calibration()
    kcodec = ss.SunShapeBlockCodec(head_dim=D, block_dim=4, n_centroids=KC, device=device)
    kcodec.fit(qc, kc, kmeans_iters=25, seed=0)
    rng = np.random.default_rng(44)
    vcal = rng.standard_normal((4096, D)).astype(np.float16)
    vcodec = ss.SunShapeBlockCodec(head_dim=D, block_dim=4, n_centroids=KC, device=device)
    vcodec.fit(qc, vcal, kmeans_iters=25, seed=1)
    sig_t = torch.tensor(sig, device=device)
    caches = []
    for layer in range(c["LAYERS"]):
        cache = ss.create_kv_cache(kcodec, n_kv_heads=c["HKV"], value_backend="sunshape",
                                   value_bits=8, value_codec=vcodec, buffer_size=0)
        g = torch.Generator(device=device).manual_seed(4000 + layer)
        k = (torch.randn((c["B"], c["HKV"], c["T"], D), generator=g, device=device) * sig_t).half()
        v = torch.randn((c["B"], c["HKV"], c["T"], D), generator=g, device=device).half()
        cache.append(k, v)
        caches.append(cache)
    del k, v
    g = torch.Generator(device=device).manual_seed(4999)
    q = torch.randn((c["B"], c["HQ"], 1, D), generator=g, device=device).half()
    return kcodec, caches, q


def run_model(args, rank, local):
    """Config 4 end to end: random-init Llama-style decoder (32 layers, 4096
    hidden, 32q/8kv, FFN 14336, RoPE 1e6, bf16), per-layer block-VQ key and
    value codecs (block_dim 4, 256 centroids) fit on the activations of a
    dense 4096-token calibration pass, batch 32 x 4096-token random prompt,
    then greedy decode steps with attention routed to sunshape_sdpa. Beside
    it, the same decode with an uncompressed bf16 KV cache and torch's dense
    SDPA (a library baseline)."""
    import torch
    from sunshape_mlx_b200 import harness as Hm, patch

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = Hm.DecoderConfig()
    model = Hm.Decoder(cfg, device=device, seed=7)
    g = torch.Generator(device=device).manual_seed(8)
    calib = torch.randint(0, cfg.vocab, (1, 4096), generator=g, device=device)
    t0 = time.perf_counter()
    codecs = Hm.fit_layer_codecs(model, calib)
    fit_s = time.perf_counter() - t0
    B, T = 32, 4096
    prompt = torch.randint(0, cfg.vocab, (B, T), generator=g, device=device)
    steps = min(args.steps, 256)
    warm = max(3, args.warmup)

    def decode(caches, pos, ids, n):
        for i in range(n):
            logits = model.forward(ids, caches, pos + i)
            ids = logits.argmax(-1, keepdim=True)
        return ids

    patch.apply()
    caches = Hm.make_caches(model, codecs)
    ids = model.forward(prompt, caches, 0).argmax(-1, keepdim=True)
    ids = decode(caches, T, ids, warm)
    torch.cuda.synchronize()
    sampler = ClockSampler(_gpu_id(local))
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    decode(caches, T + warm, ids, steps)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / steps
    kv_bytes = sum(c.nbytes for c in caches)
    del caches
    torch.cuda.empty_cache()

    # the same decode over an uncompressed bf16 cache (torch SDPA)
    class DenseCache:
        def __init__(self, cap):
            self.k = torch.empty((B, cfg.n_kv_heads, cap, cfg.head_dim), dtype=torch.bfloat16, device=device)
            self.v = torch.empty_like(self.k)
            self.n = 0

        def append(self, k, v):
            t = k.shape[2]
            self.k[:, :, self.n:self.n + t] = k
            self.v[:, :, self.n:self.n + t] = v
            self.n += t

    def dense_sdpa(q, k, v, cache, scale, mask, sinks=None):
        return torch.nn.functional.scaled_dot_product_attention(
            q, cache.k[:, :, :cache.n], cache.v[:, :, :cache.n], scale=scale, enable_gqa=True)

    patch.revert()
    dcaches = [DenseCache(T + warm + steps + 8) for _ in range(cfg.n_layers)]
    orig = patch.current_sdpa
    patch.current_sdpa = lambda: dense_sdpa
    try:
        ids = model.forward(prompt, dcaches, 0).argmax(-1, keepdim=True)
        ids = decode(dcaches, T, ids, warm)
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        decode(dcaches, T + warm, ids, steps)
        f1.record()
        torch.cuda.synchronize()
        dms = f0.elapsed_time(f1) / steps
    finally:
        patch.current_sdpa = orig
    dense_bytes = 2 * cfg.n_layers * B * cfg.n_kv_heads * (T + warm + steps) * cfg.head_dim * 2
    return {
        "metric": "end-to-end decode tokens/s (config 4)", "value": B / (ms / 1e3), "unit": "tokens/s",
        "n_gpus": 1, "steps": steps, "warmup": warm, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02) seed 7, random prompt ids seed 8)",
        "config": {"workload": "cfg4: Llama-style decoder 32 layers / 4096 hidden / 32q-8kv / FFN 14336, "
                               "batch 32, 4096-token prompt, greedy decode; block-VQ K and V (bd 4, 256 "
                               "centroids) per layer, attention via patch.apply() -> sunshape_sdpa",
                   "global_batch": B, "seq_len": T, "parallelism": "single GPU"},
        "kv_cache_bytes": kv_bytes, "dense_bf16_kv_cache_bytes": dense_bytes,
        "dense_bf16_kv_ms_per_step": dms, "codec_fit_s": fit_s,
        "gpu_launches": None, "clocks": clocks,
    }


def run_config(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from sunshape_mlx_b200.attention import PreparedDecode
    from sunshape_mlx_b200 import splitkv

    c = {3: CFG3, 4: CFG4, 5: CFG5}[args.config]
    if args.batch and args.config == 3:
        c["B"] = args.batch
    layers = c.get("LAYERS", 1)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    scale = 1 / math.sqrt(D)
    if args.config == 3:
        codec, cache, q = _build_cfg3(device)
    elif args.config == 4:
        codec, caches, q = _build_cfg4(device)
        cache = caches[0]
    else:
        codec, cache, q = _build_cfg5(device, rank, world)
    if args.config == 4:
        preps = [PreparedDecode(q, cl, scale) for cl in caches]

        def step():
            for pr in preps:
                pr.run()
        launches = 2 * layers
    elif world > 1 and args.config == 5:
        sk = splitkv.PreparedSplitKV(q, cache, scale)
        step = sk.run
        launches = 3  # table + decode (partials) + merge; plus the NCCL all-gather
    else:
        prep = PreparedDecode(q, cache, scale)
        step = prep.run
        launches = 2
    if args.profile:
        for _ in range(args.warmup + args.steps):
            step()
        torch.cuda.synchronize()
        print("profile run done", flush=True)
        return None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    sampler = ClockSampler(_gpu_id(local))
    sampler.start()
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t)
    phases = None
    if world > 1 and args.config == 5:
        phases = _splitkv_phases(sk, args.steps, device)
    if rank != 0:
        return None
    peak, peak_kind = _peaks()
    per_rank_tokens = c["T"] // world if args.config == 5 else c["T"]
    alg_bytes = layers * (c["B"] * c["HKV"] * per_rank_tokens * c["bytes_per_th"]
                          + 2 * c["B"] * c["HQ"] * D * 2)
    achieved = alg_bytes / (ms / 1e3) / 1e9
    weak = args.config in (3, 4)
    nq = c["B"] * c["HQ"] * layers * (world if weak else 1)
    line = {
        "metric": METRIC, "value": nq / (ms / 1e3), "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded anisotropic keys, N(0,1) fp16 values/queries)",
        "config": {"workload": c["workload"], "global_batch": c["B"] * (world if weak else 1),
                   "seq_len": c["T"], "parallelism": (f"dp{world} (batch shards)" if weak
                                                      else f"split-KV x{world} (token shards, NCCL all-gather + LSE merge)"),
                   "l2": f"inputs larger than L2 ({alg_bytes / 1e6:.0f} MB streamed per step per GPU)",
                   "queries_per_step": nq},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "frac_of_8TBs_nominal": achieved / 8000.0, "traffic": None,
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "bytes_per_token_head": c["bytes_per_th"]},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
    }
    if phases is not None:
        line["splitkv_phases_ms"] = phases
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = _cpu_baseline_cfg(args.config, codec, cache, q)
    return line


def _splitkv_phases(sk, steps, device):
    """Per-phase device time of the split-KV step (this rank's fused decode
    partials, the NCCL all-gather, the log-sum-exp merge), CUDA events around
    each phase, averaged over `steps` steps, max over ranks."""
    import torch
    import torch.distributed as dist

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    dist.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        ev[i][0].record()
        sk.run_partials()
        ev[i][1].record()
        sk.gather()
        ev[i][2].record()
        sk.merge()
        ev[i][3].record()
    torch.cuda.synchronize()
    t = torch.tensor([[e[k].elapsed_time(e[k + 1]) for k in range(3)] for e in ev],
                     dtype=torch.float64, device=device).mean(0)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {"decode_partials": float(t[0]), "all_gather": float(t[1]), "lse_merge": float(t[2])}


def _cpu_baseline_cfg(cfg, codec, cache, q, budget_s: float = 8.0):
    """Oracle CPU path on one kv-head of batch row 0 (its n_rep query heads):
    the reference dequantises the values and runs its 2-pass SDPA."""
    import oracle as O

    st = codec.state_dict()
    state = {"mode": "profileperm_baseline", "head_dim": D, "block_dim": BD, "n_blocks": NB,
             "n_centroids": KC, "centroids": st["centroids"].numpy(),
             "permutation": st["permutation"].numpy(), "heavy": np.zeros(NB, bool)}
    c = {3: CFG3, 4: CFG4, 5: CFG5}[cfg]
    state.update(block_dim=codec.block_dim, n_blocks=codec.n_blocks)
    rep = c["HQ"] // c["HKV"]
    idx = cache.key_indices[:1, :1].cpu().numpy()
    vals = cache.values[:1, :1].float().cpu().numpy()  # dequantised as the reference does
    qn = q[:1, :rep].float().cpu().numpy()
    n, t0 = 0, time.perf_counter()
    while True:
        O.sdpa(qn, state, idx, vals, 1 / math.sqrt(D))
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": rep * n / dt, "unit": "queries/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} x decode of {rep} query heads over 1 kv-head x {idx.shape[2]} tokens "
                      "(batch row 0), oracle NumPy 2-pass path on dequantised values, all host cores"}


# ---------------------------------------------------------------------- quantize (cache fill)
def _assign_workload(device):
    """cfg2 codec (fit on the CUDA-core path) and the 16 x 8 x 8192 key cache."""
    import torch
    import sunshape_mlx_b200 as ss
    from sunshape_mlx_b200 import kernels as K

    qc, kc, sig = _calibration()
    K.set_assign_path("simt")  # the fit's own launches stay out of tensor-kernel captures
    codec = ss.SunShapeBlockCodec(head_dim=D, block_dim=BD, n_centroids=KC, device=device)
    codec.fit(qc, kc, kmeans_iters=25, seed=0)
    K.set_assign_path("auto")
    g = torch.Generator(device=device).manual_seed(4242)
    keys = (torch.randn((B * HKV, T, D), generator=g, device=device)
            * torch.tensor(sig, device=device)).half()
    out = torch.empty((B * HKV, T, NB), dtype=torch.uint8, device=device)
    return codec, keys, out


def run_assign(args):
    import torch
    from sunshape_mlx_b200 import kernels as K
    import oracle as O

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    codec, keys, out = _assign_workload(device)
    perm = codec.permutation.to(device=device, dtype=torch.int32)
    cents = codec.centroids.to(device)
    K.set_assign_path(args.assign_path)

    def step():
        K.vq_assign(keys, cents, perm=perm, out_idx=out)

    for _ in range(max(3, args.warmup)):
        step()
    if args.profile:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        print("assign profile run done", flush=True)
        return None
    sampler = ClockSampler(_gpu_id(0))
    sampler.start()
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    K.assign_check(device)
    ms = e0.elapsed_time(e1) / args.steps
    n_th = B * HKV * T
    flops = 2.0 * KC * D * n_th  # ||c||^2 - 2k.c as a GEMM over all blocks
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, peak_kind = float(json.load(f)["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    except Exception:
        peak, peak_kind = 1590.0, "fallback"
    achieved = flops / (ms / 1e3) / 1e12
    # CPU baseline: the oracle's NumPy quantize (the reference's CPU loop) on 8192 rows
    st_np = {"mode": "profileperm_baseline", "head_dim": D, "block_dim": BD, "n_blocks": NB,
             "n_centroids": KC, "centroids": codec.centroids.cpu().numpy(),
             "permutation": codec.permutation.cpu().numpy(), "heavy": np.zeros(NB, bool)}
    sample = keys[0, :8192].float().cpu().numpy()
    t0 = time.perf_counter()
    O.quantize(st_np, sample)
    cpu_v = sample.shape[0] / (time.perf_counter() - t0)
    return {
        "metric": "block-VQ quantize (cache fill) token-heads/s", "value": n_th / (ms / 1e3),
        "unit": "token-heads/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 keys, fp16 hi/lo GEMM + f32 exact re-score",
        "data": "synthetic (seeded anisotropic fp16 keys)",
        "config": {"workload": "cfg2 cache fill: 16 x 8 kv-heads x 8192 tokens, head_dim 128, "
                               "bd 8, 256 centroids, ProfilePerm", "assign_path": args.assign_path,
                   "l2": "inputs larger than L2 (268 MB of keys per step vs 126 MB L2)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "note": "algorithmic 2*256*128 FLOP per token-head; the kernel is bound by "
                             "its CUDA-core epilogue (see the committed ncu summary of this kernel)"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "cpu_baseline": {"value": cpu_v, "unit": "token-heads/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": "8192 rows of head 0 through the oracle's "
                                                   "NumPy quantize (codec.py:472-514 loop)"},
    }


# ---------------------------------------------------------------------- value encode (cache fill)
def run_encode(args):
    """Value encoders on the config-3 value stream: 64 x 8 kv-heads x 8192
    fp16 tokens (1 GiB) per step, encoded into cache-layout buffers."""
    import torch
    from sunshape_mlx_b200.value_codecs import GroupedValueCodec, TurboQuantValueCodec
    import oracle as O

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    Bv, Tv = 64, 8192
    g = torch.Generator(device=device).manual_seed(41)
    v = torch.randn((Bv * HKV, Tv, D), generator=g, device=device).half()
    n_th = Bv * HKV * Tv
    fmts = {
        "tq2_g32_fp16": TurboQuantValueCodec(head_dim=D, bits=2, group_size=32, device=device),
        "tq2_reference": TurboQuantValueCodec(head_dim=D, bits=2, device=device),
        "grouped2_g64": GroupedValueCodec(head_dim=D, bits=2, group_size=64),
        "grouped4_g64": GroupedValueCodec(head_dim=D, bits=4, group_size=64),
    }
    peak, peak_kind = _peaks()
    res = {}
    for name, vc in fmts.items():
        packed = torch.empty((Bv * HKV, Tv, vc.packed_dim), dtype=torch.int32, device=device)
        if isinstance(vc, TurboQuantValueCodec):
            sc = (torch.empty((Bv * HKV, Tv), dtype=torch.float32, device=device) if vc.group_size is None
                  else torch.empty((Bv * HKV, Tv, vc.n_scale_groups), dtype=torch.float16, device=device))
            step = lambda: vc.quantize_into(v, packed, sc)
            out_b = vc.packed_dim * 4 + (4 if vc.group_size is None else 2 * vc.n_scale_groups)
        else:
            sc = torch.empty((Bv * HKV, Tv, vc.n_groups), dtype=torch.float32, device=device)
            zr = torch.empty_like(sc)
            step = lambda: vc.quantize_into(v, packed, sc, zr)
            out_b = vc.packed_dim * 4 + 8 * vc.n_groups
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        alg = n_th * (2 * D + out_b)
        res[name] = {"ms_per_step": ms, "token_heads_per_s": n_th / (ms / 1e3),
                     "bytes_per_token_head": 2 * D + out_b, "achieved_gbs": alg / (ms / 1e3) / 1e9,
                     "frac": alg / (ms / 1e3) / 1e9 / peak}
    main = res["tq2_g32_fp16"]
    # CPU baseline: the oracle's grouped TurboQuant encode on 8192 rows
    rot = fmts["tq2_g32_fp16"].rotation.cpu().numpy()
    sample = v[0].float().cpu().numpy()
    t0 = time.perf_counter()
    O.tq_group_quantize(sample, rot, 2, 32)
    cpu_v = sample.shape[0] / (time.perf_counter() - t0)
    return {
        "metric": "value encode (cache fill) token-heads/s", "value": main["token_heads_per_s"],
        "unit": "token-heads/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": main["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 in, 2-bit codes + fp16 scales out",
        "data": "synthetic (N(0,1) fp16 values)",
        "config": {"workload": "cfg3 value stream: 64 x 8 kv-heads x 8192 tokens, head_dim 128, "
                               "TurboQuant-style 2-bit, rotated, fp16 scale per 32 channels",
                   "l2": "inputs larger than L2 (1 GiB of values per step)"},
        "roofline": {"bound": "hbm", "achieved": main["achieved_gbs"], "peak": peak, "unit": "GB/s",
                     "frac": main["frac"], "peak_source": peak_kind},
        "variants": res,
        "gpu_launches": args.steps,
        "cpu_baseline": {"value": cpu_v, "unit": "token-heads/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": "8192 rows through the oracle's grouped "
                                                   "TurboQuant encode (NumPy)"},
    }


# ---------------------------------------------------------------------- reference arm
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _import_reference():
    """The unmodified reference package from baseline/_ref, with the NumPy
    stand-in for ``mlx.core`` (MLX has no Linux build here): every Metal
    wrapper then takes its own fallback, i.e. the reference's CPU path."""
    import types

    if not os.path.isdir(os.path.join(REF_DIR, "sunshape_mlx")):
        return None
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import mlx_numpy_shim

    pkg = types.ModuleType("mlx")
    pkg.core = mlx_numpy_shim
    sys.modules.setdefault("mlx", pkg)
    sys.modules.setdefault("mlx.core", mlx_numpy_shim)
    sys.path.insert(0, REF_DIR)
    import sunshape_mlx

    return sunshape_mlx


def run_reference(args):
    """The reference's own decode step on the host cores: its codec fit on
    the workload's calibration set, its SunShapeKVCache filled with one batch
    row (8 kv-heads x 8192 tokens, its NumPy quantize loop), then per step the
    mlx-lm call order -- update_and_fetch of one new token (which dequantizes
    the whole key cache, cache.py:205) and sunshape_sdpa (its per-query-head
    loop, attention.py:268-352) -- followed by trim(1) so every step sees
    8192 + 1 tokens. Beside it, the NumPy restatement of the same SDPA (the
    oracle port) on the same inputs, as cpu_baseline.port."""
    import oracle as O

    ref = _import_reference()
    qc, kc, sig = _calibration()
    rng = np.random.default_rng(12345)
    keys = (rng.standard_normal((1, HKV, T, D)).astype(np.float32) * sig).astype(np.float16)
    vals = rng.standard_normal((1, HKV, T, D)).astype(np.float16)
    q = rng.standard_normal((1, HQ, 1, D)).astype(np.float16)
    knew = (rng.standard_normal((1, HKV, 1, D)).astype(np.float32) * sig).astype(np.float16)
    vnew = rng.standard_normal((1, HKV, 1, D)).astype(np.float16)
    scale = 1 / math.sqrt(D)
    port = None
    if ref is None:
        kind, why = "port", "baseline/_ref missing: NumPy restatement of the reference's CPU path"
    else:
        from sunshape_mlx.attention import sunshape_sdpa
        from sunshape_mlx.cache import create_kv_cache
        from sunshape_mlx.codec import SunShapeBlockCodec

        codec = SunShapeBlockCodec(head_dim=D, block_dim=BD, n_centroids=KC)
        codec.fit(qc.astype(np.float32), kc.astype(np.float32), kmeans_iters=25, seed=0)
        cache = create_kv_cache(codec, n_kv_heads=HKV)
        cache.update_and_fetch(keys, vals)

        def step():
            cache.update_and_fetch(knew, vnew)
            out = sunshape_sdpa(q, cache, scale)
            cache.trim(1)
            return out
        kind, why = "reference", ("the reference package (baseline/_ref) over a NumPy stand-in for "
                                  "mlx.core: its CPU fallback paths")
    # the oracle port on the same inputs (the arm itself without baseline/_ref)
    st = O.fit(qc.astype(np.float32), kc.astype(np.float32), head_dim=D, block_dim=BD,
               n_centroids=KC, kmeans_iters=25, seed=0)
    idx = np.zeros((1, HKV, T, NB), np.uint8)
    for h in range(HKV):
        for a in range(0, T, 2048):
            idx[0, h, a:a + 2048] = O.quantize(st, keys[0, h, a:a + 2048].astype(np.float32))[0]

    def port_step():
        return O.sdpa(q, st, idx, vals, scale)
    if ref is None:
        step = port_step
    for _ in range(max(1, args.warmup)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    v = HQ / dt
    if ref is not None:
        port_step()
        n, p0 = 0, time.perf_counter()
        while n < 3 or time.perf_counter() - p0 < 5.0:
            port_step()
            n += 1
        port = {"value": HQ * n / (time.perf_counter() - p0), "unit": "queries/s",
                "cores": os.cpu_count(), "kind": "port",
                "sample": "decode of 1 batch row through the oracle's NumPy restatement"}
    line = {
        "metric": METRIC, "value": v, "unit": "queries/s", "impl": "reference", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded anisotropic keys, N(0,1) fp16 values/queries)",
        "config": {"workload": WORKLOAD, "global_batch": B, "seq_len": T,
                   "parallelism": "host CPU", "sample": "1 of 16 batch rows per step"},
        "cpu_baseline": {"value": v, "unit": "queries/s", "cores": os.cpu_count(), "kind": kind,
                         "sample": "per step: update_and_fetch of 1 token + decode of 1 batch row "
                                   "(32 queries x 8 kv-heads x 8193 tokens), " + why},
        "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if port is not None:
        line["cpu_baseline_port"] = port
    return line


_OUT = sys.stdout


def _emit(line_json: str, flush: bool = True) -> None:
    print(line_json, file=_OUT, flush=flush)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=2,
                    help="decode workload: 2 batched 8192-token decode, 3 TurboQuant-value 32768-token decode, 4 32-layer block-VQ K/V attention, 5 524288-token split-KV decode")
    ap.add_argument("--model", action="store_true",
                    help="with --config 4: the end-to-end decoder (tokens/s) instead of attention alone")
    ap.add_argument("--assign", action="store_true",
                    help="benchmark the cache-fill quantize (ss_vq_assign) instead of decode")
    ap.add_argument("--assign-path", choices=["tensor", "simt", "auto"], default="tensor")
    ap.add_argument("--encode", action="store_true",
                    help="benchmark the value encoders (config-3 value stream)")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the batch of --config 3 (smaller cases for profiling)")
    ap.add_argument("--profile", action="store_true",
                    help="build the workload, run warmup+steps decode launches, exit "
                         "(short command for ncu captures)")
    args = ap.parse_args()
    # stdout carries exactly the one JSON line: anything else a library prints
    # there (NCCL's version banner, for one) is sent to stderr
    global _OUT
    _OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            _emit(json.dumps(run_reference(args)))
        return
    import torch
    import torch.distributed as dist

    if args.encode:
        _emit(json.dumps(run_encode(args)))
        return
    if args.assign:
        line = run_assign(args)
        if line is not None:
            _emit(json.dumps(line))
        return
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    if args.config == 4 and args.model:
        line = run_model(args, rank, local)
        if line is not None:
            _emit(json.dumps(line))
        return
    if args.config != 2:
        try:
            line = run_config(args, world, rank, local)
            if line is not None:
                _emit(json.dumps(line))
        finally:
            if world > 1:
                dist.destroy_process_group()
        return
    if args.profile:
        from sunshape_mlx_b200.attention import PreparedDecode

        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        _, cache, q = build_workload(rank, dev)
        prep = PreparedDecode(q, cache, 1 / math.sqrt(D))
        for _ in range(args.warmup + args.steps):
            prep.run()
        torch.cuda.synchronize()
        print("profile run done", flush=True)
        return
    try:
        line = run_ours(args, world, rank, local)
        if line is not None:
            _emit(json.dumps(line))
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
