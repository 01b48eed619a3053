#!/usr/bin/env python
"""Benchmark of the B200 decode-attention path (one JSON line on rank 0).

Workload: block-verify attention, batch 1 per GPU,
q_len 5 (k = 4 draft tokens + 1 bonus), GQA 12:2, head_dim 128, BF16 K/V in
16-token pages with a seeded random page order, context 8192.  One step is the
verify attention of one target forward: 28 layers, each with its own paged cache
(28 x 8.4 MB = 235 MB of KV per step, larger than the 126 MB L2, so every step
reads HBM).  The step (device plan + 28 verify launches) is a CUDA graph replayed
K times; the K-step window is timed 5 times and the median window is reported.

  value     algorithmic attention bytes of all ranks / max-over-ranks device time
            (bytes per call = 1024.25 T + 6144 q for bf16 V; 776.25 T + 6144 q for E4M3 V)
  e2e       the same metric through the public API with host buffers: every layer
            copies its q and new K/V rows from pinned host memory, appends them,
            runs paged attention and copies the output back
  roofline  the verify kernel's in-step duration: a graph of the same step's 28 verify
            launches without the plan (programmatic dependent launches as in the step),
            timed with CUDA events over its replays, against MEASURED_PEAKS.json hbm_gbs
  cpu_baseline / --impl reference: the reference's eager attention formula
            (CPU oracle, torch on all host threads) on the same step (28 layer calls)
  extras    the other attention configs, the append-quantize kernel, the
            CPU timings of the FP8 quantiser and of greedy SpecDec, and SpecDec with a
            draft that always agrees with the target

Multi-GPU (torchrun): every rank runs its own batch-1 workload (weak scaling,
sequences are independent); no collective in the timed region.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "specdec-context-scaling_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "verify-attn HBM GB/s (% of 8 TB/s) at 2K–8K ctx; SpecDec decode tokens/s"
H, KV, D = 12, 2, 128
LAYERS = 28
PAGE = 16
# DRAM bytes (read + write) of one verify-kernel launch of the headline workload, from an
# `ncu --set full` capture of `bench.py --profile-case verify8k` (8,661,504 read + 0 written)
NCU_TRAFFIC_VERIFY8K = 8661504


def attn_bytes(T: int, q: int, fp8: bool, heads: int = H, d: int = D) -> float:
    pt = math.ceil(T / PAGE) * 4
    qo = 2 * heads * q * d * 2
    if fp8:
        return T * KV * d * 2 + T * KV * d + T * KV * 4 + pt + qo
    return T * KV * d * 4 + pt + qo


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampler for the timed region (200 ms period)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        time.sleep(0.05)
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[0] == str(self.idx):
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------------------ helpers
def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback (6.65 TB/s)"


def measured_bf16_peak():
    """Burst bf16 dense GEMM TFLOP/s measured on this pool (MEASURED_PEAKS.json), else the fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"])
        except (KeyError, ValueError):
            pass
    return 1590.0


def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        # NCCL prints its version to stdout when the communicator is created: send the
        # process's stdout to stderr meanwhile, so stdout carries the JSON line only
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def filled_cache(num_layers, lens, fp8, seed, d=D):
    """A paged cache of `num_layers` layers whose sequences hold `lens` seeded tokens
    (K ~ N(0,1); V ~ N(0,1), with 1 % +-8 sigma outliers for the E4M3 config)."""
    import torch

    from specdec_b200.engine.paged_cache import PagedKVCache
    from specdec_b200.kernels import ops

    cap = max(lens)
    cache = PagedKVCache.allocate(num_layers, len(lens), KV, d, cap, v_dtype="e4m3" if fp8 else "bf16",
                                  device="cuda", page_order_seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed)
    total = sum(lens)
    row0 = torch.tensor([sum(lens[:i]) for i in range(len(lens))], dtype=torch.int32, device="cuda")
    n_new = torch.tensor(lens, dtype=torch.int32, device="cuda")
    pos0 = torch.zeros(len(lens), dtype=torch.int32, device="cuda")
    for layer in range(num_layers):
        k = torch.randn(total, KV, d, generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn(total, KV, d, generator=g, device="cuda")
        if fp8:
            hit = torch.rand(v.shape, generator=g, device="cuda") < 0.01
            sgn = torch.where(torch.rand(v.shape, generator=g, device="cuda") < 0.5, -8.0, 8.0)
            v = torch.where(hit, sgn, v)
        ops.append_kv(k, v.to(torch.bfloat16), cache, layer, row0=row0, n_new=n_new, pos0=pos0, max_new=max(lens))
    cache.lengths.copy_(n_new)
    cache.host_lengths = list(lens)
    torch.cuda.synchronize()
    return cache


class GraphStep:
    """One verify/decode pass over every layer: device plan + per-layer paged attention, in a CUDA graph."""

    def __init__(self, cache, q_lens, ctx_lens, seed=0, events=False, heads=H, with_plan=True):
        import torch

        from specdec_b200.kernels import ops

        self.cache = cache
        self.batch = ops.RaggedBatch.from_lengths(q_lens, ctx_lens)
        L = cache.num_layers
        g = torch.Generator(device="cuda").manual_seed(seed + 1)
        self.q = [torch.randn(self.batch.total_rows, heads, cache.head_dim, generator=g, device="cuda").to(torch.bfloat16)
                  for _ in range(L)]
        self.out = [torch.empty_like(x) for x in self.q]
        self.ws = ops.attn_workspace(self.batch, heads, cache)
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.events = ([(torch.cuda.Event(enable_timing=True, external=True),
                         torch.cuda.Event(enable_timing=True, external=True)) for _ in range(L)]
                       if events else None)
        from specdec_b200 import _lib

        self._lib = _lib
        self.with_plan = with_plan
        ops.ragged_plan(self.q[0], self.cache, self.batch, self.ws, status=self.status)
        self._run()  # warm the extension (function attributes, plan) outside capture
        torch.cuda.synchronize()
        n0 = _lib.load_library().specdec_launch_count()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self._run()
        torch.cuda.current_stream().wait_stream(s)
        self.launches_per_step = int(_lib.load_library().specdec_launch_count() - n0)

    def _run(self):
        from specdec_b200.kernels import ops

        if self.with_plan:
            ops.ragged_plan(self.q[0], self.cache, self.batch, self.ws, status=self.status)
        for layer in range(self.cache.num_layers):
            # layer 0 follows the plan kernel directly (or, without the plan, the previous
            # replay's last attention kernel); later layers follow attention kernels, which
            # write no KV, page table or plan: their loads may start early
            ops.paged_attention(self.q[layer], self.cache, layer, self.batch, out=self.out[layer], workspace=self.ws,
                                reuse_plan=True, status=self.status,
                                history_ready=layer > 0 or not self.with_plan,
                                split_events=None if self.events is None else self.events[layer])

    def replay(self):
        self.graph.replay()

    def split_ms(self):
        """Mean split-kernel duration (ms) over the layers of the last replay."""
        return statistics.mean(b.elapsed_time(e) for b, e in self.events)


def time_steps(step, steps, warmup, world):
    import torch

    for _ in range(warmup):
        step.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step.replay()
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    return t0.elapsed_time(t1)


def time_windows(step, steps, warmup, world, windows=5):
    """W warm-up steps, then `windows` timed windows of exactly `steps` steps each (barrier +
    synchronize on both sides of every window); returns each window's max-over-ranks ms."""
    out = []
    for w in range(windows):
        ms = time_steps(step, steps, warmup if w == 0 else 0, world)
        out.append(max_over_ranks(ms, world))
    return out


def measure_config(T, q, fp8, steps, warmup, layers=LAYERS, seed=0):
    """(GB/s, ms/step) of one GPU for a batch-1 q/T config over `layers` distinct caches."""
    import torch

    cache = filled_cache(layers, [T], fp8, seed)
    step = GraphStep(cache, [q], [T], seed)
    ms = time_steps(step, steps, warmup, 1)
    st = int(step.status.item())
    del step, cache
    torch.cuda.empty_cache()
    if st:
        raise RuntimeError(f"device status {st:#x}")
    return layers * attn_bytes(T, q, fp8) * steps / (ms * 1e-3) / 1e9, ms / steps


def measure_ragged(steps, warmup, seed=4, fp8=True, layers=LAYERS):
    """64 sequences, T ~ U[1024, 8192], q in {1, 5} 1:1, E4M3 V (or bf16 V),
    one launch per layer over `layers` layer caches (the target's 28: one plan per step serves
    them all, as in the engine)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    lens = [int(x) for x in torch.randint(1024, 8193, (64,), generator=g)]
    q_lens = [1, 5] * 32
    perm = torch.randperm(64, generator=g).tolist()
    q_lens = [q_lens[i] for i in perm]
    cache = filled_cache(layers, lens, fp8, seed)
    step = GraphStep(cache, q_lens, lens, seed)
    ms = time_steps(step, steps, warmup, 1)
    byt = layers * sum(attn_bytes(t, q, fp8) for t, q in zip(lens, q_lens))
    st = int(step.status.item())
    del step, cache
    torch.cuda.empty_cache()
    if st:
        raise RuntimeError(f"device status {st:#x}")
    return byt * steps / (ms * 1e-3) / 1e9, ms / steps, byt / layers


DRAFT_LAYERS = 24  # Qwen2.5-0.5B


def measure_draft(steps, warmup, seed=5, layers=DRAFT_LAYERS):
    """Draft-model decode attention (Qwen2.5-0.5B geometry: 14:2 heads, head_dim 64, bf16 K/V):
    64 sequences at context 8192, q_len 1, one launch per layer over the draft's 24 layer caches."""
    import torch

    lens, q_lens = [8192] * 64, [1] * 64
    cache = filled_cache(layers, lens, False, seed, d=64)
    step = GraphStep(cache, q_lens, lens, seed, heads=14)
    ms = time_steps(step, steps, warmup, 1)
    byt = layers * sum(attn_bytes(t, q, False, heads=14, d=64) for t, q in zip(lens, q_lens))
    st = int(step.status.item())
    del step, cache
    torch.cuda.empty_cache()
    if st:
        raise RuntimeError(f"device status {st:#x}")
    return byt * steps / (ms * 1e-3) / 1e9, ms / steps, byt / layers


APPEND_BYTES_PER_TOKEN = 1800  # per layer: V bf16 512 in, codes 256 + scales 8 out, K bf16 512 in + 512 out


def measure_append(steps, warmup, n_tokens, layers=LAYERS, seed=7):
    """BASELINE configs[2]'s append-quantize kernel (specdec_append_kv, E4M3 V): one step appends
    `n_tokens` tokens of one sequence (2 KV heads x 128 dims) into each of `layers` layer caches
    -- the whole 8192-token history, or one decode / verify step's 1 or 5 tokens.  Returns
    (GB/s, us per launch); algorithmic bytes 1800 per token per layer."""
    import torch

    from specdec_b200.engine.paged_cache import PagedKVCache
    from specdec_b200.kernels import ops

    T = 8192
    cache = PagedKVCache.allocate(layers, 1, KV, D, T, v_dtype="e4m3", device="cuda", page_order_seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed)
    ks = [torch.randn(n_tokens, KV, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    vs = []
    for _ in range(layers):
        v = torch.randn(n_tokens, KV, D, generator=g, device="cuda")
        hit = torch.rand(v.shape, generator=g, device="cuda") < 0.01
        sgn = torch.where(torch.rand(v.shape, generator=g, device="cuda") < 0.5, -8.0, 8.0)
        vs.append(torch.where(hit, sgn, v).to(torch.bfloat16))
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")  # noqa: E731
    row0, n_new, pos0 = i32([0]), i32([n_tokens]), i32([T - n_tokens])

    class _Step:
        def __init__(self):
            self.graph = torch.cuda.CUDAGraph()

        def run(self):
            for layer in range(layers):
                ops.append_kv(ks[layer], vs[layer], cache, layer, row0=row0, n_new=n_new, pos0=pos0, max_new=n_tokens)

        def replay(self):
            self.graph.replay()

    st = _Step()
    st.run()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(st.graph, stream=s):
            st.run()
    torch.cuda.current_stream().wait_stream(s)
    ms = time_steps(st, steps, warmup, 1)
    per_launch_us = ms / steps / layers * 1e3
    del st, cache, ks, vs
    torch.cuda.empty_cache()
    return n_tokens * APPEND_BYTES_PER_TOKEN / (per_launch_us * 1e-6) / 1e9, per_launch_us


def cpu_fp8_baselines(T=8192):
    """The reference's quantize_kv_fp8 / dequantize_kv_fp8 (model_self.py:304-320, restated bit-exactly in
    oracle/engine.py) on the host, all threads: the V history of one layer at T tokens, and one token."""
    import torch

    from oracle.engine import dequantize_kv_fp8, quantize_kv_fp8

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    v = torch.randn(1, KV, T, D, generator=g).to(torch.bfloat16)
    v1 = v[:, :, :1].contiguous()

    def timed(fn, budget=2.0):
        for _ in range(3):
            fn()
        n, t0 = 0, time.perf_counter()
        while True:
            fn()
            n += 1
            if time.perf_counter() - t0 >= budget and n >= 20:
                break
        return (time.perf_counter() - t0) / n * 1e3, n

    codes, scale = quantize_kv_fp8(v, 128)
    q_ms, qn = timed(lambda: quantize_kv_fp8(v, 128))
    d_ms, dn = timed(lambda: dequantize_kv_fp8(codes, scale, torch.bfloat16))
    q1_ms, q1n = timed(lambda: quantize_kv_fp8(v1, 128), budget=1.0)
    return {"quantize_kv_fp8_T8192_ms": round(q_ms, 4), "dequantize_kv_fp8_T8192_ms": round(d_ms, 4),
            "quantize_kv_fp8_1token_ms": round(q1_ms, 4), "threads": torch.get_num_threads(), "kind": "port",
            "sample": f"{qn}/{dn}/{q1n} calls of oracle/engine.py quantize_kv_fp8 / dequantize_kv_fp8 "
                      f"(pinned bit-exact to the reference), V (1, 2, {T}, 128) bf16"}


def cpu_specdec_baseline(prompt_len=128, max_new=8, k=4, seed=0):
    """Greedy SpecDec decode tokens/s of the reference's strict executor (spec_dec.py:189-275,
    restated in oracle/specdec.py over the oracle decoder) on the host, all threads, with the
    configs[4] geometries (random-init bf16 Qwen2.5-1.5B target, 0.5B draft): one sequence with
    a `prompt_len`-token uniform-random prompt -- a bounded sample of the config, whose full size
    (256 sequences x 8192 prompt tokens) would take hours on the host."""
    import torch

    import oracle.engine as oeng
    from oracle.specdec import spec_decode_greedy
    from specdec_b200.engine.model import QWEN25_0P5B, QWEN25_1P5B, random_state

    torch.set_num_threads(os.cpu_count() or 1)

    def build(cfg, s):
        with torch.device("meta"):
            m = oeng.QwenLM(cfg.vocab, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate,
                            cfg.layers, rope_theta=cfg.rope_theta, attn_bias=cfg.attn_bias)
        m = m.to_empty(device="cpu").to(torch.bfloat16)
        # the GPU engine's seeded weights, drawn on the device (drawing 2 B values on the host
        # takes minutes) and copied to host memory
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        m.load_state_dict({k: v.cpu() for k, v in random_state(cfg, s, dev).items()}, strict=True)
        if dev == "cuda":
            torch.cuda.empty_cache()
        return m.eval()

    t_build = time.perf_counter()
    tgt, drf = build(QWEN25_1P5B, seed + 1), build(QWEN25_0P5B, seed + 2)
    t_build = time.perf_counter() - t_build
    prompt = torch.randint(0, QWEN25_1P5B.vocab, (1, prompt_len), generator=torch.Generator().manual_seed(seed))
    t0 = time.perf_counter()
    with torch.inference_mode():
        tl, _ = tgt._run(tgt.embed_tokens(prompt), None)
        dl, _ = drf._run(drf.embed_tokens(prompt), None)
    t_prefill = time.perf_counter() - t0
    t0 = time.perf_counter()
    res = spec_decode_greedy(tgt, drf, prompt, max_new, k=k)
    el = time.perf_counter() - t0 - t_prefill  # the executor runs its own prompt pass first
    del tgt, drf
    return {"decode_tokens_per_s": round(max_new / max(el, 1e-9), 3), "decode_s": round(el, 3),
            "rounds": res["stats"]["rounds"], "accepted": res["stats"]["accepted"], "threads": torch.get_num_threads(),
            "kind": "port",
            "sample": f"1 sequence, prompt {prompt_len} tokens, {max_new} new tokens, k={k} (oracle/specdec.py over "
                      f"oracle/engine.py, pinned to the reference); decode time = executor time minus one measured "
                      f"prompt pass of both models ({t_prefill:.2f} s); weights built in {t_build:.1f} s"}


def measure_lmhead(steps, warmup, rows, hidden, vocab=151936, seed=8):
    """The fused LM-head argmax (specdec_lmhead_argmax) against the unfused path it replaces
    (cuBLAS bf16 logits + torch.argmax), each replayed as a CUDA graph: (us fused, us unfused,
    fused TFLOP/s).  Algorithmic work 2 * rows * hidden * vocab flops; W (vocab x hidden bf16)
    is read once."""
    import torch

    from specdec_b200.kernels import ops

    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(vocab, hidden, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    ws = ops.lmhead_workspace(rows)

    def graph_of(fn):
        fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                fn()
        torch.cuda.current_stream().wait_stream(s)

        class _G:
            def replay(self):
                gr.replay()
        return _G(), gr

    fused, g1 = graph_of(lambda: ops.lmhead_argmax(x, w, out=out, workspace=ws))
    unfused, g2 = graph_of(lambda: out.copy_((x @ w.t()).argmax(-1)))
    ms_f = time_steps(fused, steps, warmup, 1) / steps
    ms_u = time_steps(unfused, steps, warmup, 1) / steps
    del g1, g2
    return ms_f * 1e3, ms_u * 1e3, 2.0 * rows * hidden * vocab / (ms_f * 1e-3) / 1e12


def measure_e2e(steps, warmup, T=8192, q=5, layers=LAYERS, seed=0):
    """Public-API path with host buffers; returns (GB/s, ms/step, h2d bytes/step, d2h bytes/step).

    One step: the step's q and new K/V rows of every layer copied from pinned host memory,
    the device plan, per layer ops.append_kv + ops.paged_attention, and the outputs copied
    back to pinned host memory.  The step's calls are captured once as a CUDA graph (as a
    serving loop runs its decode step) and replayed; every replay moves the host data."""
    import torch

    from specdec_b200.kernels import ops

    cache = filled_cache(layers, [T], False, seed)
    batch = ops.RaggedBatch.from_lengths([q], [T])
    nq, nkv = q * H * D, q * KV * D
    per = nq + 2 * nkv  # bf16 elements of one layer's inputs
    hin = torch.randn(layers * per).to(torch.bfloat16).pin_memory()
    hout = torch.empty(layers * nq, dtype=torch.bfloat16).pin_memory()
    din = torch.empty_like(hin, device="cuda")
    dout = torch.empty(layers * nq, dtype=torch.bfloat16, device="cuda")
    ws = ops.attn_workspace(batch, H, cache)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")  # noqa: E731
    row0, n_new, pos0 = i32([0]), i32([q]), i32([T - q])

    def step():
        din.copy_(hin, non_blocking=True)
        ops.ragged_plan(din[:nq].view(q, H, D), cache, batch, ws)
        for layer in range(layers):
            base = layer * per
            dq = din[base:base + nq].view(q, H, D)
            dk = din[base + nq:base + nq + nkv].view(q, KV, D)
            dv = din[base + nq + nkv:base + per].view(q, KV, D)
            ops.append_kv(dk, dv, cache, layer, row0=row0, n_new=n_new, pos0=pos0, max_new=q)
            # the append writes only this step's tokens: the history may be loaded early, as
            # the engine's decoder does after its append
            ops.paged_attention(dq, cache, layer, batch, out=dout[layer * nq:(layer + 1) * nq].view(q, H, D),
                                workspace=ws, reuse_plan=True, history_ready=layer > 0)
        hout.copy_(dout, non_blocking=True)

    step()  # warm the extension outside capture
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        graph.replay()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    h2d, d2h = hin.numel() * 2, hout.numel() * 2
    del graph, cache
    torch.cuda.empty_cache()
    return layers * attn_bytes(T, q, False) * steps / (ms * 1e-3) / 1e9, ms / steps, h2d, d2h


def measure_specdec(args, world, rank, seqs=None, draft_is_target=False):
    """greedy SpecDec with random-init Qwen2.5-1.5B (target) and
    Qwen2.5-0.5B (draft) geometries, args.specdec_seqs sequences with uniform-random
    prompts of args.specdec_prompt tokens, k = 4, args.specdec_new tokens each, sharded
    data-parallel over the ranks (one all-gather of tokens at the end).  Decode tokens/s
    counts the tokens emitted by decode rounds (the prompt pass's first token excluded)
    over the max-over-ranks device time of the round-graph replays."""
    import torch

    from specdec_b200.engine.dp import run_specdec_dp
    from specdec_b200.engine.model import QWEN25_0P5B, QWEN25_1P5B

    seqs = seqs or args.specdec_seqs
    res = run_specdec_dp(QWEN25_1P5B, QWEN25_0P5B, total_seqs=seqs, prompt_len=args.specdec_prompt,
                         max_new=args.specdec_new, k=4, seed=0, world=world, rank=rank, target_v="e4m3",
                         barrier=lambda: barrier(world), draft_is_target=draft_is_target)
    decode_tokens = seqs * (args.specdec_new - 1)
    out = {
        "decode_tokens_per_s": round(decode_tokens / res.decode_s, 1),
        "decode_s": round(res.decode_s, 4),
        "prefill_s": round(res.prefill_s, 3),
        "rounds": res.rounds,
        "accepted_per_round": round(res.acceptance, 3),
        "draft": "the target's weights (1.5B geometry)" if draft_is_target else "random-init Qwen2.5-0.5B geometry",
        "sequences": seqs, "prompt_len": args.specdec_prompt, "new_tokens": args.specdec_new,
        "k": 4, "n_gpus": world, "parallelism": f"dp{world}", "kv": "bf16 K / E4M3 V (target), bf16 (draft)",
        "weights": "random-init bf16 (seeded, identical on every rank)",
        "tokens_checksum": int(res.tokens.long().sum()),
    }
    del res
    torch.cuda.empty_cache()
    return out


def cpu_reference_step(layers=LAYERS, T=8192, q=5, seed=0):
    """One step of the reference arm / CPU baseline: the verify attention of one 28-layer target
    forward with the reference's eager formula (oracle/attention.py eager_attention, pinned to
    reference.attention), torch CPU on all host threads, over `layers` distinct K/V histories.
    Returns (run_step, bytes per step, threads)."""
    import torch

    from oracle.attention import eager_attention

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    qs = [torch.randn(1, H, q, D, generator=g).to(torch.bfloat16) for _ in range(layers)]
    ks = [torch.randn(1, KV, T, D, generator=g).to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(1, KV, T, D, generator=g).to(torch.bfloat16) for _ in range(layers)]

    def run_step():
        for layer in range(layers):
            eager_attention(qs[layer], ks[layer], vs[layer])

    return run_step, layers * attn_bytes(T, q, False), torch.get_num_threads()


def time_cpu_steps(run_step, steps, warmup, budget_s):
    """Warm-up, then up to `steps` timed steps, fewer when `budget_s` would be exceeded (at
    least 3).  Returns (seconds, steps timed, warm-up steps run)."""
    t0 = time.perf_counter()
    run_step()
    per = time.perf_counter() - t0
    warm = max(0, min(warmup, int(5.0 / max(per, 1e-9))) - 1)
    for _ in range(warm):
        run_step()
    timed = max(3, min(steps, int(budget_s / max(per, 1e-9))))
    t0 = time.perf_counter()
    for _ in range(timed):
        run_step()
    return time.perf_counter() - t0, timed, warm + 1


# ------------------------------------------------------------------------------ arms
def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    run_step, byt, thr = cpu_reference_step()
    el, timed, warm = time_cpu_steps(run_step, args.steps, args.warmup, 60.0)
    gbs = byt * timed / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": timed, "warmup": warm, "ms_per_step": round(el / timed * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "verify-attn q5 T8192 batch1 per GPU x 28 layer caches per step (configs[1])",
                   "model": "Qwen2.5-1.5B attention geometry 12:2 d128, bf16 K/V", "global_batch": 1,
                   "seq_len": 8192, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": thr, "kind": "port",
                         "sample": f"{timed} steps x 28 layer calls of the reference eager attention formula "
                                   f"(oracle/attention.py eager_attention, pinned to reference.attention; torch CPU, "
                                   f"{thr} threads); steps capped to ~60 s"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    import torch

    from specdec_b200 import _lib

    _lib.load_library()
    peak, peak_kind = measured_peak()
    bf16_peak = measured_bf16_peak()
    T, q = 8192, 5
    cache = filled_cache(LAYERS, [T], False, seed=rank)
    step = GraphStep(cache, [q], [T], seed=rank)
    with ClockSampler(local) as clk:
        windows = time_windows(step, args.steps, args.warmup, world)
    st = int(step.status.item())
    if st:
        raise RuntimeError(f"device status {st:#x}: {_lib.status_message(st)}")
    ms_max = statistics.median(windows)
    per_call = attn_bytes(T, q, False)
    value = world * LAYERS * per_call * args.steps / (ms_max * 1e-3) / 1e9
    launches = step.launches_per_step * args.steps
    del step
    # the dominant kernel's in-step duration: the same step's 28 verify launches without the
    # plan, replayed as one graph (programmatic dependent launches, as in the step), timed with
    # CUDA events over the replays -- 28 x launch_ms never exceeds ms_per_step
    vstep = GraphStep(cache, [q], [T], seed=rank, with_plan=False)
    v_ms = statistics.median(time_windows(vstep, max(args.steps, 50), args.warmup, world))
    launch_ms = v_ms / max(args.steps, 50) / LAYERS
    del vstep
    # the same kernels with CUDA events right around every launch (no overlap with neighbours)
    ev_step = GraphStep(cache, [q], [T], seed=rank, events=True)
    time_steps(ev_step, max(20, min(args.steps, 200)), args.warmup, world)
    isolated_ms = ev_step.split_ms()
    del ev_step, cache
    torch.cuda.empty_cache()

    extras = {}
    e2e = None
    cpu = None
    if world == 1 and not args.no_extras:
        ks = max(20, min(args.steps, 400))
        for TT in (2048, 4096, 8192):
            for qq in (1, 5):
                gbs, mss = measure_config(TT, qq, False, ks, 5)
                extras[f"bf16_T{TT}_q{qq}"] = {"GB/s": round(gbs, 1), "pct_of_8TBs": round(gbs / 80.0, 2),
                                              "frac_of_measured_peak": round(gbs / peak, 4),
                                              "us_per_layer": round(mss / LAYERS * 1e3, 3)}
        for qq in (1, 5):
            gbs, mss = measure_config(8192, qq, True, ks, 5)
            extras[f"e4m3v_T8192_q{qq}"] = {"GB/s": round(gbs, 1), "pct_of_8TBs": round(gbs / 80.0, 2),
                                           "frac_of_measured_peak": round(gbs / peak, 4),
                                           "us_per_layer": round(mss / LAYERS * 1e3, 3)}
        for fp8 in (True, False):
            gbs, mss, byt = measure_ragged(max(20, min(args.steps, 200)), 5, fp8=fp8)
            extras["ragged64_e4m3v" if fp8 else "ragged64_bf16"] = {
                "GB/s": round(gbs, 1), "pct_of_8TBs": round(gbs / 80.0, 2), "frac_of_measured_peak": round(gbs / peak, 4),
                "us_per_layer": round(mss / LAYERS * 1e3, 2), "bytes_per_layer": int(byt)}
        gbs, mss, byt = measure_draft(max(20, min(args.steps, 200)), 5)
        extras["draft64_d64_q1_T8192"] = {"GB/s": round(gbs, 1), "pct_of_8TBs": round(gbs / 80.0, 2),
                                          "frac_of_measured_peak": round(gbs / peak, 4),
                                          "us_per_layer": round(mss / DRAFT_LAYERS * 1e3, 2), "bytes_per_layer": int(byt)}
        app = {}
        for n_tok, label in ((8192, "history_T8192"), (1, "decode_1token"), (5, "verify_5tokens")):
            gbs, us = measure_append(max(20, min(args.steps, 200)), 5, n_tok)
            app[label] = {"GB/s": round(gbs, 1), "frac_of_measured_peak": round(gbs / peak, 4),
                          "us_per_launch": round(us, 3), "bytes_per_launch": n_tok * APPEND_BYTES_PER_TOKEN}
        app["note"] = ("specdec_append_kv with E4M3 V, one sequence x 2 KV heads x 128 dims, 28 layer caches per "
                       "step; algorithmic bytes 1800 per token per layer (V 512 in, codes 256 + scales 8 out, "
                       "K 512 in + 512 out)")
        extras["append_quantize_configs2"] = app
        lm = {}
        for rows, hidden, label in ((256, 896, "draft_256rows_h896"), (1280, 1536, "target_1280rows_h1536")):
            us_f, us_u, tf = measure_lmhead(max(20, min(args.steps, 100)), 5, rows, hidden)
            lm[label] = {"us_fused": round(us_f, 2), "us_cublas_plus_argmax": round(us_u, 2), "TFLOP/s": round(tf, 1),
                         "frac_of_measured_bf16_peak": round(tf / bf16_peak, 4)}
        lm["note"] = ("specdec_lmhead_argmax (tcgen05 GEMM over the 151936-row tied embedding fused with torch.argmax's "
                      "order; no logits written) vs x @ W^T (cuBLAS) + torch.argmax; 2 rows hidden vocab flops")
        extras["lmhead_argmax"] = lm
    if not args.no_extras:
        e_gbs, e_ms, h2d, d2h = measure_e2e(max(5, min(args.steps, 100)), 3)
        e2e = {"value": round(e_gbs * world, 3), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e_ms, 4),
               "path": "ops.append_kv + ops.paged_attention per layer (ctypes C ABI), the step's q/k/v copied in from "
                       "pinned host memory and the outputs copied back every step; the step's calls captured once as a "
                       "CUDA graph and replayed"}
        e_ms_max = max_over_ranks(e_ms, world)
        e2e["value"] = round(world * LAYERS * per_call / (e_ms_max * 1e-3) / 1e9, 3)
    specdec = specdec_full = None
    if not args.no_specdec:
        specdec = measure_specdec(args, world, rank)
        if not args.no_extras:
            specdec_full = measure_specdec(args, world, rank, seqs=max(world, args.specdec_seqs // 4),
                                           draft_is_target=True)
    cpu_extra = None
    if rank == 0 and not args.no_extras:
        run_step, byt, thr = cpu_reference_step()
        el, timed, _ = time_cpu_steps(run_step, 1000, 3, 15.0)
        c_gbs = byt * timed / el / 1e9
        cpu = {"value": round(c_gbs, 3), "unit": "GB/s", "cores": thr, "kind": "port",
               "sample": f"{timed} steps x 28 layer calls ({el:.1f} s) of the reference eager attention formula at "
                         f"q5 T8192 (oracle/attention.py, pinned to reference.attention; torch CPU, {thr} threads)"}
        del run_step
        cpu_extra = {"fp8_quantiser": cpu_fp8_baselines()}
        if not args.no_specdec:
            cpu_extra["spec_decode_greedy"] = cpu_specdec_baseline()

    achieved = per_call / (launch_ms * 1e-3) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "verify-attn q5 T8192 batch1 per GPU x 28 layer caches per step (configs[1])",
                       "model": "Qwen2.5-1.5B attention geometry 12:2 d128, bf16 K/V, 16-token pages, "
                                "random page order",
                       "global_batch": world, "seq_len": T, "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2: 28 distinct layer caches = 235 MB read per step"},
            "windows_ms": [round(w, 4) for w in windows],
            "pct_of_8TBs_per_gpu": round(value / world / 80.0, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": NCU_TRAFFIC_VERIFY8K,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, "
                                           "bench.py --profile-case verify8k",
                         "kernel": "verify_kernel<32,bf16V,pool> (tcgen05)", "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": per_call,
                         "launch_ms": round(launch_ms, 5),
                         "launch_ms_source": "in-step: graph of the step's 28 verify launches (no plan), CUDA events "
                                             "over its replays / 28",
                         "launch_ms_isolated": round(isolated_ms, 5)},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "extras": extras,
            "cpu_extras": cpu_extra,
            "specdec_e2e": specdec,
            "specdec_e2e_full_accept": specdec_full,
        }
        print(json.dumps(line), flush=True)


def run_profile_case(args):
    """Replays one workload's step graph (no timing, no JSON): the command profilers capture."""
    import torch

    from specdec_b200 import _lib

    _lib.load_library()
    if args.profile_case == "lmhead":
        # the target's LM-head argmax of 256 sequences' verify rows (1280 x 1536 x 151936)
        from specdec_b200.kernels import ops

        g = torch.Generator(device="cuda").manual_seed(8)
        x = torch.randn(1280, 1536, generator=g, device="cuda").to(torch.bfloat16)
        w = (torch.randn(151936, 1536, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        ws = ops.lmhead_workspace(1280)
        for _ in range(args.warmup + args.steps):
            ops.lmhead_argmax(x, w, workspace=ws)
        torch.cuda.synchronize()
        print(f"profile case lmhead: {args.warmup + args.steps} calls", flush=True)
        return
    if args.profile_case == "verify8k":
        cache = filled_cache(LAYERS, [8192], False, 0)
        step = GraphStep(cache, [5], [8192], 0)
    elif args.profile_case == "verify2k":
        cache = filled_cache(LAYERS, [2048], False, 0)
        step = GraphStep(cache, [5], [2048], 0)
    elif args.profile_case == "draft64":
        cache = filled_cache(2, [8192] * 64, False, 5, d=64)
        step = GraphStep(cache, [1] * 64, [8192] * 64, 5, heads=14)
    else:
        g = torch.Generator().manual_seed(4)
        lens = [int(x) for x in torch.randint(1024, 8193, (64,), generator=g)]
        q_lens = [1, 5] * 32
        perm = torch.randperm(64, generator=g).tolist()
        q_lens = [q_lens[i] for i in perm]
        cache = filled_cache(2, lens, args.profile_case == "ragged64", 4)
        step = GraphStep(cache, q_lens, lens, 4)
    for _ in range(args.warmup + args.steps):
        step.replay()
    torch.cuda.synchronize()
    st = int(step.status.item())
    if st:
        raise RuntimeError(f"device status {st:#x}: {_lib.status_message(st)}")
    print(f"profile case {args.profile_case}: {args.warmup + args.steps} replays, "
          f"{step.launches_per_step} launches per replay", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="headline line only (no extra configs/e2e/cpu)")
    ap.add_argument("--no-specdec", action="store_true", help="skip the end-to-end SpecDec tokens/s measurement")
    ap.add_argument("--specdec-seqs", type=int, default=256)
    ap.add_argument("--specdec-prompt", type=int, default=8192)
    ap.add_argument("--specdec-new", type=int, default=64)
    ap.add_argument("--profile-case", choices=["verify8k", "verify2k", "ragged64", "ragged64-bf16", "draft64", "lmhead"],
                    default=None,
                    help="only replay this workload's step graph warmup + steps times (for profilers)")
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference_arm(args, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
