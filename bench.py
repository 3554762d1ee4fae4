"""Benchmark of the continuous-batching talker decode step (codec frames/s).

Workload: 64 live streams per GPU; a random-init
(seed 0) 20-layer dense talker (hidden 1024, 16 q / 2 kv heads, head_dim 128,
SwiGLU 3072, codec vocab 3072) decoding one codec frame per stream per step
over a paged KV cache (page 16, pages randomly permuted in the pool, context
lengths log-normal(6, 0.8) clipped to [16, 8192]), followed by the config-0
code predictor (5 layers, 15 residual codebooks of 2048, T 0.9, top-k 50,
top-p 0.8) for all 64 streams.  One step = one CUDA graph replay of packing +
talker + layer-0 draw + predictor.  Synthetic data: seeded random weights,
KV contents and text rows.

The step streams ~3 GB (weights + KV) per step, far above the 126 MB L2, so
no L2 flush is needed between timed steps.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Under torchrun each rank runs an independent replica of the workload (data
parallel by request, no collective on the hot path); rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "sglang-omni_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "codec frames/s per GPU (ragged talker+codebook decode step); p50 step µs"
# DRAM traffic of the roofline kernels per algorithmic byte, from one ncu capture of the
# same kernel on the same workload (dram__bytes_read.sum + dram__bytes_write.sum over the
# algorithmic bytes of the captured launch; see profiles/).  The bench scales it to the
# timed launch by its algorithmic bytes (the traffic grows with the rows / tokens processed).
GEMM_TRAFFIC_RATIO: dict[int, float] = {1: (6_881_536 + 0) / (1024 * 3072 * 2 + 64 * 3072 * 2 + 2 * 64 * 1024 * 2 + 8 * 64 * 4)}
ATTN_TRAFFIC_RATIO: dict[int, float] = {1: (37_134_592 + 4_864) / (35_473 * 1024 + 64 * 16 * 128 * 2 * 2)}
UNIT = "frames/s"
STREAMS = 64


def context_lengths(n: int, seed: int, headroom: int) -> list[int]:
    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(np.exp(rng.normal(6.0, 0.8, n))), 16, 8192).astype(int)
    return [int(min(L, 8192 - headroom)) for L in lens]


def measured_peaks() -> tuple[float, float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples: list[list[str]] = []
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.samples.append([x.strip() for x in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU leg: the oracle restatement of the same step on the host cores
# ---------------------------------------------------------------------------
def cpu_step_rate(steps: int, warmup: int, seed: int = 0) -> tuple[float, dict, list[float]]:
    """Times the CPU restatement of the config-1 step (64 streams, 20 layers, 15
    codebooks) on the host cores; returns (frames/s, description, per-step seconds)."""
    from oracle.model import OracleTalker, rb  # noqa: F401  (test infrastructure: the CPU baseline)
    from omni_b200.config import CONFIG1_DENSE
    from omni_b200.predictor import init_predictor_weights
    from omni_b200.talker import init_talker_weights

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = CONFIG1_DENSE
    tw = init_talker_weights(cfg, seed=seed, device="cpu")
    pw = init_predictor_weights(cfg.predictor, seed=seed + 1, device="cpu")
    o = OracleTalker(cfg, tw, pw)
    lens = context_lengths(STREAMS, seed, headroom=steps + warmup + 8)
    B = STREAMS
    P = cfg.page_size
    total_slots = sum(L + steps + warmup + 1 for L in lens)
    L_ = cfg.num_hidden_layers
    g = torch.Generator().manual_seed(seed + 7)
    kpool = torch.randn(L_, total_slots, cfg.num_key_value_heads, cfg.head_dim, generator=g).bfloat16().float()
    vpool = torch.randn(L_, total_slots, cfg.num_key_value_heads, cfg.head_dim, generator=g).bfloat16().float()
    r2t = torch.zeros(B, max(lens) + steps + warmup + 2, dtype=torch.int32)
    off = 0
    for i, L in enumerate(lens):
        n = L + steps + warmup + 1
        r2t[i, :n] = torch.arange(off, off + n, dtype=torch.int32)
        off += n
    seq = torch.tensor(lens)
    feedback = torch.zeros(B, cfg.hidden_size).bfloat16()
    text = torch.randn(B, cfg.hidden_size, generator=g).bfloat16()
    l0 = dict(penalties=np.full(B, 1.05, np.float32), rep_mask=np.zeros((B, cfg.vocab_size), np.uint8),
              suppress_mask=np.zeros((B, cfg.vocab_size), np.uint8), temperature=np.full(B, 0.9, np.float32),
              top_k=np.full(B, 50), top_p=np.full(B, 0.8, np.float32), min_p=np.zeros(B, np.float32),
              seed=np.arange(B) + 1, max_top_k=50)
    sub = dict(temperature=np.full(B, 0.9, np.float32), top_k=np.full(B, 50), top_p=np.full(B, 0.8, np.float32),
               seed=np.arange(B) + 100, do_sample=np.ones(B, np.uint8), max_top_k=50, has_top_p=True)
    times = []
    for it in range(warmup + steps):
        t0 = time.perf_counter()
        seq = seq + 1
        pos = seq - 1
        loc = r2t[torch.arange(B), pos].long()
        logits, hidden = o.talker_forward(feedback, text, pos, loc, seq, r2t, kpool, vpool)
        l0["positions"] = pos.numpy()
        c0 = torch.from_numpy(o.layer0(logits, l0))
        codes, summed, _ = o.code_predictor(c0, hidden, pos, sub)
        feedback = torch.from_numpy(summed.view(np.int16)).view(torch.bfloat16)
        if it >= warmup:
            times.append(time.perf_counter() - t0)
    rate = B * len(times) / sum(times)
    desc = {"cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} full config-1 steps (64 streams, 20 layers, 15 codebooks) of the CPU "
                      f"restatement, fp32 on {torch.get_num_threads()} threads, after {warmup} warm-up steps"}
    return rate, desc, times


def cpu_slice_rate(config: int, seed: int = 0) -> dict:
    """The CPU restatement of a reduced slice of config 2 or 3, scaled to the full config
    (a bounded sample of host work; the scaling is stated in the returned description).

    config 3: the 256 streams through 1 of the 20 MoE layers (FP8 experts dequantised to
    fp32) and the 31-codebook predictor; talker time x 20 + predictor time.
    config 2: 2 new streams' prompts (two of the benchmark's prompt draw) with 14
    decode streams through the 20 dense layers in one mixed forward, then the layer-0 draw and
    the 15-codebook predictor for the 16 streams; forward time x (full token count / slice
    token count) + predictor time x (128 / 16)."""
    import dataclasses

    from oracle.model import OracleTalker  # test infrastructure: the CPU baseline
    from omni_b200.config import CONFIG1_DENSE, CONFIG3_MOE
    from omni_b200.predictor import init_predictor_weights
    from omni_b200.talker import init_talker_weights

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed + 7)
    if config == 3:
        cfg = dataclasses.replace(CONFIG3_MOE, num_hidden_layers=1)
        B, B_full, layers_full = 256, 256, CONFIG3_MOE.num_hidden_layers
    else:
        cfg = CONFIG1_DENSE
        B, B_full = 14, 112
    tw = init_talker_weights(cfg, seed=seed, device="cpu")
    pw = init_predictor_weights(cfg.predictor, seed=seed + 1, device="cpu")
    o = OracleTalker(cfg, tw, pw)
    lens = context_lengths(B, seed, headroom=8)
    prompts = []
    if config == 2:
        prng = np.random.default_rng(100)
        # two of the benchmark's 16 prompt lengths (its 3rd and 5th: 564 and 387 rows), which
        # keep the slice to tens of seconds of host work
        draw = [int(x) for x in prng.integers(64, 4097, 16)]
        prompts = [draw[2], draw[4]]
    slots = sum(L + 1 for L in lens) + sum(prompts)
    kpool = torch.randn(cfg.num_hidden_layers, slots, cfg.num_key_value_heads, cfg.head_dim,
                        generator=g).bfloat16().float()
    vpool = torch.randn_like(kpool)
    r2t = torch.zeros(B + len(prompts), max(lens + prompts) + 2, dtype=torch.int32)
    off = 0
    for i, L in enumerate(lens):
        r2t[i, : L + 1] = torch.arange(off, off + L + 1, dtype=torch.int32)
        off += L + 1
    seq = torch.tensor(lens) + 1
    pos = seq - 1
    loc = r2t[torch.arange(B), pos].long()
    feedback = torch.randn(B, cfg.hidden_size, generator=g).bfloat16()
    t0 = time.perf_counter()
    if config == 3:
        logits, hidden = o.talker_forward(feedback, None, pos, loc, seq, r2t, kpool, vpool)
        n = B
        positions = pos
    else:
        ext_pos, ext_loc, ext_ctx = [], [], []
        for j, L in enumerate(prompts):
            sl = torch.arange(off, off + L)
            r2t[B + j, :L] = sl.to(torch.int32)
            off += L
            ext_pos += list(range(L))
            ext_loc += sl.tolist()
            ext_ctx += [sl[: k + 1] for k in range(L)]
        prompt = torch.randn(sum(prompts), cfg.hidden_size, generator=g).bfloat16()
        select = torch.tensor(list(range(B)) + [B + int(x) for x in np.cumsum(prompts) - 1])
        logits, hidden = o.mixed_forward(feedback, None, pos, loc, seq, r2t, prompt, ext_pos, ext_loc, ext_ctx,
                                         select, kpool, vpool)
        n = B + len(prompts)
        positions = torch.cat([pos, torch.tensor([L - 1 for L in prompts])])
    t_talker = time.perf_counter() - t0
    l0 = dict(penalties=np.full(n, 1.05, np.float32), rep_mask=np.zeros((n, cfg.vocab_size), np.uint8),
              suppress_mask=np.zeros((n, cfg.vocab_size), np.uint8), temperature=np.full(n, 0.9, np.float32),
              top_k=np.full(n, 50), top_p=np.full(n, 0.8, np.float32), min_p=np.zeros(n, np.float32),
              seed=np.arange(n) + 1, max_top_k=50, positions=positions.numpy())
    sub = dict(temperature=np.full(n, 0.9, np.float32), top_k=np.full(n, 50), top_p=np.full(n, 0.8, np.float32),
               seed=np.arange(n) + 100, do_sample=np.ones(n, np.uint8), max_top_k=50, has_top_p=True)
    t0 = time.perf_counter()
    c0 = torch.from_numpy(o.layer0(logits, l0))
    o.code_predictor(c0, hidden, positions, sub)
    t_pred = time.perf_counter() - t0
    if config == 3:
        step_s = t_talker * (B_full / B) * (layers_full / cfg.num_hidden_layers) + t_pred * (B_full / B)
        frames = B_full
        scaling = f"talker slice time x {layers_full // cfg.num_hidden_layers} (layers) + predictor time"
        sample = f"one step of {B} streams through 1 MoE layer + the 31-codebook predictor"
    else:
        full_prompts = [int(x) for x in np.random.default_rng(100).integers(64, 4097, 16)]
        tok_slice, tok_full = B + sum(prompts), B_full + sum(full_prompts)
        step_s = t_talker * tok_full / tok_slice + t_pred * (B_full + 16) / n
        frames = B_full + 16
        scaling = (f"forward time x {tok_full}/{tok_slice} (token count) + predictor time x {B_full + 16}/{n} "
                   "(streams)")
        sample = (f"one mixed step: {B} decode streams + 2 prompts ({prompts[0]} + {prompts[1]} rows) through 20 "
                  "layers, then the 15-codebook predictor for 16 streams")
    return {"value": frames / step_s, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": sample + f", fp32 on {torch.get_num_threads()} threads; scaled: {scaling}",
            "slice_talker_s": t_talker, "slice_predictor_s": t_pred}


EXTRA_CONFIGS = (0, 2, 3, 4)


def run_extra_configs(args) -> dict:
    """Configs 0, 2, 3 and 4 measured in the same invocation as the headline (each in a
    child bench.py process on the same GPU, so that each starts with the device to itself):
    the child's JSON line, condensed.  Config 4 runs its whole 2048-stream trace (its own
    step count) whatever --steps says."""
    out = {}
    for c in EXTRA_CONFIGS:
        steps = max(5, min(args.steps, 20))
        cmd = [sys.executable, str(ROOT / "bench.py"), "--config", str(c), "--steps", str(steps), "--warmup",
               str(max(3, args.warmup)), "--cpu-steps", "1"]
        if args.no_cpu:
            cmd.append("--no-cpu")
        try:
            proc = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        except subprocess.TimeoutExpired:
            out[f"config{c}"] = {"error": "timed out"}
            continue
        line = None
        for ln in proc.stdout.splitlines():
            if ln.startswith("{"):
                line = json.loads(ln)
        if proc.returncode != 0 or line is None:
            out[f"config{c}"] = {"error": f"exit {proc.returncode}: {proc.stderr[-300:]}"}
            continue
        keep = ("value", "unit", "ms_per_step", "p50_step_us", "p99_step_us", "steps", "warmup", "gpu_launches",
                "roofline", "roofline_attention", "roofline_prefill_attention", "cpu_baseline", "e2e", "clocks")
        entry = {k: line[k] for k in keep if k in line}
        entry["workload"] = line.get("config", {}).get("workload")
        out[f"config{c}"] = entry
    # the streaming vocoder that consumes the step's codes: the Qwen3-Omni code2wav slot
    # decode (64 streams x 10 new frames, graph-replayed) and its kernels
    try:
        proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--vocoder"], capture_output=True, text=True,
                              timeout=900)
        kernels, decode = [], None
        for ln in proc.stdout.splitlines():
            if ln.startswith("{"):
                d = json.loads(ln)
                if "step" in d:
                    decode = d
                else:
                    kernels.append(d)
        out["code2wav"] = {"decode": decode, "kernels": kernels} if decode else {
            "error": f"exit {proc.returncode}: {proc.stderr[-300:]}"}
    except subprocess.TimeoutExpired:
        out["code2wav"] = {"error": "timed out"}
    return out


# ---------------------------------------------------------------------------
def run_reference_arm(args, rank: int) -> None:
    if rank != 0:
        return
    # the step count and warm-up the driver asks for (at least 3 warm-ups; at most 50 steps,
    # about half a second each on the host cores)
    steps = max(1, min(args.steps, 50))
    warmup = max(3, min(args.warmup, 10))
    if args.config == 0:
        cb = cpu_predictor_rate(steps)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": 8000.0 / cb["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config0: code predictor alone, 8 streams, 15 codebooks"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    rate, desc, times = cpu_step_rate(steps, warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
        "warmup": warmup, "ms_per_step": 1000 * float(np.median(times)), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config1: dense talker decode, 64 streams + config-0 predictor",
                   "streams": STREAMS, "layers": 20, "codebooks": 15},
        "cpu_baseline": {"value": rate, "unit": UNIT, **desc},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_kernel(fn, iters: int) -> float:
    """Average device time (s) of one fn() launch: `iters` launches are captured in a
    CUDA graph (so host-side launch cost is excluded) and the replay is timed with
    CUDA events on the capturing stream."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(iters):
            fn()
    st = torch.cuda.current_stream()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    g.replay()
    e1.record(st)
    e1.synchronize()
    del g
    return e0.elapsed_time(e1) / 1000.0 / iters


def kernel_table(runner, iters: int = 50, only: str | None = None) -> list[dict]:
    """Steady-state device time of every distinct launch of the step (each replayed
    `iters` times back to back from a CUDA graph, CUDA events), with algorithmic bytes.
    Launches of one row cycle through the layers (the talker's 20, the predictor's 5),
    as the step does, so a launch does not find its weights or KV left in L2 by the
    previous launch of the same row."""
    from omni_b200 import ops
    from omni_b200.sampling_kernels import predictor_sample_step

    cfg = runner.cfg
    t, p = runner.talker, runner.predictor
    B = runner.batch_size
    fb = runner.forward_batch()
    pc = cfg.predictor
    H = cfg.hidden_size
    L = cfg.num_hidden_layers
    eps = cfg.rms_norm_eps
    rows_out = []

    def add(name, fn, nbytes, count_per_step):
        if only is not None and only not in name:
            return
        sec = time_kernel(fn, iters)
        rows_out.append({"kernel": name, "us": sec * 1e6, "bytes": nbytes, "gbs": nbytes / sec / 1e9,
                         "per_step": count_per_step})

    wb = lambda w: w.numel() * 2  # noqa: E731

    class Cycle:
        def __init__(self, n):
            self.n, self.i = n, 0

        def __call__(self):
            v = self.i % self.n
            self.i += 1
            return v

    tl = Cycle(L)  # talker layer of the next launch
    lw, fw = t.w["layers"][0], t.folded[0]
    kc, vc = runner.kv.k_buffer[0], runner.kv.v_buffer[0]
    qkv_geo = dict(num_q_heads=cfg.num_attention_heads, num_kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                   q_norm=lw["q_norm"], k_norm=lw["k_norm"], eps=eps, cos_sin=t.cos_sin, positions=fb.positions,
                   cache_loc=fb.out_cache_loc, k_cache=kc, v_cache=vc)
    add("talker input add+sumsq", lambda: ops.add_sumsq(p.output_embeds[:B], runner.text_embeds[:B], t.h[:B], t.ss[0]),
        3 * B * H * 2, 1)
    add("talker qkv gemm (+norm,rope,kv)", lambda: ops.linear_fused(
        t.h[:B], t.folded[tl()]["qkv"], t.q[:B], epilogue=ops.EPI_QKV_ROPE, ss_in=t.ss, ss_in_parts=8, norm_eps=eps,
        qkv=qkv_geo), wb(fw["qkv"]), L)
    seq_now = runner.seq_lens[:B].cpu().numpy()
    kv_bytes = float(seq_now.sum()) * cfg.num_key_value_heads * cfg.head_dim * 2 * 2
    # each timed launch reads another layer's KV pool (as the step does), so the
    # KV of a launch is not resident in L2 from the previous one
    layer_cycle = {"i": 0}

    def next_layer_kv():
        li = layer_cycle["i"] % L
        layer_cycle["i"] += 1
        return runner.kv.k_buffer[li], runner.kv.v_buffer[li]

    add("talker paged attention", lambda: ops.paged_decode_attention(
        t.q[:B], *next_layer_kv(), page_indptr=fb.page_indptr, page_indices=fb.page_indices, seq_lens=fb.seq_lens,
        work_indptr=fb.work_indptr, num_q_heads=cfg.num_attention_heads, num_kv_heads=cfg.num_key_value_heads,
        head_dim=cfg.head_dim, page_size=cfg.page_size, pages_per_chunk=fb.pages_per_chunk,
        work_capacity=fb.work_capacity, sm_scale=t.scale, out=t.attn[:B], workspace=t.attn_workspace), kv_bytes, L)
    add("talker o_proj gemm (+res,ss)", lambda: ops.linear_fused(
        t.attn[:B], t.w["layers"][tl()]["o_proj"], t.h[:B], epilogue=ops.EPI_RESIDUAL, residual=t.h[:B],
        ss_out=t.ss), wb(lw["o_proj"]), L)
    if cfg.moe is None:
        add("talker gate_up gemm (+norm,swiglu)", lambda: ops.linear_fused(
            t.h[:B], t.folded[tl()]["gate_up"], t.act[:B], epilogue=ops.EPI_SWIGLU, ss_in=t.ss, ss_in_parts=8,
            norm_eps=eps), wb(fw["gate_up"]), L)
        add("talker down gemm (+res,ss)", lambda: ops.linear_fused(
            t.act[:B], t.w["layers"][tl()]["down_proj"], t.h[:B], epilogue=ops.EPI_RESIDUAL, residual=t.h[:B],
            ss_out=t.ss), wb(lw["down_proj"]), L)
    else:
        m, mw, mc = t.moe, lw["moe"], cfg.moe
        E, k = mc.num_experts, mc.num_experts_per_tok
        gain = lw["post_attention_layernorm"]
        ids, tw = m.topk_ids[:B], m.topk_weights[:B]
        ops.moe_rmsnorm_quant(t.h[:B], t.ss, 8, gain, eps, m.x[:B], m.xq[:B], m.xs[:B])
        ops.linear_fused(m.x[:B], mw["gate"], m.router_logits[:B], epilogue=ops.EPI_ROUTER,
                         router={"topk_ids": ids, "topk_weights": tw})
        torch.cuda.synchronize()
        used = int(torch.unique(ids).numel())
        add("moe rmsnorm+fp8 quant", lambda: ops.moe_rmsnorm_quant(t.h[:B], t.ss, 8, gain, eps, m.x[:B], m.xq[:B],
                                                                  m.xs[:B]), B * H * 5, L)
        add("moe router gemm (+softmax,top-k)", lambda: ops.linear_fused(
            m.x[:B], mw["gate"], m.router_logits[:B], epilogue=ops.EPI_ROUTER,
            router={"topk_ids": ids, "topk_weights": tw}), wb(mw["gate"]), L)
        add("moe align+gather", lambda: ops.moe_align_gather(
            ids, E, m.xq[:B], m.xs[:B], m.permuted_q, m.permuted_s, m.slot_of[:B], m.expert_offsets, m.chunks,
            m.n_chunks), 2 * B * k * H, L)
        add("moe gate_up fp8 grouped gemm (+swiglu,quant)", lambda: ops.moe_gate_up_fp8(
            m.permuted_q, m.permuted_s, mw["w13"], mw["w13_scale"], m.chunks, m.n_chunks, m.act_q, m.act_s),
            used * mw["w13"][0].numel(), L)
        add("moe down fp8 grouped gemm", lambda: ops.moe_down_fp8(
            m.act_q, m.act_s, mw["w2"], mw["w2_scale"], m.chunks, m.n_chunks, m.y), used * mw["w2"][0].numel(), L)
        add("moe shared gate_up gemm (swiglu)", lambda: ops.linear_fused(
            m.x[:B], mw["shared_gate_up"], m.shared_act[:B], epilogue=ops.EPI_SWIGLU), wb(mw["shared_gate_up"]), L)
        add("moe shared down gemm", lambda: ops.linear_fused(
            m.shared_act[:B], mw["shared_down"], m.shared_out[:B], epilogue=ops.EPI_STORE), wb(mw["shared_down"]), L)
        h_copy = t.h[:B].clone()
        ss_copy = t.ss.clone()
        add("moe combine (+res,ss)", lambda: ops.moe_combine(
            m.y, m.slot_of[:B], tw, m.x[:B], mw["shared_expert_gate"], m.shared_out[:B], h_copy, ss_copy),
            B * k * H * 2 + 4 * B * H * 2, L)
    add("talker codec_head gemm (+norm)", lambda: ops.linear_fused(
        t.h[:B], t.codec_head_folded, t.logits[:B], epilogue=ops.EPI_F32, ss_in=t.ss, ss_in_parts=8, norm_eps=eps),
        wb(t.codec_head_folded), 1)
    add("layer0 sampler", lambda: t.sample_decode_tokens(t.logits[:B], fb), B * cfg.vocab_size * 4, 1)
    plw, pfw = p.w["layers"][0], p.folded[0]
    n5 = pc.num_hidden_layers
    pl = Cycle(n5)  # predictor layer of the next launch
    hl = Cycle(pc.num_code_groups - 1)  # lm_head of the next launch
    for rows, label, per, base in ((2 * B, "pair", 1, 0), (B, "single", pc.num_code_groups - 2, 8)):
        T = rows // B
        geo = dict(num_q_heads=pc.num_attention_heads, num_kv_heads=pc.num_key_value_heads, head_dim=pc.head_dim,
                   q_norm=plw["q_norm"], k_norm=plw["k_norm"], eps=eps, cos_sin=p.cos_sin, tokens_per_req=T,
                   slot_stride=pc.cache_len, slot_base=base, k_cache=p.k_cache[0], v_cache=p.v_cache[0])
        add(f"predictor[{label}] qkv gemm (+norm,rope,kv)", lambda rows=rows, geo=geo: ops.linear_fused(
            p.h[:rows], p.folded[pl()]["qkv"], p.q[:rows], epilogue=ops.EPI_QKV_ROPE, ss_in=p.ss, ss_in_parts=8,
            norm_eps=eps, qkv=geo), wb(pfw["qkv"]), per * n5)
        add(f"predictor[{label}] attention", lambda rows=rows, T=T, base=base: ops.predictor_attention(
            p.q[:rows], p.k_cache[0], p.v_cache[0], num_q_heads=pc.num_attention_heads,
            num_kv_heads=pc.num_key_value_heads, head_dim=pc.head_dim, tokens_per_req=T, slot_stride=pc.cache_len,
            slot_base=base, sm_scale=p.scale, out=p.attn[:rows]),
            rows * (pc.cache_len // 2) * pc.num_key_value_heads * pc.head_dim * 4, per * n5)
        add(f"predictor[{label}] o_proj gemm (+res,ss)", lambda rows=rows: ops.linear_fused(
            p.attn[:rows], p.w["layers"][pl()]["o_proj"], p.h[:rows], epilogue=ops.EPI_RESIDUAL,
            residual=p.h[:rows], ss_out=p.ss), wb(plw["o_proj"]), per * n5)
        add(f"predictor[{label}] gate_up gemm (+norm,swiglu)", lambda rows=rows: ops.linear_fused(
            p.h[:rows], p.folded[pl()]["gate_up"], p.act[:rows], epilogue=ops.EPI_SWIGLU, ss_in=p.ss,
            ss_in_parts=8, norm_eps=eps), wb(pfw["gate_up"]), per * n5)
        add(f"predictor[{label}] down gemm (+res,ss)", lambda rows=rows: ops.linear_fused(
            p.act[:rows], p.w["layers"][pl()]["down_proj"], p.h[:rows], epilogue=ops.EPI_RESIDUAL,
            residual=p.h[:rows], ss_out=p.ss), wb(plw["down_proj"]), per * n5)
    add("predictor lm_head gemm (+norm)", lambda: ops.linear_fused(
        p.h[:B], p.lm_head_folded[hl()], p.logits[1, :B], epilogue=ops.EPI_STORE, ss_in=p.ss, ss_in_parts=8,
        norm_eps=eps), wb(p.lm_head_folded[1]), pc.num_code_groups - 1)
    add("predictor sample+gather", lambda: predictor_sample_step(
        p.logits[1, :B], temperatures=p.sub_temperature_tensor[:B], top_ks=p.sub_top_k_tensor[:B],
        top_ps=p.sub_top_p_tensor[:B], seeds=p.sub_sampling_seed_tensor[:B], positions=fb.positions, pos_mul=pc.num_code_groups - 1,
        pos_add=2, do_sample=None, argmax_all=False, max_top_k=p.sub_sampled_max_top_k,
        has_top_p=p.sub_sampled_has_top_p, codes=p.output_codes[:B, 2], table=p.w["codec_embedding"][1],
        gathered=p.next_in[:B], summed=p.output_embeds[:B], gathered_ss=p.next_ss[:B]),
        B * pc.vocab_size * 2 + 3 * B * H * 2, pc.num_code_groups - 1)
    return rows_out


def run_vocoder(args) -> None:
    """One JSON line per vocoder-step kernel: device time (CUDA graph of launches, inputs
    larger than L2 rotated through) and HBM bandwidth against the measured copy peak."""
    from omni_b200.kernels.bias_snake_beta import SnakeBetaCoefficients, fused_bias_snake_beta
    from omni_b200.kernels.codec_state import history_exchange, overlap_exchange
    from omni_b200.kernels.single_output_conv import clamped_single_output_conv

    hbm, _, kind = measured_peaks()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    bf = torch.bfloat16
    sets = 4  # input sets cycled through: every set is larger than L2 / sets
    lines = []

    class _Act:
        def __init__(self, c):
            self.alpha = (torch.randn(c, device=dev) * 0.5).to(bf)
            self.beta = (torch.randn(c, device=dev) * 0.5).to(bf)
            self.no_div_by_zero = 1e-9

    # SnakeBeta over a code2wav block's conv output: 64 streams x 256 positions x 1536 channels
    B, L, C = 64, 256, 1536
    coef = SnakeBetaCoefficients.from_activation(_Act(C))
    bias = torch.randn(C, device=dev, dtype=bf)
    xs = [torch.randn(B, L, C, device=dev, dtype=bf) for _ in range(sets)]
    rs = [torch.randn(B, L, C, device=dev, dtype=bf) for _ in range(sets)]
    outs = [torch.empty(B, L, C, device=dev, dtype=bf) for _ in range(sets)]
    sums = [torch.empty(B, L, C, device=dev, dtype=bf) for _ in range(sets)]
    cyc = {"i": 0}

    def snake():
        i = cyc["i"] % sets
        cyc["i"] += 1
        fused_bias_snake_beta(xs[i], bias, coef, outs[i], residual=rs[i], sum_out=sums[i])

    t = time_kernel(snake, 32)
    nbytes = 4 * B * L * C * 2
    lines.append(("bias_snake_beta (conv + bias + residual -> SnakeBeta, sum)", f"[{B}, {L}, {C}] bf16", t, nbytes))

    # the last conv of code2wav: 96 channels, 7 taps, 64 streams x 4800 samples
    B2, L2, C2, taps = 64, 4800, 96, 7
    conv = torch.nn.Conv1d(C2, 1, taps).to(device=dev, dtype=bf)
    pads = [torch.randn(B2, L2 + taps - 1, C2, device=dev, dtype=bf) for _ in range(sets)]

    def sconv():
        i = cyc["i"] % sets
        cyc["i"] += 1
        clamped_single_output_conv(pads[i], conv, L2)

    with torch.inference_mode():
        t = time_kernel(sconv, 32)
    nbytes = B2 * (L2 + taps - 1) * C2 * 2 + B2 * L2 * 2
    lines.append(("clamped_single_output_conv", f"[{B2}, {L2}+{taps - 1}, {C2}] bf16", t, nbytes))

    # codec state of a causal conv (history 6) and a transposed conv (overlap 8), 1536 channels
    R, H, N, O, E = 64, 6, 32, 8, 32
    pool = torch.randn(R, H, C, device=dev, dtype=bf)
    slot = torch.arange(R, device=dev)
    padded = torch.randn(R, H + N, C, device=dev, dtype=bf)
    opool = torch.randn(R, O, C, device=dev, dtype=bf)
    out_t = torch.randn(R, E + O, C, device=dev, dtype=bf)
    t = time_kernel(lambda: history_exchange(padded, pool, slot, N, False), 32)
    lines.append(("history_exchange", f"{R} slots x {H} samples x {C} ch bf16", t, R * C * 2 * (3 * H)))
    t = time_kernel(lambda: overlap_exchange(out_t, opool, slot, E, False), 32)
    lines.append(("overlap_exchange", f"{R} slots x {O} samples x {C} ch bf16", t, R * C * 2 * (4 * O)))

    for name, shape, secs, nbytes in lines:
        gbs = nbytes / secs / 1e9
        print(json.dumps({"kernel": name, "shape": shape, "us": secs * 1e6, "algorithmic_bytes": nbytes,
                          "achieved_gbs": gbs, "peak_gbs": hbm, "frac": gbs / hbm, "peak_kind": kind}))
    del xs, rs, outs, sums, pads

    # the implicit-GEMM causal conv (tcgen05) on code2wav decode shapes: the dilated 7-tap
    # conv of a residual unit, plain and with the next SnakeBeta fused in its epilogue
    from omni_b200 import ops

    _, tflops_peak, _ = measured_peaks()
    for rows, length, ch, dil, fused in ((64, 1600, 384, 3, False), (64, 1600, 384, 3, True),
                                         (64, 6400, 192, 9, True), (64, 320, 768, 1, True)):
        taps = 7
        hist = (taps - 1) * dil
        pads3 = [torch.randn(rows, hist + length, ch, device=dev, dtype=bf) for _ in range(2)]
        w = (torch.randn(ch, taps * ch, device=dev) / (taps * ch) ** 0.5).to(bf)
        ys = [torch.empty(rows, length, ch, device=dev, dtype=bf) for _ in range(2)]
        cf = SnakeBetaCoefficients.from_activation(_Act(ch))
        bch = torch.randn(ch, device=dev, dtype=bf)
        cyc3 = {"i": 0}

        def cgemm():
            i = cyc3["i"] % 2
            cyc3["i"] += 1
            if fused:
                ops.conv1d_gemm(pads3[i], w, taps=taps, dilation=dil, length=length, out=ys[i], bias=bch,
                                alpha_scale=cf.alpha_scale, inverse_beta=cf.inverse_beta)
            else:
                ops.conv1d_gemm(pads3[i], w, taps=taps, dilation=dil, length=length, out=ys[i])

        t = time_kernel(cgemm, 20)
        flops = 2.0 * rows * length * ch * taps * ch
        print(json.dumps({"kernel": "conv1d_gemm" + (" + SnakeBeta epilogue" if fused else ""),
                          "shape": f"[{rows}, {hist}+{length}, {ch}] -> {ch}, 7 taps, dilation {dil}",
                          "us": t * 1e6, "algorithmic_flops": flops, "achieved_tflops": flops / t / 1e12,
                          "peak_tflops": tflops_peak, "frac": flops / t / 1e12 / tflops_peak, "peak_kind": kind}))
        del pads3, ys

    # the whole code2wav slot decode: Qwen3-Omni code2wav geometry (transformers' defaults:
    # 8-layer pre-transformer, decoder_dim 1536, 16 quantizers of 2048), random bf16
    # weights, 64 streams decoding 10 new frames each (the talker's steady codec chunk),
    # graph-replayed
    from transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe import Qwen3OmniMoeCode2WavConfig
    from transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe import Qwen3OmniMoeCode2Wav
    from omni_b200.code2wav import Qwen3OmniIncrementalCodec

    cfg = Qwen3OmniMoeCode2WavConfig()
    cfg._attn_implementation = "sdpa"
    model = Qwen3OmniMoeCode2Wav(cfg).to(device=dev, dtype=bf).eval()
    codec = Qwen3OmniIncrementalCodec(model)
    S, NF = 64, 10
    pool = codec.make_pool(num_slots=S, ring_frames=codec.layout.retained + NF)
    slots = torch.arange(S, device=dev)
    codes = torch.randint(0, cfg.codebook_size, (S, cfg.num_quantizers, NF), device=dev)
    with torch.inference_mode():
        codec.decode_slots(codes, pool, slots, first_decode=True)
        t = time_kernel(lambda: codec.decode_slots(codes, pool, slots, first_decode=False), 8)
    fps = S * NF / t
    rate = 24000 / codec.samples_per_frame()
    print(json.dumps({"step": "code2wav slot decode (warm)", "streams": S, "frames_per_decode": NF,
                      "us": t * 1e6, "frames_per_s": fps, "audio_seconds_per_s": fps / rate,
                      "state_bytes_per_slot": pool.bytes_per_slot}))
    if args.profile:
        # device time per kernel over 3 eager decodes (torch profiler, CUDA activity)
        from torch.profiler import ProfilerActivity, profile

        with torch.inference_mode():
            torch.cuda.synchronize()
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                for _ in range(3):
                    codec.decode_slots(codes, pool, slots, first_decode=False)
                torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=16, max_name_column_width=60))


def run_config0(args, world: int, rank: int, local_rank: int, dist) -> None:
    """Config 0 (the reference's CPU-runnable case) on the GPU: the code predictor alone
    for 8 streams (5 layers, 15 residual codebooks of 2048, T 0.9 / top-k 50 / top-p 0.8,
    talker hidden ~ N(0, 1)), one frame a step, graph-replayed; the CPU leg times the
    oracle restatement of the same predictor loop."""
    from omni_b200 import _lib, ops
    from omni_b200.config import CONFIG0_PREDICTOR
    from omni_b200.predictor import CodePredictor, init_predictor_weights
    from omni_b200.seed import derive_sampling_seed

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    pc, B = CONFIG0_PREDICTOR, 8
    H, G, V0 = pc.hidden_size, pc.num_code_groups, 3072
    pw = init_predictor_weights(pc, seed=1, device=dev)
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    emb0 = (torch.randn(V0, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    p = CodePredictor(pc, pw, max_batch=B, device=dev, layer0_embedding=emb0)
    seeds = [derive_sampling_seed("subtalker", derive_sampling_seed("omni-b200", rank, f"req{i}")) for i in range(B)]
    p.set_sampling(temperature=[0.9] * B, top_k=[50] * B, top_p=[0.8] * B, seeds=seeds, do_sample=[True] * B,
                   batch=B)
    c0 = torch.randint(0, V0, (B,), generator=g, device=dev)
    hidden = torch.randn(B, H, generator=g, device=dev).to(torch.bfloat16)
    norm = torch.ones(H, dtype=torch.bfloat16, device=dev)
    ss = hidden.float().view(B, H // 128, 128).pow(2).sum(-1).t().contiguous()
    positions = torch.arange(B, device=dev) * 7

    def step():
        p.code_predictor_forward(c0, hidden, positions, final_norm=norm, final_ss=ss, final_eps=pc.rms_norm_eps)

    step()
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    s_ = torch.cuda.Stream(dev)
    s_.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s_):
        step()
    torch.cuda.current_stream(dev).wait_stream(s_)
    launches_per_step = _lib.launch_count() - n0
    W, K = max(3, args.warmup), args.steps
    for _ in range(W):
        graph.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    with ClockSampler(local_rank) as clocks:
        ev[0].record(st)
        for i in range(K):
            graph.replay()
            ev[i + 1].record(st)
        torch.cuda.synchronize()
    step_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(K)]
    total_ms = ev[0].elapsed_time(ev[K])
    # end to end: the inputs in from pinned host memory, the codes out, every step
    c0_h = c0.cpu().pin_memory()
    hid_h = hidden.cpu().pin_memory()
    codes_h = torch.empty(B, G, dtype=torch.long).pin_memory()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(st)
    for _ in range(K):
        c0.copy_(c0_h, non_blocking=True)
        hidden.copy_(hid_h, non_blocking=True)
        graph.replay()
        codes_h.copy_(p.output_codes[:B], non_blocking=True)
        st.synchronize()
    t1.record(st)
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1)
    # the dominant kernel: the predictor gate_up GEMM (+ folded norm, SwiGLU) over the 5 layers in turn
    cyc = {"i": 0}
    eps = pc.rms_norm_eps

    def gate_up():
        li = cyc["i"] % pc.num_hidden_layers
        cyc["i"] += 1
        ops.linear_fused(p.h[:B], p.folded[li]["gate_up"], p.act[:B], epilogue=ops.EPI_SWIGLU, ss_in=p.ss,
                         ss_in_parts=H // 128, norm_eps=eps)

    gu_s = time_kernel(gate_up, 60)
    wgu = p.folded[0]["gate_up"]
    gu_bytes = wgu.numel() * 2 + B * H * 2 + B * pc.intermediate_size * 2
    params = sum(v.numel() for lw in pw["layers"] for k, v in lw.items() if k.endswith("proj"))
    step_bytes = (G - 1) * (params + pc.vocab_size * H) * 2
    from omni_b200.replicas import aggregate_step_times

    total_max, e2e_max, frames = aggregate_step_times(total_ms, e2e_ms, float(B * K), dist, dev)
    if rank == 0:
        hbm, _, peak_kind = measured_peaks()
        achieved = gu_bytes / gu_s / 1e9
        line = {
            "metric": METRIC, "value": frames / (total_max / 1000.0), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": total_ms / K, "p50_step_us": 1000 * float(np.median(step_ms)),
            "p99_step_us": 1000 * float(np.percentile(step_ms, 99)), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config0: code predictor alone, 8 streams (5 layers, H 1024, 16q/8kv hd 64, "
                                   "SwiGLU 3072, 15 residual codebooks of 2048, T 0.9 / top-k 50 / top-p 0.8, "
                                   "talker hidden N(0,1)), one frame a step",
                       "streams_per_gpu": B, "parallelism": f"dp{world} replicas (no collective)",
                       "step_bytes": step_bytes,
                       "step_bandwidth_gbs": step_bytes / (total_ms / K / 1000.0) / 1e9,
                       "l2": "weights 126 MB of predictor layers + 63 MB of lm_heads cycle each step (> L2)"},
            "e2e": {"value": frames / (e2e_max / 1000.0), "unit": UNIT, "h2d_bytes_per_step": B * 8 + B * H * 2,
                    "d2h_bytes_per_step": B * G * 8},
            "gpu_launches": launches_per_step * K,
            "roofline": {"bound": "hbm", "kernel": "gemm_kernel<2>: predictor gate_up + folded norm + SwiGLU "
                                                   "(8 rows)",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "traffic": None,
                         "algorithmic_bytes": gu_bytes, "launch_us": gu_s * 1e6, "peak_kind": peak_kind},
            "clocks": clocks.summary(),
        }
        if not args.no_cpu:
            line["cpu_baseline"] = cpu_predictor_rate(args.cpu_steps)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def cpu_predictor_rate(steps: int) -> dict:
    """The oracle restatement of config 0's predictor loop (8 streams, fp32) on the host cores."""
    from oracle.model import OracleTalker  # test infrastructure: the CPU baseline
    from omni_b200.config import CONFIG0_PREDICTOR, TalkerConfig
    from omni_b200.predictor import init_predictor_weights
    from omni_b200.talker import init_talker_weights

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = TalkerConfig(num_hidden_layers=1, predictor=CONFIG0_PREDICTOR)
    o = OracleTalker(cfg, init_talker_weights(cfg, seed=0, device="cpu"),
                     init_predictor_weights(CONFIG0_PREDICTOR, seed=1, device="cpu"))
    B = 8
    g = torch.Generator().manual_seed(3)
    c0 = torch.randint(0, cfg.vocab_size, (B,), generator=g)
    hid = torch.randn(B, cfg.hidden_size, generator=g).bfloat16().float()
    sub = dict(temperature=np.full(B, 0.9, np.float32), top_k=np.full(B, 50), top_p=np.full(B, 0.8, np.float32),
               seed=np.arange(B) + 100, do_sample=np.ones(B, np.uint8), max_top_k=50, has_top_p=True)
    times = []
    for it in range(steps + 1):
        t0 = time.perf_counter()
        o.code_predictor(c0, hid, torch.arange(B) * 7, sub)
        if it:
            times.append(time.perf_counter() - t0)
    return {"value": B * len(times) / sum(times), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} config-0 predictor steps (8 streams, 15 codebooks) of the CPU restatement, "
                      f"fp32 on {torch.get_num_threads()} threads, after 1 warm-up step"}


def run_config4(args, world: int, rank: int, local_rank: int, dist) -> None:
    """Config 4: 2048 streams arriving by a Poisson process, sharded over the GPUs by
    request (round-robin binding, no collective), each GPU running the continuous-
    batching event loop (C++ scheduler: admission with the prefill-coalescing gate,
    mixed decode + prefill steps, page allocation, compaction) over the MoE talker
    of config 3 until every stream has all its frames.  The timed region is the whole
    run, end to end through the public loop: text and prompt rows copied in from
    pinned host memory, every step's codes copied out."""
    import dataclasses

    from omni_b200 import _lib
    from omni_b200.config import CONFIG3_MOE
    from omni_b200.continuous import ContinuousTalkerRunner, poisson_arrival_trace
    from omni_b200.model_runner import TalkerDecodeRunner
    from omni_b200.replicas import shard_streams
    from omni_b200.scheduler import MIXED, OmniScheduler, SchedulerConfig

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    frames_range = (64, 192)
    cfg = dataclasses.replace(CONFIG3_MOE, max_context=8192 + frames_range[1])
    max_batch, max_prefill = 320, 8192
    trace = poisson_arrival_trace(args.streams, world, 256, frames_range)
    mine = set(shard_streams(args.streams, world, rank))
    arrivals: dict[int, list] = {}
    for rid, step, L, F in trace:
        if rid in mine:
            arrivals.setdefault(step, []).append((rid, L, F))
    want_frames = sum(F for rid, _, _, F in trace if rid in mine)
    num_pages = 32768
    sc = SchedulerConfig(num_pages=num_pages, page_size=cfg.page_size, max_batch=max_batch,
                         max_context=cfg.max_context, max_prefill_tokens=max_prefill,
                         coalesce_requests=args.coalesce, coalesce_when_idle=False, coalesce_wait_us=40_000,
                         reserve_ratio=1.0, page_seed=rank + 1, emit_messages=True, codec_coalesce_frames=10,
                         codec_coalesce_early_frames=10)
    runner = TalkerDecodeRunner(cfg, max_batch=max_batch + 1, num_pages=num_pages, seed=0, device=dev,
                                max_prefill_tokens=max_prefill)
    cr = ContinuousTalkerRunner(runner, OmniScheduler(sc), seed=rank)
    cr.capture_buckets()  # warm-up: the decode graph of every bucket (start-up capture)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = _lib.launch_count()
    step_s, rows_seen, mixed, idle = [], [], 0, 0
    frames = emitted = 0
    last = max(arrivals) if arrivals else 0
    with ClockSampler(local_rank) as clocks:
        e0.record(st)
        t_start = time.perf_counter()
        step = 0
        while True:
            for rid, L, F in arrivals.get(step, []):
                cr.sched.add_request(rid, L, F)
            t0 = time.perf_counter()
            out = cr.step()
            step += 1
            if out is None:
                idle += 1
                if step > last and cr.sched.stats()["waiting"] == 0 and cr.sched.stats()["running"] == 0:
                    break
                continue
            msgs = cr.pop_messages()  # the code chunks handed to the vocoder stage
            step_s.append(time.perf_counter() - t0)
            rows_seen.append(len(out.rids))
            frames += len(out.rids)
            emitted += sum(m[2].shape[0] for m in msgs)
            mixed += out.mode == MIXED
        e1.record(st)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t_start
    total_ms = e0.elapsed_time(e1)
    launches = _lib.launch_count() - n0
    st_sched = cr.sched.stats()
    assert frames == want_frames and st_sched["finished"] == len(mine), "a stream did not get all its frames"
    assert emitted == want_frames, "a frame did not reach the vocoder queue"
    assert cr.device_status() == 0
    steps = len(step_s)
    h2d, d2h = cr.h2d_bytes, cr.d2h_bytes
    from omni_b200.replicas import aggregate_step_times

    total_ms_max, wall_ms_max, frames_all = aggregate_step_times(total_ms, wall * 1000.0, frames, dist, dev)
    if rank == 0:
        value = frames_all / (total_ms_max / 1000.0)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": 0,
            "ms_per_step": total_ms / max(steps, 1), "p50_step_us": 1e6 * float(np.median(step_s)),
            "p99_step_us": 1e6 * float(np.percentile(step_s, 99)), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"config4: {args.streams} streams (prompts lognormal(6,0.8) clip [16,8192], "
                                   f"frames U[{frames_range[0]},{frames_range[1]}]) arriving by a seeded Poisson "
                                   "process in step time at 256 live streams per GPU, sharded round-robin over the "
                                   "GPUs; continuous batching (C++ scheduler, mixed decode + prefill steps, "
                                   f"prefill-coalescing gate {args.coalesce} requests / 40 ms, decode graphs per "
                                   "bucket, frames to the vocoder queue in the talker's chunks: 10 single frames, "
                                   "then 10 a chunk) over the config-3 MoE talker + 31-codebook predictor, run to "
                                   "completion",
                       "streams_rank0": len(mine), "parallelism": f"dp{world} replicas (no collective)",
                       "warmup": "decode graphs of every bucket recorded before the timed region",
                       "mixed_steps_rank0": mixed, "mean_rows_rank0": float(np.mean(rows_seen)),
                       "graph_steps_rank0": cr.graph_steps, "eager_steps_rank0": cr.eager_steps,
                       "retracted_rank0": st_sched["retracted"], "idle_iterations_rank0": idle,
                       "l2": "inputs > L2 (MoE experts 3 GB + KV streamed per step)"},
            "e2e": {"value": frames_all / (wall_ms_max / 1000.0), "unit": UNIT,
                    "h2d_bytes_per_step": h2d / max(steps, 1), "d2h_bytes_per_step": d2h / max(steps, 1),
                    "note": "the timed loop is itself end to end (host scheduler, pinned copies in and out)"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        cr.graphs.clear()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=2)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="with --config 1 on one GPU: skip the configs 0 / 2 / 3 lines under 'configs'")
    ap.add_argument("--kernels", action="store_true", help="print the per-kernel time table and exit")
    ap.add_argument("--only", default=None, help="with --kernels: only the rows whose name contains this text")
    ap.add_argument("--ep", action="store_true",
                    help="with --config 3 under torchrun: experts sharded over the ranks (NCCL all-to-all)")
    ap.add_argument("--layers", type=int, default=0,
                    help="with --kernels: talker layers to build (0 = the config's 20); for small profiling runs")
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4],
                    help="0: the code predictor alone, 8 streams; "
                         "1: dense talker, 64 streams (the headline); 2: mixed prefill (16 new streams, prompts "
                         "U[64, 4096]) + 112 decode streams; 3: MoE talker with FP8 experts, 256 streams; "
                         "4: continuous batching of Poisson arrivals over the config-3 model")
    ap.add_argument("--streams", type=int, default=2048, help="with --config 4: streams of the whole job")
    ap.add_argument("--coalesce", type=int, default=8,
                    help="with --config 4: prefill-coalescing gate (requests; <= 1 turns it off)")
    ap.add_argument("--vocoder", action="store_true",
                    help="time the streaming vocoder step's kernels (one JSON line each) and exit")
    ap.add_argument("--profile", action="store_true",
                    help="with --vocoder: print the code2wav decode's device time per kernel")
    args = ap.parse_args()
    if args.vocoder:
        run_vocoder(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # the CPU arm needs no process group: rank 0 runs and prints, the others exit
        run_reference_arm(args, rank)
        return
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))

    if args.config == 4:
        run_config4(args, world, rank, local_rank, dist)
        return
    if args.config == 0:
        run_config0(args, world, rank, local_rank, dist)
        return

    from omni_b200 import _lib, ops
    from omni_b200.config import CONFIG1_DENSE, CONFIG3_MOE
    from omni_b200.model_runner import TalkerDecodeRunner

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    global STREAMS
    prompts: list[int] = []
    if args.config == 3:
        cfg, STREAMS = CONFIG3_MOE, 256
    elif args.config == 2:
        cfg = CONFIG1_DENSE
        prng = np.random.default_rng(100 + rank)
        prompts = [int(x) for x in prng.integers(64, 4097, 16)]
        STREAMS = 112  # decode streams; every step also prefills the 16 prompts
    else:
        cfg = CONFIG1_DENSE
    if args.layers and args.kernels:
        import dataclasses

        cfg = dataclasses.replace(cfg, num_hidden_layers=args.layers)
    W, K = max(3, args.warmup), args.steps
    total_steps = 2 * (W + K) + 4
    lens = context_lengths(STREAMS, seed=rank, headroom=total_steps + 8)
    P = cfg.page_size
    pages = int(sum(math.ceil((L + total_steps) / P) for L in lens) * 1.25) + STREAMS
    pages += sum(math.ceil(L / P) for L in prompts)
    ep = bool(args.ep and cfg.moe is not None and world > 1)
    runner = TalkerDecodeRunner(cfg, max_batch=STREAMS + len(prompts), num_pages=pages, seed=0, device=dev,
                                expert_parallel=ep, max_prefill_tokens=sum(prompts))
    runner.admit(lens, seed=rank)
    if prompts:
        runner.admit_prefill(prompts, seed=rank)
    frames_per_step = STREAMS + len(prompts)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    runner.text_embeds.normal_(generator=g)
    if args.kernels:
        runner.step(use_graph=False)
        torch.cuda.synchronize()
        table = kernel_table(runner, only=args.only)
        if rank == 0:
            tot = max(1e-9, sum(r["us"] * r["per_step"] for r in table))
            for r in table:
                print(f'{r["kernel"]:34s} {r["us"]:8.2f} us  x{r["per_step"]:3d}/step  {r["gbs"]:8.1f} GB/s  '
                      f'{100 * r["us"] * r["per_step"] / tot:5.1f}% of kernel time')
            print(f"sum of isolated kernel times per step: {tot:.1f} us")
        return
    n0 = _lib.launch_count()
    runner.capture(warmup=1)
    launches_per_step = (_lib.launch_count() - n0) // 2  # one eager warm-up step + the captured step

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident leg ----
    for _ in range(W):
        runner.step()
    barrier()
    st = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    with ClockSampler(local_rank) as clocks:
        ev[0].record(st)
        for i in range(K):
            runner.step()
            ev[i + 1].record(st)
        barrier()
    step_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(K)]
    total_ms = ev[0].elapsed_time(ev[K])

    # ---- end-to-end leg: pinned host text rows in, host codes out, every step ----
    H = cfg.hidden_size
    G = cfg.predictor.num_code_groups
    text_host = torch.randn(STREAMS, H).to(torch.bfloat16).pin_memory()
    codes_host = torch.empty((frames_per_step, G), dtype=torch.long).pin_memory()
    for _ in range(W):
        runner.decode(text_host, codes_host)
    barrier()
    t_e0 = torch.cuda.Event(enable_timing=True)
    t_e1 = torch.cuda.Event(enable_timing=True)
    t_e0.record(st)
    for _ in range(K):
        runner.decode(text_host, codes_host)
    t_e1.record(st)
    barrier()
    e2e_ms = t_e0.elapsed_time(t_e1)

    # ---- the dominant kernel (the residual-epilogue GEMM, gemm_kernel<1>: 34.6% of the
    # step's device time in the launch list) and the paged attention, each timed in
    # isolation over the 20 layers in turn (weights / KV far beyond L2), as in the step ----
    fb = runner.forward_batch()
    t = runner.talker
    gcyc = {"i": 0}
    dense = cfg.moe is None
    gw = [lw["down_proj"] if dense else lw["o_proj"] for lw in t.w["layers"]]
    R = STREAMS + sum(prompts)  # rows of the talker forward (config 2: decode rows + prompt rows)
    g_in = t.act[:R] if dense else t.attn[:R]
    g_name = ("gemm_kernel<1>: talker down projection + residual + row sums of squares" if dense else
              "gemm_kernel<1>: talker o_proj + residual + row sums of squares")

    def gemm_next():
        li = gcyc["i"] % cfg.num_hidden_layers
        gcyc["i"] += 1
        ops.linear_fused(g_in, gw[li], t.h[:R], epilogue=ops.EPI_RESIDUAL, residual=t.h[:R], ss_out=t.ss)

    gemm_s = time_kernel(gemm_next, 20 if prompts else 60)
    gk, gn = g_in.shape[1], gw[0].shape[0]
    # weights + activations in + residual in + output + per-128-feature sums of squares
    gemm_bytes = gn * gk * 2 + R * gk * 2 + 2 * R * gn * 2 + (gn // 128) * R * 4
    gemm_flops = 2.0 * R * gk * gn
    pf_s = pf_flops = None
    if prompts:
        ext = runner.extend
        pcyc = {"i": 0}
        Bd = STREAMS

        def prefill_next():
            li = pcyc["i"] % cfg.num_hidden_layers
            pcyc["i"] += 1
            ops.prefill_attention(t.q[Bd:R], runner.kv.k_buffer[li], runner.kv.v_buffer[li],
                                  qo_indptr=ext.qo_indptr, seq_lens=ext.seq_lens, page_indptr=ext.page_indptr,
                                  page_indices=ext.page_indices, tile_indptr=ext.tile_indptr,
                                  max_tiles=ext.max_tiles, num_q_heads=cfg.num_attention_heads,
                                  num_kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim, page_size=P,
                                  sm_scale=t.scale, out=t.attn[Bd:R])

        pf_s = time_kernel(prefill_next, 20)
        # causal QK^T and PV: 2 x 2 x Hq x D x L (L + 1) / 2 per prompt
        pf_flops = sum(2.0 * cfg.num_attention_heads * cfg.head_dim * L * (L + 1) for L in prompts)
    attn_args = dict(page_indptr=fb.page_indptr, page_indices=fb.page_indices, seq_lens=fb.seq_lens,
                     work_indptr=fb.work_indptr, num_q_heads=cfg.num_attention_heads,
                     num_kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim, page_size=P,
                     pages_per_chunk=fb.pages_per_chunk, work_capacity=fb.work_capacity, sm_scale=t.scale,
                     out=t.attn[:STREAMS], workspace=t.attn_workspace)
    # 20 layers' KV pools in turn (each ~37 MB; together far beyond L2), as in the step
    cyc = {"i": 0}

    def attn_next():
        li = cyc["i"] % cfg.num_hidden_layers
        cyc["i"] += 1
        ops.paged_decode_attention(t.q[:STREAMS], runner.kv.k_buffer[li], runner.kv.v_buffer[li], **attn_args)

    attn_s = time_kernel(attn_next, 60)
    seq_now = runner.seq_lens[:STREAMS].cpu().numpy()
    attn_bytes = float(seq_now.sum()) * cfg.num_key_value_heads * cfg.head_dim * 2 * 2 \
        + STREAMS * cfg.num_attention_heads * cfg.head_dim * 2 * 2

    # ---- gather over ranks: max of the device times, sum of the frames ----
    from omni_b200.replicas import aggregate_step_times

    total_ms, e2e_ms, frames = aggregate_step_times(total_ms, e2e_ms, frames_per_step * K, dist, dev)
    if rank == 0:
        hbm, tflops, peak_kind = measured_peaks()
        value = frames / (total_ms / 1000.0)
        e2e = frames / (e2e_ms / 1000.0)
        achieved = attn_bytes / attn_s / 1e9
        g_achieved = gemm_bytes / gemm_s / 1e9
        workload = {
            1: "config1: dense talker decode (20 layers, 64 streams, paged KV page 16, ctx lognormal(6,0.8) "
               "clip [16,8192]) + config-0 predictor (15 codebooks)",
            2: "config2: one fused forward of 112 decode streams (config-1 contexts) + 16 new streams' prompts "
               f"(U[64,4096], sum {sum(prompts)} rows, KV written to the paged pool) through the 20-layer talker, "
               "then layer-0 draw + 15-codebook predictor for all 128 streams",
            3: "config3: MoE talker decode (20 layers, 128 experts top-8 inter 384 FP8 e4m3 128x128 block scales "
               "+ shared expert 1536, 256 streams, paged KV page 16, ctx lognormal(6,0.8) clip [16,8192]) + "
               "predictor (31 codebooks of 1024)"}[args.config]
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": total_ms / K, "p50_step_us": 1000 * float(np.median(step_ms)),
            "p99_step_us": 1000 * float(np.percentile(step_ms, 99)), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload,
                       "streams_per_gpu": STREAMS,
                       "parallelism": (f"ep{world}: experts sharded, NCCL all-to-all dispatch/combine per MoE layer"
                                       if ep else f"dp{world} replicas (no collective)"),
                       "sum_ctx_rank0": int(sum(lens)), "l2": "inputs > L2 (~3 GB streamed per step)"},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": STREAMS * H * 2,
                    "d2h_bytes_per_step": frames_per_step * G * 8},
            "gpu_launches": launches_per_step * K,
            "roofline": {"bound": "hbm", "kernel": g_name, "achieved": g_achieved, "peak": hbm, "unit": "GB/s",
                         "frac": g_achieved / hbm,
                         "traffic": (GEMM_TRAFFIC_RATIO[args.config] * gemm_bytes
                                     if args.config in GEMM_TRAFFIC_RATIO else None),
                         "algorithmic_bytes": gemm_bytes, "launch_us": gemm_s * 1e6, "peak_kind": peak_kind},
            "roofline_attention": {"bound": "hbm", "kernel": "paged_decode_attention_kernel", "achieved": achieved,
                                   "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                                   "traffic": (ATTN_TRAFFIC_RATIO[args.config] * attn_bytes
                                               if args.config in ATTN_TRAFFIC_RATIO else None),
                                   "algorithmic_bytes": attn_bytes,
                                   "launch_us": attn_s * 1e6, "peak_kind": peak_kind},
            "clocks": clocks.summary(),
        }
        if prompts:
            # the rows are many: the projections are tensor-bound
            line["roofline"] = {"bound": "tensor", "kernel": g_name + f" ({R} rows)",
                                "achieved": gemm_flops / gemm_s / 1e12, "peak": tflops, "unit": "TFLOP/s",
                                "frac": gemm_flops / gemm_s / 1e12 / tflops, "traffic": None,
                                "algorithmic_flops": gemm_flops, "launch_us": gemm_s * 1e6, "peak_kind": peak_kind}
            line["roofline_prefill_attention"] = {
                "bound": "tensor",
                "kernel": ("prefill_attention_pair_kernel" if (cfg.num_attention_heads // cfg.num_key_value_heads) % 2 == 0
                           else "prefill_attention_tc_kernel") + " (tcgen05, S, P and O in TMEM)",
                "achieved": pf_flops / pf_s / 1e12, "peak": tflops, "unit": "TFLOP/s",
                "frac": pf_flops / pf_s / 1e12 / tflops, "algorithmic_flops": pf_flops, "launch_us": pf_s * 1e6,
                "peak_kind": peak_kind}
        if not args.no_cpu and args.config == 1:
            rate, desc, _ = cpu_step_rate(args.cpu_steps, 1)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, **desc}
        elif not args.no_cpu and args.config in (2, 3):
            line["cpu_baseline"] = cpu_slice_rate(args.config)
        if args.config == 1 and world == 1 and not args.no_extra:
            line["configs"] = run_extra_configs(args)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        runner.graph = None
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
