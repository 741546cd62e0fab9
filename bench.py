"""Benchmark of the decoder token loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step" = one decoded token): the full 26-layer voxtral decoder
(dim 3072, 32/8 heads, head_dim 128, SwiGLU 9216, RMSNorm eps 1e-5, RoPE
theta 1e6), token embedding and untied LM head 131072 x 3072, bf16 weights
~N(0, 0.02) from seed 0, batch 1, KV window 8192, 512 random prompt ids
prefilled, then greedy decode.  Every step streams 6.86 GB of weights, far
more than the 126 MB L2, so no L2 flush is needed between steps.

With N > 1 (torchrun, one process per GPU) every rank decodes its own
independent stream (no collective on the data path: weak scaling); value is
the total tokens/s of all ranks over the slowest rank's time.

With N > 1 the ranks then decode one stream together, tensor parallel
(2048-token context, 1024 greedy steps), reported as "tensor_parallel".

Two more single-stream objects time --ctx-steps greedy steps from a cache
pre-filled with generator tokens: "long_context" at 1536 tokens (the end
context of the 512 + 1024-step workload) and "rolling" at the full 8192-token
window, where every step evicts the oldest token; the rolling object also
reports the ring state after the run against the kv.rs:48-88 index rule.

An "encoder" object streams 10 s of synthetic audio per GPU through the
encoder front end (log-mel + conv stem) in 80 ms chunks and reports audio
seconds per second, beside the oracle on a 2 s sample.

The same run then measures the multi-stream workload (8 independent streams
per GPU, contexts uniform in [256, 4096) with the cache prefilled from
N(0,1) bf16, greedy decode with tensor-core GEMMs) and reports it as the
"multi_stream" object of the JSON line (64 streams at 8 GPUs).

--impl reference times the reference's CPU algorithm (the oracle port: the
reference is Rust and cannot be built here) with all host threads on the same
workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

import ctypes
import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DIM, HIDDEN, NH, NKV, HD = 3072, 9216, 32, 8, 128
LAYERS, VOCAB, WINDOW = 26, 131072, 8192
PROMPT = 512
LONG_CONTEXT = 1536
METRIC = "decoder tokens/s (1 stream per GPU)"
WORKLOAD = "26-layer decoder token loop, batch 1, prefill 512 random ids then greedy decode, KV window 8192"

LAYER_WEIGHT_BYTES = 2 * (DIM * (NH * HD) + 2 * DIM * (NKV * HD) + (NH * HD) * DIM + 3 * DIM * HIDDEN)
HEAD_BYTES = 2 * VOCAB * DIM
EMBED_ROW_BYTES = 2 * DIM
KV_BYTES_PER_TOKEN_LAYER = 2 * NKV * HD * 4   # f32 K and V
C_SZ = ctypes.c_size_t


def step_bytes(ctx_len: int) -> int:
    """Algorithmic HBM bytes of one decode step at a given cache length."""
    return LAYERS * LAYER_WEIGHT_BYTES + HEAD_BYTES + EMBED_ROW_BYTES + LAYERS * KV_BYTES_PER_TOKEN_LAYER * ctx_len


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 tensor-core TFLOP/s: the measured burst figure (a prefill is
    a burst of a few milliseconds), else the fallback."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


class NvmlClockSampler:
    """SM clock and clock-event reasons read through NVML every 2 ms on a
    thread (read-only queries), so that even a 30 ms timed region gets samples;
    falls back to the nvidia-smi sampler when NVML is unavailable."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.fallback = None
        self.samples, self.reasons = [], set()
        self.max_mhz = 0.0
        self._stop = None
        self._thread = None

    def start(self):
        try:
            import threading

            import pynvml as N
            N.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            idx = int(vis.split(",")[self.gpu]) if vis and vis.split(",")[self.gpu].isdigit() else self.gpu
            h = N.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM))
            get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self.fallback = ClockSampler(self.gpu)
            self.fallback.start()
            return
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)))
                    bits = int(get_reasons(h))
                    for b, name in self.REASONS.items():
                        if bits & b:
                            self.reasons.add(name)
                except Exception:
                    pass
                self._stop.wait(0.002)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()

    def stop(self):
        if self.fallback is not None:
            return self.fallback.stop()
        if self._thread is None:
            return None
        self._stop.set()
        self._thread.join()
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml"}


# ---------------------------------------------------------------------------
# CPU baselines (oracle port of the reference's Rust kernels)
# ---------------------------------------------------------------------------

def cpu_token_rate(threads: int, n_layer_steps: int, n_head: int):
    """Per-token time of the oracle: n_layer_steps full-size layer steps plus
    n_head LM-head linears, all with f32 weights as the reference stores
    them, extrapolated to 26 layers + head.  Returns (tokens/s, sample text)."""
    from oracle import oracle as o
    o.build()
    o.set_threads(threads)
    c = dict(dim=DIM, hidden_dim=HIDDEN, n_heads=NH, n_kv_heads=NKV, head_dim=HD, sliding_window=WINDOW,
             norm_eps=1e-5, rope_theta=1e6)
    shapes = {"wq": NH * HD * DIM, "wk": NKV * HD * DIM, "wv": NKV * HD * DIM, "wo": DIM * NH * HD,
              "w1": HIDDEN * DIM, "w2": DIM * HIDDEN, "w3": HIDDEN * DIM}
    mats = {n: o.gen_normal_f32(0, i + 1, 0.02, s) for i, (n, s) in enumerate(shapes.items())}
    ones = np.ones(DIM, np.float32)
    lw = o.LayerWeights(ones, ones, **mats)
    cfg = o.config(**c)
    cache = o.RollingKvCache(1, NKV, HD, WINDOW)
    kvp = o.gen_normal_f32(0, 5000000, 1.0, PROMPT * NKV * HD)
    cache.layer_set(0, kvp, kvp, PROMPT, 0)
    x = o.gen_normal_f32(0, 2000000, 1.0, DIM)
    t0 = time.perf_counter()
    for i in range(n_layer_steps):
        x = o.decoder_layer_forward_step(cfg, 0, lw, cache, x, PROMPT + i)
    t_layer = (time.perf_counter() - t0) / n_layer_steps
    del mats, lw
    head = o.gen_normal_f32(0, 1000001, 0.02, VOCAB * DIM)
    t0 = time.perf_counter()
    for _ in range(n_head):
        xn = o.rms_norm_rows(x, ones, DIM, 1e-5)
        logits = o.linear(xn, 1, DIM, head, VOCAB)
        int(np.argmax(logits))
    t_head = (time.perf_counter() - t0) / n_head
    t_tok = LAYERS * t_layer + t_head
    sample = (f"{n_layer_steps} full-size layer steps at context {PROMPT} + {n_head} LM-head linears, f32 weights,"
              f" {threads} thread(s); per-token time = 26 x {t_layer * 1e3:.1f} ms + {t_head * 1e3:.1f} ms")
    return 1.0 / t_tok, sample


def run_reference(args):
    """Reference arm: the oracle port of the reference's CPU kernels on all host
    threads.  One step = one token through 26 layer steps + final norm + LM
    head + argmax, f32 weights as the reference stores them.  The 26 layers
    share one set of layer weights (the CPU time of a layer step does not
    depend on the weight values; each layer keeps its own KV cache)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle as o
    o.build()
    threads = os.cpu_count() or 1
    o.set_threads(threads)
    c = dict(dim=DIM, hidden_dim=HIDDEN, n_heads=NH, n_kv_heads=NKV, head_dim=HD, sliding_window=WINDOW,
             norm_eps=1e-5, rope_theta=1e6)
    shapes = {"wq": NH * HD * DIM, "wk": NKV * HD * DIM, "wv": NKV * HD * DIM, "wo": DIM * NH * HD,
              "w1": HIDDEN * DIM, "w2": DIM * HIDDEN, "w3": HIDDEN * DIM}
    mats = {n: o.gen_normal_f32(0, i + 1, 0.02, s_) for i, (n, s_) in enumerate(shapes.items())}
    ones = np.ones(DIM, np.float32)
    lw = o.LayerWeights(ones, ones, **mats)
    head = o.gen_normal_f32(0, 1000001, 0.02, VOCAB * DIM)
    cfg = o.config(**c)
    cache = o.RollingKvCache(LAYERS, NKV, HD, WINDOW)
    kvp = o.gen_normal_f32(0, 5000000, 1.0, PROMPT * NKV * HD)
    for l in range(LAYERS):
        cache.layer_set(l, kvp, kvp, PROMPT, 0)

    def token(pos, x):
        for l in range(LAYERS):
            x = o.decoder_layer_forward_step(cfg, l, lw, cache, x, pos)
        xn = o.rms_norm_rows(x, ones, DIM, 1e-5)
        return int(np.argmax(o.linear(xn, 1, DIM, head, VOCAB)))

    pos = PROMPT
    for _ in range(args.warmup):
        token(pos, o.gen_normal_f32(0, 2000000 + pos, 0.02, DIM))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        token(pos, o.gen_normal_f32(0, 2000000 + pos, 0.02, DIM))
        pos += 1
    dt = time.perf_counter() - t0
    rate = args.steps / dt
    sample = (f"{args.steps} tokens (after {args.warmup} warm-up), each 26 layer steps + LM head at context "
              f"{PROMPT}..{pos}, f32 weights, {threads} threads (row-parallel linear, bit-identical to serial)")
    line = {"metric": METRIC, "value": rate, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 / rate, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "layers": LAYERS, "dim": DIM, "vocab": VOCAB, "window": WINDOW},
            "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def prompt_ids(seed: int, n: int) -> np.ndarray:
    """Seeded uniform token ids in [0, VOCAB) (splitmix64 counter hash)."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15) + np.arange(1, n + 1, dtype=np.uint64) * np.uint64(
            0xD1B54A32D192ED03)
        z ^= z >> np.uint64(30)
        z *= np.uint64(0xBF58476D1CE4E5B9)
        z ^= z >> np.uint64(27)
        z *= np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    return ((z >> np.uint64(32)) * np.uint64(VOCAB) >> np.uint64(32)).astype(np.int32)


def traffic_from_profiles():
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemv_w13_26layer_decode.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("dram_bytes_per_launch"):
            try:
                return float(line.split("=")[1].split()[0])
            except (IndexError, ValueError):
                return None
    return None


MS_STREAMS = 8
MS_WORKLOAD = ("26-layer decoder, 8 independent streams per GPU, contexts uniform in [256, 4096) with the KV "
               "cache prefilled from N(0,1) bf16, greedy decode, tensor-core (tcgen05) GEMMs")


def run_multi_stream(V, ctx, args, rank, world, dist):
    """The multi-stream workload: 8 streams per GPU decoded together, every
    weight read once per step for all 8.  Returns the per-rank measurements."""
    o_ids = np.random.default_rng(1000 + rank)
    lens = [int(x) for x in o_ids.integers(256, 4096, MS_STREAMS)]
    kv = V.RollingKvCache(ctx, LAYERS, NKV, HD, WINDOW, n_streams=MS_STREAMS)
    for s, n in enumerate(lens):
        kv.stream(s).fill_random(n, 0, 5000000 + 100 * (rank * MS_STREAMS + s), 1.0)
    toks = [int(t) for t in o_ids.integers(0, VOCAB, MS_STREAMS)]
    pos = list(lens)
    out = ctx.model_generate_batch(kv, toks, pos, args.warmup)
    toks = [int(t) for t in out[-1]]
    pos = [p + args.warmup for p in pos]
    ctx.synchronize()
    steps = args.ms_steps
    if dist:
        dist.barrier()
    ctx.synchronize()
    launches0 = ctx.kernel_launches()
    ctx.record_event(4)
    tp = (C_SZ * MS_STREAMS)(*pos)
    ti = np.ascontiguousarray(toks, dtype=np.int32)
    V.lib().vox_model_generate_batch(ctx.h, kv.h, ti.ctypes.data_as(V.I32P), tp, steps, None)
    ctx.record_event(5)
    ctx.synchronize()
    ms = ctx.elapsed_ms(4, 5)
    launches = ctx.kernel_launches() - launches0
    ctx_mean = sum(lens) / MS_STREAMS + args.warmup + steps / 2
    # end to end: host ids in, host next ids out, per step
    pos = [p + steps for p in pos]
    if dist:
        dist.barrier()
    ctx.record_event(6)
    e2e_steps = min(steps, 64)
    for i in range(e2e_steps):
        nxt, _ = ctx.model_step_batch(kv, toks, [p + i for p in pos])
        toks = [int(t) for t in nxt]
    ctx.record_event(7)
    e2e_ms = ctx.elapsed_ms(6, 7) / e2e_steps
    kv.close()
    return {"ms": ms, "steps": steps, "launches": launches, "lens": lens, "ctx_mean": ctx_mean, "e2e_ms": e2e_ms}


def run_context(V, ctx, args, rank, dist, fill, steps):
    """Greedy decode from a cache pre-filled with `fill` generator tokens
    (N(0,1) rounded to bf16, stored f32) at positions fill.., timed on the
    device.  With fill = the window every step evicts the oldest token; the
    ring state of every layer is then checked against kv.rs:48-88 on
    indices.  Returns the per-rank measurements."""
    kv = V.RollingKvCache(ctx, LAYERS, NKV, HD, WINDOW)
    kv.fill_random(fill, 0, 5000000 + 7919 * rank, 1.0)
    tok = int(prompt_ids(rank + 77, 1)[0])
    out = ctx.model_generate(kv, tok, fill, args.warmup)
    tok, pos = int(out[-1]), fill + args.warmup
    ctx.synchronize()
    if dist:
        dist.barrier()
    launches0 = ctx.kernel_launches()
    ctx.record_event(8)
    V.lib().vox_model_generate(ctx.h, kv.h, tok, pos, steps, None)
    ctx.record_event(9)
    ctx.synchronize()
    ms = ctx.elapsed_ms(8, 9)
    launches = ctx.kernel_launches() - launches0
    n_app = args.warmup + steps
    want = (min(fill + n_app, WINDOW), (max(0, fill + n_app - WINDOW)) % WINDOW, max(0, fill + n_app - WINDOW))
    ring_ok = all(tuple(kv.device_state(l)) == want for l in range(LAYERS))
    ctx_a, ctx_b = min(pos, WINDOW), min(pos + steps, WINDOW)
    kv.close()
    return {"ms": ms, "steps": steps, "launches": launches, "context": [ctx_a, ctx_b], "ring_ok": ring_ok,
            "ring_state": list(want)}


PREFILL_FLOPS_PER_TOKEN = LAYER_WEIGHT_BYTES  # 2 FLOPs per bf16 weight (2 bytes) per token


def run_prefill(V, ctx, rank, dist, reps=3):
    """The 512-id prompt of the token-loop workload through vox_model_prefill
    (tensor-core passes) into an empty cache, timed on the device and by the
    host wall clock around the call (host ids in, the call returns when the
    cache is written); the same prompt as 512 token steps
    (vox_model_prefill_steps) once, for comparison.  Returns per-rank times."""
    kv = V.RollingKvCache(ctx, LAYERS, NKV, HD, WINDOW)
    prompt = prompt_ids(rank + 31, PROMPT)
    ctx.model_prefill(kv, prompt, 0)  # warm-up (tiles the weights once)
    dev, wall = [], []
    for _ in range(reps):
        kv.reset()
        ctx.synchronize()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        ctx.record_event(10)
        launches0 = ctx.kernel_launches()
        ctx.model_prefill(kv, prompt, 0)
        ctx.record_event(11)
        ctx.synchronize()
        wall.append((time.perf_counter() - t0) * 1e3)
        dev.append(ctx.elapsed_ms(10, 11))
        launches = ctx.kernel_launches() - launches0
    ok = all(tuple(kv.device_state(l)) == (PROMPT, 0, 0) for l in range(LAYERS))
    kv.reset()
    ctx.record_event(12)
    ctx.model_prefill_steps(kv, prompt, 0)
    ctx.record_event(13)
    ctx.synchronize()
    steps_ms = ctx.elapsed_ms(12, 13)
    kv.close()
    return {"ms": min(dev), "wall_ms": min(wall), "steps_ms": steps_ms, "launches": launches, "ring_ok": ok}


JOB_DECODE = 1024


def run_config1_job(V, ctx, rank, dist):
    """Config 1 as one job: the 512-id prompt (vox_model_prefill) then 1024 greedy
    steps (vox_model_generate) into an empty cache, timed on the device and by the
    host clock around the two calls (host ids in, the 1024 generated ids out)."""
    kv = V.RollingKvCache(ctx, LAYERS, NKV, HD, WINDOW)
    prompt = prompt_ids(rank + 53, PROMPT)
    ctx.model_prefill(kv, prompt, 0)  # warm-up of both graphs and passes
    ctx.model_generate(kv, int(prompt[-1]), PROMPT, 8)
    kv.reset()
    ctx.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    ctx.record_event(14)
    ctx.model_prefill(kv, prompt[:-1], 0)
    ctx.record_event(15)
    out = ctx.model_generate(kv, int(prompt[-1]), PROMPT - 1, JOB_DECODE)
    ctx.record_event(13)
    ctx.synchronize()
    wall = (time.perf_counter() - t0) * 1e3
    pre_ms, total_ms = ctx.elapsed_ms(14, 15), ctx.elapsed_ms(14, 13)
    ok = all(tuple(kv.device_state(l))[0] == PROMPT - 1 + JOB_DECODE for l in range(LAYERS))
    kv.close()
    return {"prefill_ms": pre_ms, "ms": total_ms, "wall_ms": wall, "tokens": int(out.size), "ring_ok": ok}


def context_object(run, t_max, world, peak, workload):
    steps = run["steps"]
    mean_ctx = sum(run["context"]) / 2
    gbs = step_bytes(int(mean_ctx)) / (t_max / steps / 1e3) / 1e9
    return {"metric": "decoder tokens/s (1 stream per GPU)", "value": steps * world / (t_max / 1e3),
            "unit": "tokens/s", "ms_per_step": t_max / steps, "steps": steps, "context": run["context"],
            "workload": workload, "bytes_per_step": step_bytes(int(mean_ctx)),
            "step_roofline": {"achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak},
            "gpu_launches": run["launches"]}


TP_CONTEXT = 2048
TP_WORKLOAD = ("26-layer decoder, batch 1, tensor parallel over all GPUs (q|k|v, w1|w3 and LM head "
               "column-sharded, o-proj and w2 row-sharded; the 3072-wide residual is all-reduced after "
               "o-proj and w2 by stores into the other GPUs' memory fused into the GEMVs), prefill of "
               "2048 random ids then greedy decode")


ENC_DIM, ENC_CHUNK, ENC_SECONDS = 1280, 1280, 10


def run_encoder(V, local, cpu_sample_s=2.0):
    """The encoder front end streaming synthetic 16 kHz audio (N(0, 0.1^2)) in
    80 ms chunks (1280 samples, one decoder position each): log-mel + the
    causal conv stem (128 mel bins -> dim 1280, weights ~N(0, 0.02) rounded to
    bf16), through the public host-buffer API, so every chunk's samples go
    host -> device and its positions device -> host.  Returns GPU and oracle
    (1 thread, a cpu_sample_s-second sample) timings per second of audio."""
    from oracle import oracle as o
    o.build()
    rng = np.random.default_rng(11)
    audio = (0.1 * rng.standard_normal(16000 * ENC_SECONDS)).astype(np.float32)
    w0 = o.bf16_to_f32(o.gen_normal_bf16(0, 7000, 0.02, ENC_DIM * 128 * 3))
    w1 = o.bf16_to_f32(o.gen_normal_bf16(0, 7001, 0.02, ENC_DIM * ENC_DIM * 3))
    b0 = o.gen_normal_f32(0, 7002, 0.02, ENC_DIM)
    b1 = o.gen_normal_f32(0, 7003, 0.02, ENC_DIM)

    def stream(mel, stem, n_samples):
        positions, done = 0, 0
        while done < n_samples:
            before = mel.frames()
            mel.feed(audio[done:done + ENC_CHUNK])
            frames, _ = mel.data(before, mel.frames() - before)
            positions += stem.process(frames).shape[0]
            done += ENC_CHUNK
        return positions

    mel, stem = V.MelCtx(0, device=local), V.ConvStemState(128, ENC_DIM, w0, b0, w1, b1, device=local)
    stream(mel, stem, 16000)  # warm-up second
    mel.close()
    stem.close()
    mel, stem = V.MelCtx(0, device=local), V.ConvStemState(128, ENC_DIM, w0, b0, w1, b1, device=local)
    t0 = time.perf_counter()
    n_pos = stream(mel, stem, audio.size)
    gpu_s = time.perf_counter() - t0
    launches = int(V.lib().vox_encoder_kernel_launches(mel.h, stem.h))
    mel.close()
    stem.close()
    o.set_threads(1)
    n_cpu = int(16000 * cpu_sample_s)
    omel, ostem = o.MelCtx(0), o.ConvStemState(128, ENC_DIM, w0, b0, w1, b1)
    t0 = time.perf_counter()
    stream(omel, ostem, n_cpu)
    cpu_s = time.perf_counter() - t0
    return {"audio_s": ENC_SECONDS, "gpu_s": gpu_s, "positions": n_pos, "launches": launches,
            "cpu_audio_s": cpu_sample_s, "cpu_s": cpu_s}


TP_PARITY_PROMPT, TP_PARITY_FORCED, TP_PARITY_GREEDY = 31, 4, 64


def tp_parity_reference(V, ctx):
    """The parity sequence on this rank's single-GPU Context (the same weights
    the tensor-parallel ranks hold): a 31-id prompt prefilled, 4
    teacher-forced steps with their logits, then 64 greedy steps."""
    ids = prompt_ids(4242, TP_PARITY_PROMPT + TP_PARITY_FORCED)
    kv = V.RollingKvCache(ctx, LAYERS, NKV, HD, WINDOW)
    ctx.model_prefill(kv, ids[:TP_PARITY_PROMPT], 0)
    logits, toks = [], []
    for i in range(TP_PARITY_FORCED):
        t, lg = ctx.model_step(kv, int(ids[TP_PARITY_PROMPT + i]), TP_PARITY_PROMPT + i, want_logits=True)
        logits.append(lg)
        toks.append(t)
    pos = TP_PARITY_PROMPT + TP_PARITY_FORCED
    toks += [int(x) for x in ctx.model_generate(kv, toks[-1], pos, TP_PARITY_GREEDY)]
    kv.close()
    return ids, logits, toks


def tp_parity_check(tp, ids, ref_logits, ref_toks):
    """The same sequence through the tensor-parallel decoder: this rank's
    logit slice against the reference's, and every token."""
    tp.reset()
    tp.prefill([int(i) for i in ids[:TP_PARITY_PROMPT]], 0)
    lo, hi = tp.shard.vocab_begin, tp.shard.vocab_begin + tp.shard.vocab_local
    diff, toks = 0.0, []
    for i in range(TP_PARITY_FORCED):
        t, lg = tp.step(int(ids[TP_PARITY_PROMPT + i]), TP_PARITY_PROMPT + i, want_logits=True)
        diff = max(diff, float(np.max(np.abs(lg.astype(np.float64) - ref_logits[i][lo:hi]))))
        toks.append(t)
    pos = TP_PARITY_PROMPT + TP_PARITY_FORCED
    toks += [int(x) for x in tp.generate(toks[-1], pos, TP_PARITY_GREEDY)]
    return diff, toks == ref_toks


def run_tensor_parallel(V, args, rank, world, local, dist, parity_ref=None):
    """One stream decoded by all ranks together; returns this rank's timings
    (and, given the single-GPU reference sequence, the parity result)."""
    cfg = V.DecoderConfig(dim=DIM, hidden_dim=HIDDEN, n_heads=NH, n_kv_heads=NKV, head_dim=HD,
                          sliding_window=WINDOW, norm_eps=1e-5, rope_theta=1e6)
    uid = V.share_tp_unique_id(rank)
    steps = args.tp_steps
    with V.TensorParallelDecoder(cfg, rank, world, uid, LAYERS, VOCAB, device=local,
                                 max_positions=TP_CONTEXT + args.warmup + steps + 8) as tp:
        tp.init_random(0, 0.02)
        tp.connect_peers()  # exchange over NVLink peer memory, fused into the GEMVs
        prompt = prompt_ids(0, TP_CONTEXT)  # the same ids on every rank
        tp.prefill(prompt, 0)
        pos = TP_CONTEXT
        toks = tp.generate(int(prompt[-1]), pos, args.warmup)
        pos += args.warmup
        dist.barrier()
        launches0 = tp.kernel_launches()
        tp.record_event(0)
        V.lib().vox_tp_generate(tp.h, int(toks[-1]), pos, steps, None)
        tp.record_event(1)
        ms = tp.elapsed_ms(0, 1)
        launches = tp.kernel_launches() - launches0
        parity = None
        if parity_ref is not None:
            parity = tp_parity_check(tp, *parity_ref)
    return {"ms": ms, "steps": steps, "launches": launches, "ctx": [pos, pos + steps], "parity": parity}


def run_ours(args):
    rank, world, local = dist_env()
    V = importlib.import_module("voxtral-rust_b200")
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    cfg = V.DecoderConfig(dim=DIM, hidden_dim=HIDDEN, n_heads=NH, n_kv_heads=NKV, head_dim=HD,
                          sliding_window=WINDOW, norm_eps=1e-5, rope_theta=1e6)
    total_pos = PROMPT + args.warmup + 2 * args.steps + 8
    total_pos = max(total_pos, 4096 + args.warmup + args.ms_steps + 72)
    total_pos = max(total_pos, WINDOW + args.warmup + args.ctx_steps + 8)
    ctx = V.Context(cfg, n_layers=LAYERS, vocab=VOCAB, device=local, max_positions=total_pos)
    ctx.init_random(seed=0, std=0.02)
    kv = V.RollingKvCache(ctx, LAYERS, NKV, HD, WINDOW)
    prompt = prompt_ids(rank, PROMPT)
    ctx.model_prefill(kv, prompt, 0)
    pos = PROMPT
    tok = int(prompt[-1])
    # warm-up (untimed)
    if args.warmup:
        toks = ctx.model_generate(kv, tok, pos, args.warmup)
        tok, pos = int(toks[-1]), pos + args.warmup
    ctx.synchronize()

    # ---- device-resident timed region ----
    clocks = NvmlClockSampler(local)
    clocks.start()
    if dist:
        dist.barrier()
    ctx.synchronize()
    ctx_len0 = min(pos, WINDOW)
    launches0 = ctx.kernel_launches()
    ctx.record_event(0)
    V.lib().vox_model_generate(ctx.h, kv.h, tok, pos, args.steps, None)
    ctx.record_event(1)
    ctx.synchronize()
    ms = ctx.elapsed_ms(0, 1)
    launches = ctx.kernel_launches() - launches0
    clk = clocks.stop()
    pos += args.steps
    ctx_len1 = min(pos, WINDOW)
    # the generate call advanced the device token; read it back through one step below
    # ---- end-to-end: host token in, host next token out, per step ----
    if dist:
        dist.barrier()
    ctx.record_event(2)
    cur = tok
    for i in range(args.steps):
        cur, _ = ctx.model_step(kv, cur, pos + i)
    ctx.record_event(3)
    e2e_ms = ctx.elapsed_ms(2, 3)
    pos += args.steps

    # ---- dominant kernel on its own (w1|w3 SwiGLU GEMV, one launch per layer) ----
    k_ms, k_bytes = ctx.profile_gemv(2, LAYERS * 4)

    long_run = None if args.ctx_steps == 0 else run_context(V, ctx, args, rank, dist, LONG_CONTEXT, args.ctx_steps)
    roll_run = None if args.ctx_steps == 0 else run_context(V, ctx, args, rank, dist, WINDOW, args.ctx_steps)
    pf_run = None if args.no_prefill else run_prefill(V, ctx, rank, dist)
    job_run = None if args.no_prefill else run_config1_job(V, ctx, rank, dist)
    ms_run = None if args.ms_steps == 0 else run_multi_stream(V, ctx, args, rank, world, dist)
    enc_run = None if args.no_encoder else run_encoder(V, local)
    tp_run = None
    if world > 1 and args.tp_steps > 0:
        parity_ref = tp_parity_reference(V, ctx)
        ctx.close()  # release the replica's memory first
        tp_run = run_tensor_parallel(V, args, rank, world, local, dist, parity_ref)

    t_max, e2e_max = ms, e2e_ms
    ms_max = ms_e2e_max = tp_max = long_max = roll_max = enc_max = pf_max = pf_wall_max = pf_steps_max = 0.0
    job_max = job_wall_max = job_pre_max = 0.0
    if job_run:
        job_max, job_wall_max, job_pre_max = job_run["ms"], job_run["wall_ms"], job_run["prefill_ms"]
    if pf_run:
        pf_max, pf_wall_max, pf_steps_max = pf_run["ms"], pf_run["wall_ms"], pf_run["steps_ms"]
    if enc_run:
        enc_max = enc_run["gpu_s"]
    if ms_run:
        ms_max, ms_e2e_max = ms_run["ms"], ms_run["e2e_ms"]
    if tp_run:
        tp_max = tp_run["ms"]
    if long_run:
        long_max, roll_max = long_run["ms"], roll_run["ms"]
    if dist:
        import torch
        t = torch.tensor([ms, e2e_ms, ms_max, ms_e2e_max, tp_max, long_max, roll_max, enc_max, pf_max, pf_wall_max,
                          pf_steps_max, job_max, job_wall_max, job_pre_max], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        (t_max, e2e_max, ms_max, ms_e2e_max, tp_max, long_max, roll_max, enc_max, pf_max, pf_wall_max,
         pf_steps_max, job_max, job_wall_max, job_pre_max) = (float(x) for x in t)
        if roll_run:
            ok = torch.tensor([1.0 if roll_run["ring_ok"] and long_run["ring_ok"] else 0.0])
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            roll_run["ring_ok"] = long_run["ring_ok"] = bool(ok.item() > 0)
        if tp_run and tp_run["parity"] is not None:
            d = torch.tensor([tp_run["parity"][0], 0.0 if tp_run["parity"][1] else 1.0], dtype=torch.float64)
            dist.all_reduce(d, op=dist.ReduceOp.MAX)
            tp_run["parity"] = (float(d[0]), bool(d[1] == 0.0))
    if rank != 0:
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    tokens = args.steps * world
    value = tokens / (t_max / 1e3)
    e2e = tokens / (e2e_max / 1e3)
    peak, peak_kind = peaks()
    achieved = k_bytes / (k_ms / 1e3) / 1e9
    mean_ctx = (ctx_len0 + ctx_len1) / 2
    step_gbs = step_bytes(int(mean_ctx)) / (t_max / args.steps / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "dim": DIM, "hidden": HIDDEN, "heads": f"{NH}/{NKV}",
                   "head_dim": HD, "vocab": VOCAB, "window": WINDOW, "weight_dtype": "bf16", "kv_dtype": "f32",
                   "streams_per_gpu": 1, "context": [ctx_len0, ctx_len1],
                   "l2": "inputs larger than L2: 6.86 GB of weights streamed per step",
                   "bytes_per_step": step_bytes(int(mean_ctx)), "parallelism": f"dp{world} (independent streams)"},
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 32, "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "gemv_kernel (w1|w3 SwiGLU, 18432 x 3072 bf16)",
                     "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic_from_profiles(),
                     "algorithmic_bytes_per_launch": k_bytes, "launch_ms": k_ms},
        "step_roofline": {"achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak},
        "clocks": clk,
    }
    if long_run:
        line["long_context"] = context_object(
            long_run, long_max, world, peak,
            f"as the headline line, cache pre-filled to {LONG_CONTEXT} tokens (the end context of the "
            f"512 + 1024-step run), greedy decode")
        line["rolling"] = context_object(
            roll_run, roll_max, world, peak,
            f"rolling-window stress: cache pre-filled to the full {WINDOW}-token window, greedy decode, "
            f"every step evicts the oldest token (ring index arithmetic, no copy)")
        line["rolling"]["ring_state_after"] = {"len_tokens": roll_run["ring_state"][0],
                                               "start": roll_run["ring_state"][1],
                                               "pos_offset": roll_run["ring_state"][2],
                                               "matches_kv_rs_index_rule": roll_run["ring_ok"]}
    if pf_run:
        flops = PREFILL_FLOPS_PER_TOKEN * LAYERS * PROMPT
        tflops = flops / (pf_max / 1e3) / 1e12
        tpeak, tpeak_kind = tensor_peak()
        line["prefill"] = {
            "metric": "prompt prefill tokens/s (tensor-core passes)", "value": PROMPT * world / (pf_max / 1e3),
            "unit": "tokens/s", "ms": pf_max, "prompt_tokens": PROMPT, "gpu_launches": pf_run["launches"],
            "workload": (f"the {PROMPT}-id prompt of the token-loop workload into an empty cache, 26 layers: "
                         f"vox_model_prefill, one pass of dense tcgen05 GEMMs over all {PROMPT} tokens "
                         f"(activations as bf16 hi + lo parts), causal attention on tcgen05, ring append"),
            "e2e": {"value": PROMPT * world / (pf_wall_max / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * PROMPT, "d2h_bytes_per_step": 4},
            "token_steps_ms": pf_steps_max, "speedup_vs_token_steps": pf_steps_max / pf_max,
            "ring_state_ok": pf_run["ring_ok"],
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": tpeak, "peak_kind": tpeak_kind,
                         "unit": "TFLOP/s", "frac": tflops / tpeak,
                         "flops": flops, "note": "algorithmic FLOPs of the 26 layers' linears (2 per weight per "
                                                 "token); the hi/lo split doubles the tensor-core work"}}
    if job_run:
        line["config1_job"] = {
            "metric": "config 1 job: generated tokens/s (512-id prompt prefilled, then 1024 greedy steps)",
            "value": JOB_DECODE * world / (job_max / 1e3), "unit": "tokens/s", "ms": job_max,
            "prefill_ms": job_pre_max, "decode_ms": job_max - job_pre_max,
            "workload": (f"per GPU: the {PROMPT}-id prompt of config 1 (positions 0..{PROMPT - 2} through "
                         f"vox_model_prefill, the last id starts the decode) then {JOB_DECODE} greedy steps "
                         f"(vox_model_generate) from an empty 26-layer cache, window {WINDOW}"),
            "e2e": {"value": JOB_DECODE * world / (job_wall_max / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * PROMPT, "d2h_bytes_per_step": 4 * JOB_DECODE},
            "ring_state_ok": job_run["ring_ok"]}
    if enc_run:
        chunks = enc_run["audio_s"] * 16000 // ENC_CHUNK
        line["encoder"] = {
            "metric": "encoder front end: audio seconds processed per second (log-mel + conv stem)",
            "value": enc_run["audio_s"] * world / enc_max, "unit": "audio s/s", "streams": world,
            "workload": (f"{enc_run['audio_s']} s of 16 kHz synthetic audio per GPU in 80 ms chunks (1280 samples): "
                         f"MelCtx feed (128 bins) then ConvStemState process (conv0 128->{ENC_DIM}, conv1 "
                         f"{ENC_DIM}->{ENC_DIM} stride 2, GELU), host buffers in and out"),
            "ms_per_chunk": enc_max * 1e3 / chunks, "positions_per_stream": enc_run["positions"],
            "gpu_launches": enc_run["launches"],
            "e2e": {"value": enc_run["audio_s"] * world / enc_max, "unit": "audio s/s",
                    "h2d_bytes_per_step": ENC_CHUNK * 4 + 8 * 128 * 4, "d2h_bytes_per_step": 8 * 128 * 4 + 4 * ENC_DIM * 4},
            "cpu_baseline": {"value": enc_run["cpu_audio_s"] / enc_run["cpu_s"], "unit": "audio s/s", "cores": 1,
                             "kind": "port", "sample": f"{enc_run['cpu_audio_s']} s of the same audio, same chunks, "
                                                       f"oracle MelCtx + ConvStemState, 1 thread"}}
    if ms_run:
        n_tok = ms_run["steps"] * MS_STREAMS * world
        ms_bytes = (LAYERS * LAYER_WEIGHT_BYTES + HEAD_BYTES + MS_STREAMS * EMBED_ROW_BYTES +
                    LAYERS * KV_BYTES_PER_TOKEN_LAYER * MS_STREAMS * ms_run["ctx_mean"])
        ms_gbs = ms_bytes / (ms_max / ms_run["steps"] / 1e3) / 1e9
        line["multi_stream"] = {
            "metric": "decoder tokens/s (8 streams per GPU)", "value": n_tok / (ms_max / 1e3), "unit": "tokens/s",
            "streams_per_gpu": MS_STREAMS, "total_streams": MS_STREAMS * world, "steps": ms_run["steps"],
            "ms_per_step": ms_max / ms_run["steps"], "workload": MS_WORKLOAD,
            "contexts_rank0": ms_run["lens"], "bytes_per_step": int(ms_bytes),
            "step_roofline": {"achieved": ms_gbs, "peak": peak, "unit": "GB/s", "frac": ms_gbs / peak},
            "e2e": {"value": MS_STREAMS * world / (ms_e2e_max / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 40 * MS_STREAMS, "d2h_bytes_per_step": 4 * MS_STREAMS},
            "gpu_launches": ms_run["launches"]}
    if tp_run:
        tp_steps = tp_run["steps"]
        tp_ctx = sum(tp_run["ctx"]) / 2
        tp_bytes = step_bytes(int(tp_ctx))  # weights + KV of the whole model, split over the ranks
        tp_gbs = tp_bytes / (tp_max / tp_steps / 1e3) / 1e9
        line["tensor_parallel"] = {
            "metric": "decoder tokens/s (1 stream, tensor parallel)", "tp": world,
            "value": tp_steps / (tp_max / 1e3), "unit": "tokens/s", "ms_per_token": tp_max / tp_steps,
            "steps": tp_steps, "workload": TP_WORKLOAD, "context": tp_run["ctx"],
            "step_roofline": {"achieved": tp_gbs, "peak": peak * world, "unit": "GB/s",
                              "frac": tp_gbs / (peak * world), "note": "aggregate HBM of all ranks"},
            "gpu_launches": tp_run["launches"]}
        if tp_run["parity"] is not None:
            line["tensor_parallel"]["parity"] = {
                "against": "the single-GPU Context on the same weights (each rank's logit slice)",
                "tokens_identical": tp_run["parity"][1], "n_steps": TP_PARITY_FORCED + TP_PARITY_GREEDY,
                "teacher_forced_steps": TP_PARITY_FORCED, "greedy_steps": TP_PARITY_GREEDY,
                "max_abs_logit_diff": tp_run["parity"][0]}
    if world == 1 and not args.no_cpu:
        rate, sample = cpu_token_rate(1, args.cpu_layer_steps, 1)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": 1, "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--cpu-layer-steps", type=int, default=24)
    ap.add_argument("--no-encoder", action="store_true", help="skip the encoder front-end run")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prompt prefill run")
    ap.add_argument("--ctx-steps", type=int, default=256,
                    help="greedy steps of the long-context (1536) and full-window rolling runs (0 skips them)")
    ap.add_argument("--ms-steps", type=int, default=512,
                    help="greedy steps of the 8-streams-per-GPU run (0 skips it)")
    ap.add_argument("--tp-steps", type=int, default=1024,
                    help="greedy steps of the tensor-parallel run when N > 1 (0 skips it)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
