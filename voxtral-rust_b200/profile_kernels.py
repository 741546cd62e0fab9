"""Times one of the token step's kernels on its own (small device footprint,
suitable for an ncu capture).

    python voxtral-rust_b200/profile_kernels.py --which w13 --layers 2 --launches 8
    python voxtral-rust_b200/profile_kernels.py --which step --layers 2 --steps 8

--which o|w13|w2|head runs vox_profile_gemv (launches cycle over the layers);
--which encoder streams `--seconds` of synthetic 16 kHz audio through the
encoder front end (log-mel + conv stem, 128 mel bins -> dim 1280) in 80 ms
chunks; --which step runs whole token steps of a full-width model with `--layers`
layers and the 131072-token vocabulary; --which batch runs multi-stream steps
of `--streams` streams (contexts uniform in [256, 4096)); --which
bo|bw13|bw2|bhead|bqkv times one multi-stream tensor-core GEMM, --which
bchain the o-proj, w1|w3, w2, q|k|v chain as one launch; --which prefill
runs `--steps` prefills of `--context` tokens into an empty cache of a
full-width model with `--layers` layers (vocabulary 131072).
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--which", default="w13",
                    choices=["o", "w13", "w2", "head", "step", "batch", "bo", "bw13", "bw2", "bhead", "bqkv",
                             "bchain", "encoder", "prefill"])
    ap.add_argument("--seconds", type=float, default=2.0)
    ap.add_argument("--streams", type=int, default=8)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--launches", type=int, default=8)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--context", type=int, default=512)
    ap.add_argument("--fill", action="store_true",
                    help="step: fill the cache from the generator instead of prefilling tokens")
    ap.add_argument("--mode", type=int, default=0, help="0 auto, 1 per-layer kernels, 2 persistent kernel")
    args = ap.parse_args()
    V = importlib.import_module("voxtral-rust_b200")
    if args.which == "encoder":
        import time

        import numpy as np
        rng = np.random.default_rng(11)
        dim = 1280
        w0 = (0.02 * rng.standard_normal(dim * 128 * 3)).astype(np.float32)
        w1 = (0.02 * rng.standard_normal(dim * dim * 3)).astype(np.float32)
        b0 = (0.02 * rng.standard_normal(dim)).astype(np.float32)
        b1 = (0.02 * rng.standard_normal(dim)).astype(np.float32)
        audio = (0.1 * rng.standard_normal(int(16000 * args.seconds))).astype(np.float32)
        mel, stem = V.MelCtx(0), V.ConvStemState(128, dim, w0, b0, w1, b1)
        t0, n_pos = time.perf_counter(), 0
        for i in range(0, audio.size, 1280):
            before = mel.frames()
            mel.feed(audio[i:i + 1280])
            frames, _ = mel.data(before, mel.frames() - before)
            n_pos += stem.process(frames).shape[0]
        dt = time.perf_counter() - t0
        print(f"encoder: {args.seconds:.1f} s of audio in {dt * 1e3:.1f} ms, {n_pos} positions")
        return
    cfg = V.DecoderConfig(dim=3072, hidden_dim=9216, n_heads=32, n_kv_heads=8, head_dim=128,
                          sliding_window=8192, norm_eps=1e-5, rope_theta=1e6)
    batched = args.which.startswith("b")
    vocab = 131072 if args.which in ("head", "step", "prefill") or batched else 0
    with V.Context(cfg, n_layers=args.layers, vocab=vocab, step_mode=args.mode) as ctx:
        ctx.init_random(0, 0.02)
        if args.which == "step":
            kv = V.RollingKvCache(ctx, args.layers, 8, 128, 8192)
            if args.fill:
                kv.fill_random(args.context, 0, 5000000, 1.0)
            else:
                ctx.model_prefill(kv, [i % vocab for i in range(args.context)], 0)
            ctx.synchronize()
            ctx.record_event(0)
            ctx.model_generate(kv, 1, args.context, args.steps)
            ctx.record_event(1)
            ms = ctx.elapsed_ms(0, 1) / args.steps
            print(f"step: {ms * 1e3:.1f} us per token ({args.layers} layers + LM head)")
            return
        if args.which == "prefill":
            kv = V.RollingKvCache(ctx, args.layers, 8, 128, 8192)
            ids = [(7919 * i) % vocab for i in range(args.context)]
            best = None
            for _ in range(args.steps):
                kv.reset()
                ctx.synchronize()
                ctx.record_event(0)
                ctx.model_prefill(kv, ids, 0)
                ctx.record_event(1)
                ms = ctx.elapsed_ms(0, 1)
                best = ms if best is None else min(best, ms)
            print(f"prefill: {args.context} tokens through {args.layers} layers in {best:.3f} ms")
            return
        if args.which == "batch":
            import numpy as np
            rng = np.random.default_rng(1000)
            lens = [int(x) for x in rng.integers(256, 4096, args.streams)]
            kv = V.RollingKvCache(ctx, args.layers, 8, 128, 8192, n_streams=args.streams)
            for s, n in enumerate(lens):
                kv.stream(s).fill_random(n, 0, 5000000 + 100 * s, 1.0)
            toks = [int(x) for x in rng.integers(0, vocab, args.streams)]
            ctx.model_generate_batch(kv, toks, lens, 2)  # warm-up
            pos = [n + 2 for n in lens]
            ctx.synchronize()
            ctx.record_event(0)
            ctx.model_generate_batch(kv, toks, pos, args.steps)
            ctx.record_event(1)
            ms = ctx.elapsed_ms(0, 1) / args.steps
            print(f"batch step: {ms * 1e3:.1f} us per step of {args.streams} streams "
                  f"({args.layers} layers + LM head), contexts {lens}")
            return
        if batched:
            which = {"bo": 1, "bw13": 2, "bw2": 3, "bhead": 4, "bqkv": 5, "bchain": 6}[args.which]
            ctx.profile_bgemm(which, args.streams, 2)  # warm-up
            ms, nbytes = ctx.profile_bgemm(which, args.streams, args.launches)
            print(f"{args.which}: {ms * 1e3:.2f} us per launch, {nbytes} B, {nbytes / ms / 1e6:.1f} GB/s")
            return
        which = {"o": 1, "w13": 2, "w2": 3, "head": 4}[args.which]
        ctx.profile_gemv(which, 2)  # warm-up
        ms, nbytes = ctx.profile_gemv(which, args.launches)
        print(f"{args.which}: {ms * 1e3:.2f} us per launch, {nbytes} B, {nbytes / ms / 1e6:.1f} GB/s")


if __name__ == "__main__":
    main()
