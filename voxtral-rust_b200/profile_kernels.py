"""Times one of the token step's kernels on its own (small device footprint,
suitable for an ncu capture).

    python voxtral-rust_b200/profile_kernels.py --which w13 --layers 2 --launches 8
    python voxtral-rust_b200/profile_kernels.py --which step --layers 2 --steps 8

--which o|w13|w2|head runs vox_profile_gemv (launches cycle over the layers);
--which step runs whole token steps of a full-width model with `--layers`
layers and the 131072-token vocabulary; --which batch runs multi-stream steps
of `--streams` streams (contexts uniform in [256, 4096)); --which
bo|bw13|bw2|bhead|bqkv times one multi-stream tensor-core GEMM, --which
bchain the o-proj, w1|w3, w2, q|k|v chain as one launch.
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
                             "bchain"])
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
    cfg = V.DecoderConfig(dim=3072, hidden_dim=9216, n_heads=32, n_kv_heads=8, head_dim=128,
                          sliding_window=8192, norm_eps=1e-5, rope_theta=1e6)
    batched = args.which.startswith("b")
    vocab = 131072 if args.which in ("head", "step") or batched else 0
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
