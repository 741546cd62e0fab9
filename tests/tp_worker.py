"""One rank of the tensor-parallel parity check (run by tests/test_gpu_tp.py
under torch.distributed.run, one process per GPU, 2, 4 or 8 ranks): this
rank's logit slice and the greedy tokens against the oracle's full model."""
import argparse
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from tests.vox_testlib import FULL, assert_logits_close, config_dict, oracle_model, top2_margin, vox  # noqa: E402

# 8 kv heads (4 q heads each, the model's group) so that every case shards 2, 4 and 8 ways
SMALL = config_dict(dim=256, hidden_dim=512, n_heads=32, n_kv_heads=8, head_dim=32, sliding_window=64,
                    rope_theta=1e4)
# (config, layers, vocab, checked steps, prefilled tokens before them)
CASES = {
    # small shapes, window 64 so the ring evicts during the run
    "small": (SMALL, 2, 1024, 80, 0),
    "full": (FULL, 2, 8192, 6, 0),
    # past the prompt, the checked steps cross the context at which attention
    # switches from one cluster per kv head to the split-K kernel (3584 tokens)
    "switch": (dict(SMALL, sliding_window=8192), 2, 1024, 8, 3578),
}


def leave(V, dist, rank, world, local):
    """Failure detection with the peer-memory exchange: every rank runs three
    steps, then the last rank stops calling (it stays alive, between steps,
    with nothing in flight).  The others' next step must end with
    VOX_ERR_DEVICE_TIMEOUT through the kernels' bounded peer waits, and the
    context must refuse further steps.  NCCL is not used here."""
    import time
    c = SMALL
    uid = V.share_tp_unique_id(rank)
    failures = []
    with V.TensorParallelDecoder(V.DecoderConfig(**c), rank, world, uid, 2, 1024, device=local) as tp:
        tp.init_random(0, 0.02)
        tp.connect_peers()
        tp.set_timeout_ms(20000)
        for p in range(3):
            tp.step(5 + p, p)
        if rank != world - 1:
            t0 = time.time()
            try:
                tp.step(9, 3)
                failures.append("the step after a rank stopped did not fail")
            except V.VoxError as e:
                if e.code != V.ERR_DEVICE_TIMEOUT:
                    failures.append(f"unexpected error {e}")
            if time.time() - t0 > 15:
                failures.append(f"the failed step took {time.time() - t0:.1f} s")
            try:
                tp.step(9, 4)
                failures.append("a broken context accepted another step")
            except V.VoxError as e:
                if e.code != V.ERR_DEVICE_TIMEOUT:
                    failures.append(f"unexpected error {e}")
        dist.barrier()  # the stopped rank waits here, alive, until the others are done
    print(f"rank {rank}: case leave (peer), failures {failures}", flush=True)
    return failures


def main():
    import datetime

    import torch.distributed as dist
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="small", choices=sorted(CASES) + ["leave"])
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="peer: stores into the other GPUs' memory fused into the GEMVs; nccl: all-reduce")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    V = vox()
    if args.case == "leave":
        failures = leave(V, dist, rank, world, local)
        dist.barrier()
        dist.destroy_process_group()
        sys.exit(1 if failures else 0)
    from oracle import oracle as o
    o.build()
    o.set_threads(max(1, (os.cpu_count() or 2) // world))
    c, n_layers, vocab, n_steps, n_pre = CASES[args.case]
    uid = V.share_tp_unique_id(rank)
    seed = 0
    m = oracle_model(o, c, n_layers, vocab, seed)
    oc = o.RollingKvCache(n_layers, c["n_kv_heads"], c["head_dim"], c["sliding_window"])
    ids = o.gen_uniform_ids(seed, 3000000, vocab, n_pre + n_steps)
    failures = []
    with V.TensorParallelDecoder(V.DecoderConfig(**c), rank, world, uid, n_layers, vocab, device=local) as tp:
        tp.init_random(seed, 0.02)
        if args.exchange == "peer":
            tp.connect_peers()
        sh = tp.shard
        lo, hi = sh.vocab_begin, sh.vocab_begin + sh.vocab_local
        worst = 0.0
        if n_pre:
            tp.prefill([int(i) for i in ids[:n_pre]], 0)
            for p in range(n_pre):
                m.step(oc, int(ids[p]), p, want_logits=False)
        for p in range(n_pre, n_pre + n_steps):
            tok, logits = tp.step(int(ids[p]), p, want_logits=True)
            ref_logits, ref_tok = m.step(oc, int(ids[p]), p)
            try:
                worst = max(worst, assert_logits_close(logits, ref_logits[lo:hi], f"rank {rank} step {p}"))
                assert tok == ref_tok, f"step {p}: {tok} != {ref_tok} (margin {top2_margin(ref_logits):.3e})"
            except AssertionError as e:
                failures.append(str(e))
                break
        for l in range(n_layers):
            ln, start, off = tp.kv_state(l)
            want = (oc.layer_len_tokens(l), oc.layer_pos_offset(l))
            if (ln, off) != want:
                failures.append(f"layer {l}: ring state {(ln, off)} != {want}")
        # greedy continuation on the device against the oracle's
        pos = n_pre + n_steps
        tok0 = int(ids[-1])
        got = tp.generate(tok0, pos, 3)
        t = tok0
        for i in range(3):
            ref_logits, t = m.step(oc, t, pos + i)
            if got[i] != t:
                failures.append(f"greedy step {i}: {got[i]} != {t}")
                break
    print(f"rank {rank}: case {args.case} ({args.exchange}), worst logit diff {worst:.3e}, failures {failures}",
          flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(1 if failures else 0)


if __name__ == "__main__":
    main()
