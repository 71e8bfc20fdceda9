"""Device time of the sharded selection's kernels on one GPU (diagnostic).

    python -m adakv_b200.shard_timing [--world 2 4 8] [--policy adaptive] [--eager N]

Emulates the ranks of a sequence-sharded cfg4 step (one 1,048,576-token
sequence, 64 query / 8 KV heads, avg_budget 256, k_max 1024) on one device:
every shard's record is prepared and gathered in one process, then rank 0's
``adakv_shard_prep``, ``adakv_shard_clamp`` and ``adakv_shard_finish`` are
each timed as CUDA-graph replays of 20 launches (CUDA events on the
launching stream).  Score rows are seeded Gaussians.  ``--eager N`` instead
launches rank 0's prep N times without graphs (a short run for a profiler).
"""
from __future__ import annotations

import argparse

import torch

from .sharded import StatsSelector, shard_blocks, shard_range

Hq, Hkv, D, BS, S = 64, 8, 128, 16, 1 << 20


def _graph_us(fn, reps=20, rounds=5):
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(rounds):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000.0 / (reps * rounds)


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world", type=int, nargs="+", default=[2, 4, 8])
    ap.add_argument("--policy", choices=["adaptive", "fixed"], default="adaptive")
    ap.add_argument("--eager", type=int, default=0)
    args = ap.parse_args()
    kw = dict(avg_budget=256, k_min=2, k_max=1024, budget_policy=args.policy)
    nb = S // BS
    g = torch.Generator(device="cuda").manual_seed(3)
    sc = torch.randn((Hq, nb), device="cuda", generator=g) * 2.8
    for world in args.world:
        L = shard_blocks(nb, world)
        sels, rows = [], []
        for r in range(world):
            lo, n = shard_range(nb, world, r)
            sels.append(StatsSelector(S, Hq, Hkv, D, BS, torch.bfloat16, "cuda", lo, n, **kw))
            row = torch.zeros((Hq, L), dtype=torch.float32, device="cuda")
            row[:, :n] = sc[:, lo:lo + n]
            rows.append(row)
        st = sels[0]
        if args.eager:
            for _ in range(args.eager):
                st.prep(rows[0])
            torch.cuda.synchronize()
            print(f"world {world}: {args.eager} eager prep launches", flush=True)
            continue
        recs = torch.stack([s.prep(rows[r]).clone() for r, s in enumerate(sels)])
        ccs = None
        if st.adaptive:
            ccs = torch.stack([s.clamp(rows[r], recs).clone() for r, s in enumerate(sels)])
        tp = _graph_us(lambda: st.prep(rows[0]))
        tc = _graph_us(lambda: st.clamp(rows[0], recs)) if st.adaptive else 0.0
        tf = _graph_us(lambda: st.finish(recs, ccs, 0))
        print(f"world {world} ({args.policy}): prep {tp:.1f} us, clamp {tc:.1f} us, "
              f"finish {tf:.1f} us; record {st.record_bytes} B", flush=True)


if __name__ == "__main__":
    main()
