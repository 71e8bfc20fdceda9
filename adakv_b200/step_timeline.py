"""Per-phase timeline of the one-kernel decode step (diagnostic).

    python -m adakv_b200.step_timeline [--ctx 131072] [--heads 32 8] [--warm]
                                       [--cluster N] [--iters 20]

Runs the persistent decode-step kernel (``ADAKV_KNOB_STEP_PATH`` = 2) on a
seeded synthetic cfg1 case with the test-only timeline flag
(``ADAKV_KNOB_FLAGS`` bit 1) set, reads the per-CTA globaltimer stamps through
``adakv_debug_timeline`` and prints, per phase boundary, the min / median /
max over CTAs (median over iterations) in microseconds from the first CTA's
start.  ``--warm`` steps back to back (no L2 flush between steps);
otherwise a 256 MB buffer is written and read before each timed step.
``--cluster`` caps the selection phase's thread-block cluster (0: 8).
Stamps of the selection phase (``B_*``) are taken over the CTAs that select.
"""
from __future__ import annotations

import argparse
import ctypes

import numpy as np

# stamp slot -> name, in the order the kernel writes them
SLOTS = {
    0: "start", 8: "A_first", 9: "A_last", 1: "A_done",
    10: "B_arrive", 19: "B_stats", 2: "B_row", 16: "B_pass2", 17: "B_sync2", 11: "B_Hpub",
    3: "B_budget", 20: "B_thresh", 21: "B_marked", 12: "B_sync3", 14: "B_select",
    18: "B_sync4", 4: "B_bitmap",
    5: "C_bitmaps", 22: "C_list", 13: "C_gather", 23: "C_comb", 6: "C_partial", 7: "end",
}
NSLOT = 24
MAX_CTAS = 256


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ctx", type=int, default=131072)
    ap.add_argument("--heads", type=int, nargs=2, default=[32, 8], metavar=("HQ", "HKV"))
    ap.add_argument("--warm", action="store_true")
    ap.add_argument("--cluster", type=int, default=0)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)

    import torch

    from adakv_b200 import _lib
    from adakv_b200.batch import BatchedDecoder
    from adakv_b200.synth import make_decode_case

    Hq, Hkv = args.heads
    S = args.ctx
    case = make_decode_case(0, 1, Hq, Hkv, 128, S, 16, "bf16")
    _lib.debug_knob(_lib.KNOB_STEP_CLUSTER, args.cluster)
    _lib.debug_knob(_lib.KNOB_STEP_PATH, 2)
    try:
        dec = BatchedDecoder(1, Hq, Hkv, 128, 16, S, torch.bfloat16, "cuda", avg_budget=64, k_max=512)
        dec.load(torch.from_numpy(case.K).cuda().bfloat16(), torch.from_numpy(case.V).cuda().bfloat16(), [S])
        q = torch.from_numpy(case.q).cuda().bfloat16()
        kt = torch.randn(1, Hkv, 1, 128, device="cuda").bfloat16()
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        for _ in range(5):
            dec.step(q, k_new=kt, v_new=kt, advance=False)
        torch.cuda.synchronize()
        if dec.last_path() != 2:
            raise SystemExit("the one-kernel step does not apply to this geometry")
        _lib.debug_knob(_lib.KNOB_FLAGS, 2)
        rows = []
        for _ in range(args.iters + 5):
            if args.warm:
                for _ in range(3):
                    dec.step(q, k_new=kt, v_new=kt, advance=False)
            else:
                flush.zero_()
                flush.sum(dtype=torch.int64)
            dec.step(q, k_new=kt, v_new=kt, advance=False)
            buf = (ctypes.c_uint64 * (MAX_CTAS * NSLOT))()
            _lib.check(_lib.lib().adakv_debug_timeline(dec._geo, dec.workspace.data_ptr(), dec.ws_bytes,
                                                       buf, MAX_CTAS, _lib.stream_ptr(dec.device)))
            rows.append(np.frombuffer(buf, dtype=np.uint64).reshape(MAX_CTAS, NSLOT).astype(np.int64))
        status = dec.status()
    finally:
        _lib.debug_knob(_lib.KNOB_FLAGS, 0)
        _lib.debug_knob(_lib.KNOB_STEP_PATH, 0)
        _lib.debug_knob(_lib.KNOB_STEP_CLUSTER, 0)

    T = np.stack(rows[5:])                     # [iteration, cta, slot]
    grid = int((T[-1, :, 0] > 0).sum())         # CTAs that ran
    sel = int((T[-1, :, 2] > 0).sum())          # CTAs that selected
    T = T[:, :grid]
    rel = (T - T[:, :, 0].min(axis=1)[:, None, None]) / 1000.0
    print(f"{'warm' if args.warm else 'cold'} step, ctx {S}, {Hq}/{Hkv} heads: grid {grid} CTAs, "
          f"{sel} selecting; microseconds from the first CTA start (median over {args.iters} steps)")
    print(f"  {'stamp':10s} {'min':>8s} {'median':>8s} {'max':>8s}")
    for slot, name in SLOTS.items():
        x = rel[:, :sel if name.startswith("B_") else grid, slot]
        print(f"  {name:10s} {np.median(x.min(1)):8.2f} {np.median(np.median(x, 1)):8.2f} "
              f"{np.median(x.max(1)):8.2f}")
    print("status", status)


if __name__ == "__main__":
    main()
