"""Per-phase timeline of one decode step (configs[1] geometry).

    PRISM_B200_PERSIST=1 python prism-inference_b200/phase_trace.py [--tokens N]
    PRISM_B200_TRACE=1 python prism-inference_b200/phase_trace.py [--tokens N]

Builds the random-init configs[1] model as bench.py does and ingests N
tokens.  Persistent step: runs prism_b200_model_step_timings three times
and prints, per kind of phase, CTA 0's average barrier wait and work time,
and for projection phases the split of the work into input staging, tile
bookkeeping, tile arrival, integer dots, row chains and the rest (from the
kernel's SM-clock stamps, converted at the nominal 1965 MHz).

Kernel-sequence step (PRISM_B200_TRACE=1): runs decode steps and prints,
per kind of launch, the average gap from the previous launch's last CTA
exit to this launch's grid dependency release, then CTA 0's times to stage
the input, see its first tile resident, finish its dots and chains and
exit, and the time to the last CTA's exit.
"""
import argparse
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import prism_b200 as pb  # noqa: E402
import qwen35  # noqa: E402

SM_MHZ = 1965.0


def phase_names(cfg):
    names = ["embed"]
    for l in range(cfg.layers):
        names += (["attn_group", "attention", "attn_out"] if cfg.is_full(l)
                  else ["gdn_group", "gdn", "gdn_out"]) + ["ffn_pair", "ffn_down"]
    return names + ["lm_head"]


def launch_names(cfg):
    names = []
    for l in range(cfg.layers):
        names += (["attn_group", "attention", "attn_out"] if cfg.is_full(l)
                  else ["gdn_group", "gdn", "gdn_out"]) + ["ffn_pair", "ffn_down"]
    return names + ["lm_head"]


def sequence_trace(args):
    cfg = qwen35.CONFIG1
    ex = pb.ProjectionExecutor(0)
    model = qwen35.Qwen35Model(ex, cfg)
    model.load(qwen35.synthetic_weights(cfg, seed=0))
    for t in qwen35.prompt_tokens(cfg, args.tokens, seed=1):
        model.evaluate(t, logits=False)
    L = model.L
    L.prism_b200_model_phase_trace.restype = ctypes.c_int64
    L.prism_b200_model_phase_trace.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    names = launch_names(cfg)
    agg = {}
    for _ in range(3):
        model.evaluate(int(qwen35.prompt_tokens(cfg, 1, seed=2)[0]), logits=False)
        buf = np.zeros(8 * len(names), np.uint64)
        n = L.prism_b200_model_phase_trace(model.h, buf.ctypes.data, buf.size)
        t = buf[:n].astype(np.int64).reshape(-1, 8)
        print("step: first launch entry to last exit %.1f us, %d launches" %
              ((t[-1, 7] - t[0, 0]) / 1e3, len(t)))
        for p in range(len(t)):
            r = t[p]
            gap = (r[1] - t[p - 1, 7]) / 1e3 if p else 0.0
            if r[2]:   # projections: [2] staged .. [5] chains
                seg = [(r[2] - r[1]) / 1e3, (r[3] - r[2]) / 1e3, (r[4] - r[3]) / 1e3,
                       (r[5] - r[4]) / 1e3, (r[6] - r[5]) / 1e3]
            else:
                seg = [0.0, 0.0, 0.0, 0.0, (r[6] - r[1]) / 1e3]
            tail = (r[7] - r[6]) / 1e3
            a = agg.setdefault(names[p], np.zeros(9))
            a += [1, gap, (r[1] - r[0]) / 1e3] + seg + [tail]
    print("%-10s %3s %6s %7s | %6s %6s %6s %6s %6s | %6s (avg us)" %
          ("launch", "n", "gap", "early", "stage", "tile", "dots", "chain", "cta0", "tail"))
    tot = 0.0
    for k, a in agg.items():
        c = a[0]
        tot += (a[1] + sum(a[3:])) / 3
        print("%-10s %3d %6.2f %7.2f | %6.2f %6.2f %6.2f %6.2f %6.2f | %6.2f  total %7.1f" %
              (k, c / 3, a[1] / c, a[2] / c, a[3] / c, a[4] / c, a[5] / c, a[6] / c, a[7] / c,
               a[8] / c, (a[1] + sum(a[3:])) / 3))
    print("sum of gap + release-to-exit over one step: %.1f us" % tot)
    model.close()
    ex.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32)
    args = ap.parse_args()
    if os.environ.get("PRISM_B200_PERSIST") != "1":
        if os.environ.get("PRISM_B200_TRACE") != "1":
            raise SystemExit("set PRISM_B200_PERSIST=1 or PRISM_B200_TRACE=1")
        return sequence_trace(args)
    cfg = qwen35.CONFIG1
    ex = pb.ProjectionExecutor(0)
    model = qwen35.Qwen35Model(ex, cfg)
    model.load(qwen35.synthetic_weights(cfg, seed=0))
    for t in qwen35.prompt_tokens(cfg, args.tokens, seed=1):
        model.evaluate(t, logits=False)
    L = model.L
    L.prism_b200_model_phase_trace.restype = ctypes.c_int64
    L.prism_b200_model_phase_trace.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    for _ in range(3):
        model.step_timings()
        buf = np.zeros(8 * 256, np.uint64)
        n = L.prism_b200_model_phase_trace(model.h, buf.ctypes.data, buf.size)
        t = buf[:n].astype(np.int64).reshape(-1, 8)
        print("step %.1f us, %d phases" % ((t[-1, 7] - t[0, 0]) / 1e3, len(t)))
    names = phase_names(cfg)
    agg = {}
    for p in range(len(t)):
        r = t[p]
        wait = (r[0] - t[p - 1, 7]) / 1e3 if p else 0.0
        work = (r[7] - r[0]) / 1e3
        c = [r[5], r[1], r[6], r[2], r[3], r[4]]
        sub = [(c[i] - c[i - 1]) / SM_MHZ if r[1] else 0.0 for i in range(1, 6)]
        tail = work - (c[5] - c[0]) / SM_MHZ if r[1] else 0.0
        a = agg.setdefault(names[p], np.zeros(9))
        a += [1, wait, work] + sub + [tail]
    print("%-10s %3s %8s %7s | %6s %6s %6s %6s %6s %6s (avg us)" %
          ("phase", "n", "barrier", "work", "stage", "prep", "wait", "dots", "chain", "tail"))
    for k, a in agg.items():
        c = a[0]
        print("%-10s %3d %8.2f %7.2f | %6.2f %6.2f %6.2f %6.2f %6.2f %6.2f  total %7.1f" %
              (k, c, a[1] / c, a[2] / c, a[3] / c, a[4] / c, a[5] / c, a[6] / c, a[7] / c,
               a[8] / c, a[1] + a[2]))
    model.close()
    ex.close()


if __name__ == "__main__":
    main()
