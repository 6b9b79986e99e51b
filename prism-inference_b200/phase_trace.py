"""Per-phase timeline of one persistent decode step (configs[1] geometry).

    PRISM_B200_PERSIST=1 python prism-inference_b200/phase_trace.py [--tokens N]

Builds the random-init configs[1] model as bench.py does, ingests N tokens,
runs prism_b200_model_step_timings three times on the persistent step and
prints, per kind of phase, CTA 0's average barrier wait and work time, and
for projection phases the split of the work into input staging, tile
bookkeeping, tile arrival, integer dots, row chains and the rest (from the
kernel's SM-clock stamps, converted at the nominal 1965 MHz).
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32)
    args = ap.parse_args()
    if os.environ.get("PRISM_B200_PERSIST") != "1":
        raise SystemExit("set PRISM_B200_PERSIST=1 (the trace exists for the persistent step)")
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
