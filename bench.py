"""Benchmark of the B200 quantized decode hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|matvec|gdn|gemm|serve]

Prints ONE JSON line (rank 0).

Default workload (configs[1] of the benchmark configuration): batch-1
greedy decode of the random-init Qwen3.5-style hybrid decoder -- hidden
2560, 32 layers (every 4th gated full attention, the rest Gated DeltaNet),
16 q / 4 kv heads x 256, FFN 9216, vocab 151936 tied, all linear weights
TQ2_0 (codes uniform in {-1,0,+1}, fp16 scales U(0.01,0.05), seed 0).  A
512-token random prompt (seed 1) is ingested first (reported as prefill
tok/s), then K timed decode steps run device-driven: each step consumes the
previous step's greedy token.  Every step streams ~0.99 GB of weights and
state (>> 126 MB L2).

``--workload matvec`` is configs[0]: one TQ2_0 projection W 4096 x 4096 of
N(0,1) x quantized to Q8_K on the device, over 64 rotating device copies
of W (277 MB > L2).

``--workload gdn`` is configs[2] (GDN decode at B = 1/16/64, chunked
prefill of 4096 tokens); ``--workload gemm`` is configs[3] (2048-token
projections on the tensor cores, TQ2_0 and Q2_K, both FFN shapes);
``--workload serve`` is configs[4] (256 sequences per GPU with 8192-token
Q8_0 KV contexts, greedy batched decode).  ``--workload kvq`` times the
reference's rotated scalar KV attention (rsq4 / rsq4k3v records) at the
configs[1] head geometry over 2048-32768 positions, and the codec's encode.

``--impl reference`` times the reference's CPU arithmetic on the host
cores -- the C restatement in oracle/, since the Rust reference cannot be
built in this image -- on the same workload and prints the same line with
"impl": "reference".

Multi-GPU: batch-1 decode does not shard, so N ranks (torchrun) run N
independent replicas; `value` is the sum of all ranks' tokens over the
max-over-ranks device time.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "prism-inference_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

PROMPT = 512
DECODE_METRIC = "decode tok/s (batch 1)"
MATVEC_METRIC = "packed-matvec HBM GB/s (TQ2_0 x Q8_K, batch 1)"
MV_ROWS = MV_COLS = 4096
MV_COPIES = 64
MV_BYTES = MV_ROWS * (MV_COLS // 256) * 66 + (MV_COLS // 256) * 292 + MV_ROWS * 4


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6650 GB/s"


class Clocks:
    """Sample SM clocks and throttle reasons during the timed region."""

    def __init__(self, index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.index = index
        self.p = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        time.sleep(0.2)
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if "Active" in v and "Not" not in v:
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit("--gpus %d but WORLD_SIZE=%d" % (n_gpus, world))
    return world, rank, local


def max_over_ranks(value, world, dev):
    if world == 1:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---- CPU baselines (oracle restatement of the reference arithmetic) -------

def cpu_decode_baseline(weights, cfg, tokens, seconds=15.0, threads=None, logits=True):
    """The reference's decode step on the host cores: the oracle decodes
    prompt tokens from position 0 for about `seconds` (the ingestion rate
    when `logits` is False: Decoder::ingest computes no LM head)."""
    from oracle import oracle
    threads = threads or os.cpu_count()
    om = oracle.Qwen35(cfg, weights)
    om.step(tokens[0], logits=logits, threads=threads)  # warm
    n, t0 = 0, time.perf_counter()
    out = []
    while time.perf_counter() - t0 < seconds and n + 1 < len(tokens):
        out.append(om.step(tokens[n + 1], logits=logits, threads=threads))
        n += 1
    dt = time.perf_counter() - t0
    om.close()
    return ({"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
             "sample": "%d %s steps of the oracle Qwen35 at positions 1..%d, %.1f s, "
                       "projections row-chunked over %d threads as reference RowParallelism"
                       % (n, "decode" if logits else "ingestion (no LM head)", n, dt, threads)},
            out)


def device_state(model, cfg):
    """The model's position and every layer's cached / recurrent state, in
    the oracle's layouts (Qwen35.load_state)."""
    states = {}
    for l in range(cfg.layers):
        if cfg.is_full(l):
            states[(l, 2)] = model.read_state(l, 2)
            states[(l, 3)] = model.read_state(l, 3)
        else:
            states[(l, 0)] = model.read_state(l, 0)
            states[(l, 1)] = model.read_state(l, 1)
    return model.position, states


def cpu_decode_continued(weights, cfg, position, states, tokens, seconds=15.0, threads=None):
    """The reference's decode step on the host cores at the benchmarked
    positions: the oracle continues from a state at `position` (the device's
    state after the same prompt) and decodes `tokens` for about `seconds`.
    Returns (cpu_baseline, logits of every step it computed)."""
    from oracle import oracle
    threads = threads or os.cpu_count()
    om = oracle.Qwen35(cfg, weights)
    om.load_state(position, states)
    out = [om.step(tokens[0], threads=threads)]  # first step untimed
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and n + 1 < len(tokens):
        out.append(om.step(tokens[n + 1], threads=threads))
        n += 1
    dt = time.perf_counter() - t0
    om.close()
    return ({"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
             "sample": "%d decode steps of the oracle Qwen35 at positions %d..%d (continuing "
                       "from the device's state after the %d-token prompt), %.1f s, "
                       "projections row-chunked over %d threads as reference RowParallelism"
                       % (n, position + 1, position + n, position, dt, threads)},
            out)


def oracle_weights(cfg, seed=0):
    """The configuration's random-init weights built on the host by the
    oracle's generator (the same bytes as the library's; the reference arm
    never maps the product library)."""
    from oracle import oracle
    import qwen35
    return qwen35.synthetic_weights(cfg, seed=seed, generator=oracle.synth_weights)


def phase_trace_report(model, cfg, steps=3, out=sys.stderr):
    """Per-phase critical path of the dataflow step from its globaltimer
    stamps (prism_b200_model_phase_trace / _phase_trace_ctas), printed as a
    table: for each phase kind, the time from the previous phase's last CTA
    to this phase's last CTA (mean over the layers), CTA 0's split of it,
    and the attention phase's sub-steps.  The stamps add a few stores per
    phase; the step traced is otherwise the timed one."""
    import ctypes
    L = model.L
    for fn in ("prism_b200_model_phase_trace", "prism_b200_model_phase_trace_ctas"):
        getattr(L, fn).restype = ctypes.c_int64
        getattr(L, fn).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    if model.step_mode != 2:
        print("phase trace: the dataflow step is not in use", file=out)
        return
    totals = []
    for _ in range(steps):
        totals.append(model.step_timings()[3])
    names = ["embed"]
    for l in range(cfg.layers):
        names += (["attn_qkv", "attention", "attn_out"] if cfg.is_full(l)
                  else ["gdn_proj", "gdn_rec", "gdn_out"])
        names += ["ffn_upgate", "ffn_down"]
    names += ["lm_head"]
    P = len(names)
    buf = np.zeros(16 * P, np.uint64)
    n = L.prism_b200_model_phase_trace(model.h, buf.ctypes.data, buf.size)
    t = buf[:n].reshape(-1, 16).astype(np.int64)
    cb = np.zeros(P * 4 * 1024, np.uint64)
    n2 = L.prism_b200_model_phase_trace_ctas(model.h, cb.ctypes.data, cb.size)
    G = n2 // P // 4
    cc = cb[:P * G * 4].reshape(P, G, 4).astype(np.int64)
    ca, cs, ce = cc[:, :, 0], cc[:, :, 1], cc[:, :, 2]
    us = lambda x: x / 1e3
    print("traced steps: %s ms (one cooperative kernel per step, %d CTAs)"
          % (", ".join("%.3f" % x for x in totals), G), file=out)
    print("%-11s %3s %8s | %8s %8s %8s %8s %8s" % ("phase", "n", "crit_us", "arrive", "stage",
                                                    "wgt", "dots", "chain"), file=out)
    agg = {}
    for i, nm in enumerate(names[1:], 1):
        crit = us(ce[i].max() - ce[i - 1].max())
        row = [crit]
        if nm not in ("gdn_rec", "attention"):
            valid = ca[i] > 0
            arrive = us(np.median(ca[i][valid] - ce[i - 1].max())) if valid.any() else 0.0
            c0 = t[i]
            row += [arrive, us(c0[1] - c0[0]), us(c0[2] - c0[1]), us(c0[3] - c0[2]),
                    us(c0[4] - c0[3])]
        agg.setdefault(nm, []).append(row)
    total = 0.0
    for nm, rows in agg.items():
        r = np.mean(np.array(rows), axis=0)
        total += r[0] * len(rows)
        cols = " ".join("%8.2f" % x for x in r[1:]) if len(r) > 1 else ""
        print("%-11s %3d %8.2f | %s" % (nm, len(rows), r[0], cols), file=out)
    print("critical path sum %.1f us" % total, file=out)
    # every CTA's stamps after the previous phase's last CTA: median / max of
    # inputs arrived, staged (RMSNorm + Q8_K done), end; and the staged time
    # of the CTA that ends last
    dist = {}
    for i, nm in enumerate(names[1:], 1):
        if nm in ("gdn_rec", "attention"):
            continue
        prev = ce[i - 1].max()
        valid = ca[i] > 0
        if not valid.any():
            continue
        cp_ = cc[i, :, 3]
        a_, s_, e_, p_ = (ca[i][valid] - prev, cs[i][valid] - prev, ce[i][valid] - prev,
                          cp_[valid] - prev)
        last = np.argmax(e_)
        dist.setdefault(nm, []).append([np.median(a_), a_.max(), np.median(s_), s_.max(),
                                        np.median(e_), e_.max(), s_[last], a_[last],
                                        np.median(p_), p_[last]])
    # CTA 0's stage split (staged input phases): sum of squares, scale,
    # warp 0's quantization, closing barrier
    split = {}
    for i, nm in enumerate(names[1:], 1):
        c0 = t[i]
        if nm in ("gdn_rec", "attention") or not (c0[13] and c0[14] and c0[15]):
            continue
        split.setdefault(nm, []).append([c0[13] - c0[0], c0[14] - c0[13], c0[15] - c0[14],
                                         c0[1] - c0[15]])
    for nm, rows in split.items():
        r = np.mean(np.array(rows), axis=0) / 1e3
        print("%-11s stage split (CTA 0, us from phase start): inputs+sumsq %.2f, scale %.2f, "
              "quantize(w0) %.2f, barrier %.2f" % ((nm,) + tuple(r)), file=out)
    print("%-11s | %8s %8s | %8s %8s | %8s %8s | %9s %9s | %8s %9s" % (
        "per CTA", "arr_med", "arr_max", "stg_med", "stg_max", "end_med", "end_max",
        "last_stg", "last_arr", "pln_med", "last_pln"), file=out)
    for nm, rows in dist.items():
        r = np.mean(np.array(rows), axis=0) / 1e3
        print("%-11s | %8.2f %8.2f | %8.2f %8.2f | %8.2f %8.2f | %9.2f %9.2f | %8.2f %9.2f"
              % ((nm,) + tuple(r)), file=out)
    att = [i for i, nm in enumerate(names) if nm == "attention"]
    if att:
        keys = [(1, "inputs"), (2, "norm+rope"), (3, "K pass"), (4, "scores in"), (10, "max"),
                (11, "exp"), (12, "trees"), (13, "totals"), (8, "probs"), (9, "V pass"), (7, "end")]
        steps_ = np.array([[us(t[i, b] - t[i, a]) for (a, _), (b, _) in
                            zip([(0, "start")] + keys[:-1], keys)] for i in att])
        print("attention (CTA 0, mean over layers): " + ", ".join(
            "%s %.2f" % (k[1], v) for k, v in zip(keys, steps_.mean(axis=0))), file=out)


def cpu_matvec_baseline(seconds=10.0, threads=None):
    from oracle import oracle
    import synth
    threads = threads or os.cpu_count()
    w = synth.tq2_weights(MV_ROWS, MV_COLS, 0)
    x = synth.activations(MV_COLS, 0)
    oracle.matvec(35, w, MV_ROWS, MV_COLS, oracle.q8k_quantize(x), threads=threads)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.matvec(35, w, MV_ROWS, MV_COLS, oracle.q8k_quantize(x), threads=threads)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": reps * MV_BYTES / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": "%d x (Q8_K quantize + 4096x4096 TQ2_0 matvec), %.1f s, row chunks over "
                      "%d threads as reference RowParallelism" % (reps, dt, threads)}


# ---- GPU: projection microbenchmark ---------------------------

def gpu_matvec(ex, dev, steps=200, warmup=10):
    """Graph-captured back-to-back quantize + project steps over rotating
    copies; returns (GB/s whole step, GB/s projection kernel, us/launch,
    parity)."""
    import torch
    import prism_b200 as pb
    import synth
    w_host = synth.tq2_weights(MV_ROWS, MV_COLS, 0)
    x_host = synth.activations(MV_COLS, 0)
    t = pb.Tensor(pb.KIND_TQ2_0, MV_COLS, MV_ROWS, w_host)
    weights = [ex.upload(t) for _ in range(MV_COPIES)]
    x_dev = torch.from_numpy(x_host).to(dev)
    act = torch.empty((MV_COLS // 256) * 292, dtype=torch.uint8, device=dev)
    y = torch.empty(MV_ROWS, dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(device=dev)

    def capture(with_quant):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(steps):
                if with_quant:
                    ex.quantize_q8k_device(x_dev.data_ptr(), MV_COLS, act.data_ptr(),
                                           stream=s.cuda_stream)
                ex.project_device(weights[i % MV_COPIES], act.data_ptr(), y.data_ptr(),
                                  stream=s.cuda_stream)
        return g

    ex.quantize_q8k_device(x_dev.data_ptr(), MV_COLS, act.data_ptr(), stream=s.cuda_stream)
    res = []
    for with_quant in (True, False):
        g = capture(with_quant)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        with torch.cuda.stream(s):
            g.replay()
        e1.record(s)
        torch.cuda.synchronize()
        res.append(e0.elapsed_time(e1) / steps)  # ms per step
        del g
    ex.sync()
    from oracle import oracle
    y_ref = oracle.matvec(35, w_host, MV_ROWS, MV_COLS, oracle.q8k_quantize(x_host), threads=8)
    parity = bool(np.array_equal(y.cpu().numpy().view(np.uint32), y_ref.view(np.uint32)))
    for w in weights:
        w.release()
    step_ms, kern_ms = res
    return MV_BYTES / (step_ms / 1e3) / 1e9, MV_BYTES / (kern_ms / 1e3) / 1e9, kern_ms * 1e3, parity


# ---- GPU: decode ----------------------------------------------

def run_decode(args):
    import torch
    import prism_b200 as pb
    import qwen35

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    cfg = qwen35.CONFIG1
    K, W = args.steps, args.warmup
    PROMPT = args.prompt
    if PROMPT + W + K + 1 > cfg.context:
        raise SystemExit("prompt + warmup + steps exceeds the 1024-token context")
    t_build = time.perf_counter()
    weights = qwen35.synthetic_weights(cfg, seed=0)
    ex = pb.ProjectionExecutor(local)
    model = qwen35.Qwen35Model(ex, cfg)
    model.load(weights)
    t_build = time.perf_counter() - t_build
    prompt = qwen35.prompt_tokens(cfg, PROMPT, seed=1)
    stream = torch.cuda.ExternalStream(model.stream(), device=dev)

    # prefill: ingest the first PROMPT-1 prompt tokens (no LM head),
    # device-timed, as sequential decode-path steps and as one batched pass
    # (prism_b200_model_prefill_async; same resulting state)
    def timed_ingest(batched):
        model.reset()
        model.set_prompt(prompt)
        torch.cuda.synchronize()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record(stream)
        if batched:
            model.prefill_async(PROMPT - 1)
        else:
            model.ingest_async(PROMPT - 1)
        q1.record(stream)
        torch.cuda.synchronize()
        ex.sync()
        return max_over_ranks(q0.elapsed_time(q1), world, dev)

    seq_ms = timed_ingest(False)
    timed_ingest(True)  # first pass allocates the prompt buffers
    prefill_ms = timed_ingest(True)
    prefill_tps = world * (PROMPT - 1) / (prefill_ms / 1e3)
    prefill_seq_tps = world * (PROMPT - 1) / (seq_ms / 1e3)

    # decode: the first step consumes the last prompt token
    model.decode_async(W)
    torch.cuda.synchronize()
    ex.sync()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        d0.record(stream)
        model.decode_async(K)
        d1.record(stream)
        torch.cuda.synchronize()
    ex.sync()
    decode_ms = max_over_ranks(d0.elapsed_time(d1), world, dev)
    tps = world * K / (decode_ms / 1e3)
    ms_per_token = decode_ms / K
    context_mid = PROMPT + W + K // 2
    bytes_per_token = cfg.weight_bytes_per_token(context_mid)

    # per-layer phase timings of one more step (events between phases)
    att, ffn, head_ms, total_ms = model.step_timings()
    if args.phase_trace and rank == 0:
        phase_trace_report(model, cfg)
    bb = pb.BLOCK_BYTES[cfg.weight_kind]
    ffn_bytes = 3 * cfg.ffn * cfg.hidden // 256 * bb
    ffn_ms = float(np.median(ffn))

    # end to end through the public API: host token in, greedy token out
    model.reset()
    model.set_prompt(prompt)
    model.prefill_async(PROMPT - 1)
    tok = int(prompt[-1])
    for _ in range(W):
        _, tok = model.evaluate(tok, logits=False)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        _, tok = model.evaluate(tok, logits=False)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    e2e_tps = world * K / (e2e_ms / 1e3)

    # configs[0] projection on the same device
    mv_step, mv_kern, mv_us, mv_parity = gpu_matvec(ex, dev) if not args.no_matvec else (0, 0, 0, None)

    peak, peak_src = peaks()
    achieved_ffn = ffn_bytes / (ffn_ms / 1e3) / 1e9
    flow = model.step_mode == 2
    step_gbs = bytes_per_token / (ms_per_token / 1e3) / 1e9
    if flow:
        # one kernel is the whole step: its roofline is the step's
        roofline = {
            "bound": "hbm", "achieved": step_gbs, "peak": peak, "unit": "GB/s",
            "frac": step_gbs / peak, "peak_source": peak_src,
            "kernel": "decode_flow_kernel<35>: the whole decode step as one cooperative "
                      "launch (weights, recurrent and convolution state, KV rows of the "
                      "context), event-timed over the decode steps",
            "algorithmic_bytes_per_launch": bytes_per_token,
            "traffic": traffic_from_profiles("decode_flow_kernel"),
            "traffic_source": TRAFFIC_SOURCE,
            "step": {"achieved": step_gbs, "frac": step_gbs / peak,
                     "bytes_per_token": bytes_per_token},
            "ffn_phase_pair": {"achieved": achieved_ffn, "frac": achieved_ffn / peak,
                               "bytes": ffn_bytes,
                               "note": "the FFN up+gate and down phases of one layer, median "
                                       "over layers, from the traced step's phase times"}}
    else:
        roofline = {
            "bound": "hbm", "achieved": achieved_ffn, "peak": peak, "unit": "GB/s",
            "frac": achieved_ffn / peak, "peak_source": peak_src,
            "kernel": "FFN of one layer: matvec_kernel<35,kEpiSwiglu> (up+gate) + "
                      "matvec_kernel<35,kEpiStore> (down), median over layers, event-timed "
                      "without PDL",
            "algorithmic_bytes_per_launch": ffn_bytes,
            "traffic": traffic_from_profiles("ffn_layer"),
            "traffic_source": TRAFFIC_SOURCE,
            "step": {"achieved": step_gbs, "frac": step_gbs / peak,
                     "bytes_per_token": bytes_per_token}}
    line = {
        "metric": DECODE_METRIC, "value": tps, "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": decode_ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "i8xternary->i32,f32",
        "data": "synthetic (random-init weights, random prompt; no public dataset)",
        "config": {
            "workload": "configs[1]: Qwen3.5-style hybrid decoder, hidden 2560, 32 layers "
                        "(8 gated attention + 24 Gated DeltaNet), 16q/4kv x 256, FFN 9216, "
                        "vocab 151936 tied, TQ2_0 weights seed 0; 512-token prompt seed 1; "
                        "batch-1 greedy decode",
            "prompt": PROMPT, "decode_steps": K,
            "l2": "every step streams %.3f GB of weights and state (> 126 MB L2)"
                  % (bytes_per_token / 1e9),
            "graph": ("one CUDA graph per step holding one cooperative kernel: the dataflow "
                      "step (phases hand tagged activations to each other through global "
                      "memory, no grid barrier)") if flow else
                     "one CUDA graph per step, programmatic dependent launch between kernels",
            "step_mode": "flow" if flow else "sequence",
        },
        "clocks": clk.summary(),
        "gpu_launches": K if flow else K * (3 + 5 * cfg.layers),
        "e2e": {"value": e2e_tps, "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 12,
                "api": "prism_b200_model_evaluate per token (host token in, greedy token out)"},
        "roofline": roofline,
        "prefill": {"value": prefill_tps, "unit": "tok/s",
                    "tokens": PROMPT - 1, "ms": prefill_ms,
                    "note": "batched prompt ingestion (prism_b200_model_prefill_async: "
                            "tensor-core projections over the prompt, exact sequential "
                            "GDN recurrence, causal attention per token; no LM head); "
                            "state bit-identical to sequential ingestion",
                    "sequential": {"value": prefill_seq_tps, "unit": "tok/s", "ms": seq_ms,
                                   "note": "the same prompt as one-token decode-path "
                                           "ingestion steps"}},
        "matvec": {"metric": MATVEC_METRIC, "value": mv_step, "unit": "GB/s",
                   "kernel_gbs": mv_kern, "us_per_launch": mv_us, "frac": mv_kern / peak,
                   "bit_exact": mv_parity,
                   "workload": "configs[0] 4096x4096 TQ2_0, 64 rotating copies, graph-captured"},
        "timings_ms": {"attention_full": float(np.median(att[[l for l in range(cfg.layers) if cfg.is_full(l)]])),
                       "attention_gdn": float(np.median(att[[l for l in range(cfg.layers) if not cfg.is_full(l)]])),
                       "ffn": ffn_ms, "head": head_ms, "step_eager": total_ms},
        "build_s": t_build,
    }
    if rank == 0 and not args.no_cpu:
        # the oracle continues from the device's state after the prompt, so
        # it decodes the benchmarked positions; every step it computes is
        # also compared with the device's logits for the same token
        cont = [int(prompt[-1])] + [int(t) for t in qwen35.prompt_tokens(cfg, 400, seed=2)]
        model.reset()
        model.set_prompt(prompt)
        model.prefill_async(PROMPT - 1)
        ex.sync()
        position, states = device_state(model, cfg)
        cb, cpu_logits = cpu_decode_continued(weights, cfg, position, states, cont, seconds=15.0)
        line["cpu_baseline"] = cb
        bit_equal, max_err = 0, 0.0
        for i, lr in enumerate(cpu_logits):
            lg, _ = model.evaluate(cont[i])
            bit_equal += int(np.array_equal(lg.view(np.uint32), lr.view(np.uint32)))
            max_err = max(max_err, float(np.max(np.abs(lg - lr))))
        line["parity"] = {"steps_compared": len(cpu_logits),
                          "positions": [position, position + len(cpu_logits) - 1],
                          "logits_bit_identical_steps": bit_equal,
                          "logits_max_abs_err": max_err,
                          "note": "device vs oracle logits at every step the CPU leg "
                                  "decoded, both continuing from the device's state after "
                                  "the prompt"}
    model.close()
    ex.close()
    if not args.no_serve:
        line["serve_tp"] = serve_tp_summary(args, world, rank, local, dev)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_matvec(args):
    import torch
    import prism_b200 as pb
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    ex = pb.ProjectionExecutor(local)
    with Clocks(local) as clk:
        step_gbs, kern_gbs, us, parity = gpu_matvec(ex, dev, steps=args.steps, warmup=args.warmup)
    peak, peak_src = peaks()
    value = world * step_gbs
    line = {
        "metric": MATVEC_METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": MV_BYTES / (step_gbs * 1e9) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "i8xternary->i32,f32", "data": "synthetic",
        "config": {"workload": "configs[0]: TQ2_0 matvec W 4096x4096, x 4096 N(0,1) -> Q8_K",
                   "l2": "64 rotating device copies of W (277 MB > 126 MB L2)"},
        "parity_bit_exact": parity, "clocks": clk.summary(), "gpu_launches": 2 * args.steps,
        "roofline": {"bound": "hbm", "achieved": kern_gbs, "peak": peak, "unit": "GB/s",
                     "frac": kern_gbs / peak, "peak_source": peak_src,
                     "kernel": "matvec_kernel<35,kEpiStore>", "us_per_launch": us,
                     "traffic": traffic_from_profiles("matvec_tq2_4096"),
                     "traffic_source": TRAFFIC_SOURCE},
    }
    if rank == 0 and not args.no_cpu:
        line["cpu_baseline"] = cpu_matvec_baseline()
    ex.close()
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


GDN_METRIC = "Gated DeltaNet decode step GB/s (B=64) and chunked prefill TFLOP/s"


def cpu_gdn_baseline(seconds=10.0):
    """The oracle's sequential GDN head step (reference src/graph.rs:801-822)
    over the configs[2] heads, one host thread: state bytes read and written
    per second."""
    from oracle import oracle
    d = 128
    rng = np.random.default_rng(3)
    st = rng.standard_normal((d, d)).astype(np.float32) * 0.1
    q = rng.standard_normal(d).astype(np.float32)
    k = rng.standard_normal(d).astype(np.float32)
    q /= np.linalg.norm(q)
    k /= np.linalg.norm(k)
    v = rng.standard_normal(d).astype(np.float32)
    oracle.gdn_head_step(st, q, k, v, 0.9, 0.5)
    t0, n = time.perf_counter(), 0
    while time.perf_counter() - t0 < seconds:
        st, _ = oracle.gdn_head_step(st, q, k, v, 0.9, 0.5)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n * 2 * d * d * 4 / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": "%d head steps (128 x 128 fp32 state read and written), %.1f s, one "
                      "thread" % (n, dt)}


def run_gdn(args):
    """the Gated DeltaNet kernels alone.  16 heads, d = 128,
    fp32 state; decode = one recurrent step for B in {1, 16, 64} (HBM bound:
    the state is read and written); prefill = 4096 tokens in chunks of 64
    (binary32 compute bound)."""
    import torch
    import prism_b200 as pb
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    ex = pb.ProjectionExecutor(local)
    H, D = 16, 128
    peak, peak_src = peaks()
    rng = np.random.default_rng(0)

    def make(batch, T):
        q = torch.randn(batch, T, H, D, device=dev)
        k = torch.randn(batch, T, H, D, device=dev)
        q /= q.norm(dim=-1, keepdim=True)
        k /= k.norm(dim=-1, keepdim=True)
        v = torch.randn(batch, T, H, D, device=dev)
        decay = torch.exp(-torch.nn.functional.softplus(torch.randn(batch, T, H, device=dev)))
        beta = torch.sigmoid(torch.randn(batch, T, H, device=dev))
        state = torch.zeros(batch, H, D, D, device=dev)
        out = torch.zeros(batch, T, H, D, device=dev)
        return q, k, v, decay, beta, state, out

    s = torch.cuda.Stream(device=dev)
    decode = {}
    for batch in (1, 16, 64):
        # rotate over enough state copies that every step misses L2
        copies = max(2, int(300e6 // (batch * H * D * D * 4)) + 1)
        sets = [make(batch, 1) for _ in range(copies)]
        def step(i):
            q, k, v, g, b, st, o = sets[i % copies]
            pb.gdn_decode_device(ex, batch, H, H, st.data_ptr(), q.data_ptr(), k.data_ptr(),
                                 v.data_ptr(), g.data_ptr(), b.data_ptr(), o.data_ptr(),
                                 stream=s.cuda_stream)
        for i in range(args.warmup):
            step(i)
        K = 50
        g_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_, stream=s):
            for i in range(K):
                step(i)
        with torch.cuda.stream(s):
            g_.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        with torch.cuda.stream(s):
            g_.replay()
        e1.record(s)
        torch.cuda.synchronize()
        us = max_over_ranks(e0.elapsed_time(e1) * 1e3 / K, world, dev)
        nbytes = 2 * batch * H * D * D * 4 + batch * H * D * 4 * 4 + batch * H * 8
        decode["B%d" % batch] = {"us_per_step": us, "gbs": nbytes / us / 1e3,
                                 "frac": nbytes / us / 1e3 / peak, "bytes": nbytes}
        del g_, sets
    ex.sync()
    prefill = {}
    T = 4096
    for batch in (1, 16):
        q, k, v, g, b, st, o = make(batch, T)
        def run():
            pb.gdn_prefill_device(ex, batch, T, H, H, 64, st.data_ptr(), q.data_ptr(),
                                  k.data_ptr(), v.data_ptr(), g.data_ptr(), b.data_ptr(),
                                  o.data_ptr(), stream=s.cuda_stream)
        run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(3):
            run()
        e1.record(s)
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / 3, world, dev)
        # algorithmic flops of the recurrence: 3 d^2 MACs per token per head
        # (S.k, S.q, rank-1 update) = 6 d^2 T H flops per sequence
        flops = 6.0 * D * D * T * H * batch
        prefill["B%d" % batch] = {"ms": ms, "tflops": flops / (ms / 1e3) / 1e12,
                                  "tokens_per_s": batch * T / (ms / 1e3)}
        del q, k, v, g, b, st, o
    ex.sync()
    ex.close()
    fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    line = {
        "metric": GDN_METRIC,
        "value": world * decode["B64"]["gbs"], "unit": "GB/s", "n_gpus": world, "steps": 50,
        "warmup": args.warmup, "ms_per_step": decode["B64"]["us_per_step"] / 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (configs[2] distributions)",
        "config": {"workload": "configs[2]: 16 heads, d_k = d_v = 128, fp32 state; decode "
                               "B in {1,16,64}; prefill T=4096 chunk 64",
                   "l2": "decode rotates state copies > 300 MB"},
        "decode": decode, "prefill": prefill,
        "roofline": {"bound": "hbm", "achieved": decode["B64"]["gbs"], "peak": peak,
                     "unit": "GB/s", "frac": decode["B64"]["frac"], "peak_source": peak_src,
                     "kernel": "gdn_step_kernel (B=64)",
                     "traffic": traffic_from_profiles("gdn_step_kernel"),
                     "traffic_source": TRAFFIC_SOURCE,
                     "prefill_fp32_peak_tflops_nominal": fp32_peak},
        "gpu_launches": 50,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


GEMM_M = 2048
GEMM_SHAPES = [(2560, 9216), (9216, 2560)]   # (K, N): gate/up and down
KVQ_METRIC = "rotated KV attention positions/s (configs[1] heads, rsq4, 8192 positions)"
KVQ_CONTEXTS = (2048, 8192, 32768)


def cpu_kvq_baseline(seconds=10.0, n=2048):
    """The oracle's attend_head (the reference's scalar Source arithmetic)
    over n rsq4 positions for the 16 heads of configs[1], one thread."""
    from oracle import oracle
    rng = np.random.default_rng(0)
    k = rng.standard_normal((n * 4, 256)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((n * 4, 256)).astype(np.float16).astype(np.float32)
    keys = oracle.kvq_encode(4, oracle.KVQ_KEY_SEED, k).reshape(n, 4, -1)
    vals = oracle.kvq_encode(4, oracle.KVQ_VALUE_SEED, v).reshape(n, 4, -1)
    q = rng.standard_normal((16, 256)).astype(np.float16).astype(np.float32)
    g = rng.standard_normal((16, 256)).astype(np.float32)
    reps, t0 = 0, time.perf_counter()
    while reps < 1 or time.perf_counter() - t0 < seconds:
        oracle.kvq_attend("rsq4", q, keys, vals, 16, 4, 1 / 16, g)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": reps * n * 16 / dt, "unit": "positions/s", "cores": 1, "kind": "port",
            "sample": "%d calls of the oracle's rsq4 attend_head over %d positions x 16 "
                      "heads (4 KV heads), %.1f s" % (reps, n, dt)}


def run_kvq(args):
    """The reference's rotated scalar KV attention (src/graph/quantized_kv.rs
    attend_head) on the device at the configs[1] attention geometry: 16
    query heads over 4 KV heads of 256 channels, 2048 / 8192 / 32768 cached
    positions, rsq4 (132 B keys and values) and rsq4k3v (100 B values).
    Record sets rotate so that every launch reads them from HBM; the codec's
    encode throughput is measured alongside."""
    import torch
    import prism_b200 as pb
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ex = pb.ProjectionExecutor(local)
    peak, peak_src = peaks()
    H, KV = 16, 4
    s = torch.cuda.Stream(device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    out = {}
    for policy, name in ((pb.KV_RSQ4, "rsq4"), (pb.KV_RSQ4K3V, "rsq4k3v")):
        vbits = 3 if policy == pb.KV_RSQ4K3V else 4
        vb = pb.kvq_record_bytes(vbits)
        for n in KVQ_CONTEXTS:
            per = n * KV * (132 + vb)
            copies = max(2, int(300e6 // per) + 1)
            sets = []
            with torch.cuda.stream(s):  # the rows and their encodes on one stream
                for c in range(copies):
                    kr = torch.randn(n * KV, 256, device=dev, generator=g).half().float()
                    vr = torch.randn(n * KV, 256, device=dev, generator=g).half().float()
                    keys = torch.empty(n * KV * 132, dtype=torch.uint8, device=dev)
                    vals = torch.empty(n * KV * vb, dtype=torch.uint8, device=dev)
                    ex.kvq_encode_device(4, pb.KVQ_KEY_SEED, kr.data_ptr(), n * KV,
                                         keys.data_ptr(), stream=s.cuda_stream)
                    ex.kvq_encode_device(vbits, pb.KVQ_VALUE_SEED, vr.data_ptr(), n * KV,
                                         vals.data_ptr(), stream=s.cuda_stream)
                    sets.append((keys, vals))
                    del kr, vr
            torch.cuda.synchronize()
            ex.sync()
            q = torch.randn(H, 256, device=dev, generator=g).half().float()
            gate = torch.randn(H, 256, device=dev, generator=g)
            o = torch.empty(H, 256, device=dev)
            torch.cuda.synchronize()

            def launch(i):
                keys, vals = sets[i % copies]
                ex.kvq_attend_device(policy, q.data_ptr(), keys.data_ptr(), vals.data_ptr(), n,
                                     H, KV, 1 / 16, gate.data_ptr(), o.data_ptr(),
                                     stream=s.cuda_stream)
            for i in range(max(args.warmup, 3)):
                launch(i)
            K = 20
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                for i in range(K):
                    launch(i)
            with torch.cuda.stream(s):
                gr.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with Clocks(local) as clk:
                e0.record(s)
                with torch.cuda.stream(s):
                    gr.replay()
                e1.record(s)
                torch.cuda.synchronize()
            ex.sync()
            us = e0.elapsed_time(e1) * 1e3 / K
            out["%s_%d" % (name, n)] = {
                "us_per_launch": us, "positions_per_s": n * H / (us * 1e-6),
                "record_bytes": per, "gbs": per / us / 1e3, "hbm_frac": per / us / 1e3 / peak,
                "clocks": clk.summary()}
            del gr, sets
    # encode throughput: 65536 rows of 256 channels, 4-bit, version 1 and 2
    rows = torch.randn(65536, 256, device=dev, generator=g)
    recs = torch.empty(65536 * 132, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    enc = {}
    for ver in (1, 2):
        def encode():
            ex.kvq_encode_device(4, pb.KVQ_KEY_SEED, rows.data_ptr(), 65536, recs.data_ptr(),
                                 version=ver, stream=s.cuda_stream)
        encode()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(5):
            encode()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 5
        enc["v%d" % ver] = {"ms": ms, "rows_per_s": 65536 / (ms * 1e-3),
                            "gbs": 65536 * (1024 + 132) / (ms * 1e-3) / 1e9}
    ex.sync()
    ex.close()
    head = out["rsq4_8192"]
    cb = None if args.no_cpu else cpu_kvq_baseline(seconds=10.0)
    line = {
        "metric": KVQ_METRIC, "value": head["positions_per_s"], "unit": "positions/s",
        "n_gpus": 1, "steps": 20, "warmup": max(args.warmup, 3),
        "ms_per_step": head["us_per_launch"] / 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64 scores, f32 values",
        "data": "synthetic: N(0,1) rows rounded to binary16, encoded on the device",
        "config": {"workload": "configs[1] attention geometry (16 q / 4 kv heads x 256) over "
                               "rotated scalar records, one launch per layer-token",
                   "l2": "record sets rotate over > 300 MB per context"},
        "attention": out, "encode_65536_rows": enc,
        "roofline": {"bound": "hbm", "achieved": head["gbs"], "peak": peak, "unit": "GB/s",
                     "frac": head["hbm_frac"], "peak_source": peak_src,
                     "kernel": "kvq_attend_kernel (rsq4, 8192 positions)",
                     "traffic": traffic_from_profiles("kvq_attend_kernel"),
                     "traffic_source": TRAFFIC_SOURCE,
                     "note": "latency-bound, not HBM-bound: each CTA's 32 binary32 value "
                             "chains run in position order (the reference's accumulation "
                             "contract), fed by the other warps; the binary64 score lanes "
                             "and the in-order chains set the time (profiles/"
                             "kvq_attend_rsq4.md)"},
        "cpu_baseline": cb, "gpu_launches": 20,
    }
    print(json.dumps(line), flush=True)


GEMM_METRIC = "prefill GEMM int-op/s (2048 tokens x Q8_K, TQ2_0 and Q2_K weights)"


def int8_peak(ex=None):
    """Dense int8 tensor peak: measured on this device by the library's
    tcgen05.mma.kind::i8 microbenchmark (prism_b200_tensor_peak_i8) when an
    executor is given; otherwise twice the measured bf16 burst (B200's dense
    int8 rate is twice its dense bf16 rate)."""
    if ex is not None:
        try:
            return ex.tensor_peak_i8(), ("measured: tcgen05.mma.kind::i8 128x256x32 back to back "
                                         "from shared memory, one CTA per SM "
                                         "(prism_b200_tensor_peak_i8)")
        except Exception:
            pass
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            bf16 = json.load(f).get("bf16_tflops")
        if bf16:
            return 2.0 * float(bf16), "2 x measured bf16 dense burst (MEASURED_PEAKS.json bf16_tflops)"
    return 2.0 * 1590.0, "2 x fallback bf16 1.59 PFLOP/s"


def run_gemm_tp(args, world, rank, local, dev):
    """configs[3] on N GPUs, partitioned as the FFN it belongs to: the
    2048-token FFN chain (gate and up K=2560 -> N=9216, SwiGLU, down
    9216 -> 2560, TQ2_0) with gate/up column-parallel and down row-parallel,
    its partial sums all-reduced over NVLink peer memory from the down GEMM's
    epilogue (prism_b200_ffn_*).  A step is one chain call; the value is the
    three GEMMs' int-ops per step over the max-over-ranks device time (total
    work fixed: strong scaling)."""
    import torch
    import prism_b200 as pb
    import synth
    K, N = GEMM_SHAPES[0]
    ex = pb.ProjectionExecutor(local)
    tens = [pb.Tensor(35, K, N, synth.tq2_weights(N, K, 3)),
            pb.Tensor(35, K, N, synth.tq2_weights(N, K, 4)),
            pb.Tensor(35, N, K, synth.tq2_weights(K, N, 5))]
    f = pb.FfnChain(ex, *tens, max_tokens=GEMM_M, tp_rank=rank, tp_size=world)
    handles = [None] * world
    torch.distributed.all_gather_object(handles, f.exchange_handle())
    f.connect(handles)
    x = torch.randn(GEMM_M, K, device=dev)
    r = torch.randn(GEMM_M, K, device=dev)
    y = torch.empty(GEMM_M, K, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # > 126 MB L2
    s = torch.cuda.ExternalStream(ex.stream(), device=dev)
    steps = min(args.steps, 20)

    def run():
        f.device(GEMM_M, x.data_ptr(), r.data_ptr(), y.data_ptr())

    for _ in range(args.warmup):
        run()
    ex.sync()
    torch.distributed.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    with Clocks(local) as clk:
        for e0, e1 in ev:
            with torch.cuda.stream(s):
                flush.zero_()
            e0.record(s)
            run()
            e1.record(s)
        torch.cuda.synchronize()
    ex.sync()
    ms = max_over_ranks(float(np.mean([e0.elapsed_time(e1) for e0, e1 in ev])), world, dev)
    ops = 3 * 2.0 * GEMM_M * K * N
    # end to end through the host-buffer call (tokens and residual in, rows out)
    xh = np.random.default_rng(6).standard_normal((GEMM_M, K)).astype(np.float32)
    rh = np.random.default_rng(7).standard_normal((GEMM_M, K)).astype(np.float32)
    f(xh, rh)
    torch.distributed.barrier()
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        f(xh, rh)
    e2e_s = max_over_ranks((time.perf_counter() - t0) / reps, world, dev)
    torch.distributed.barrier()
    f.close()
    peak, peak_src = int8_peak(ex)
    ex.close()
    line = {
        "metric": GEMM_METRIC, "value": ops / ms / 1e9, "unit": "Tint-op/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "i8 x u8 -> i32, f32 chain",
        "data": "synthetic (configs[3] distributions)",
        "config": {"workload": "configs[3] as a tensor-parallel FFN chain: M=2048 tokens, "
                               "gate/up K=2560 N=9216 column-parallel, down K=9216 N=2560 "
                               "row-parallel, TQ2_0, residual added; a step = one chain",
                   "parallelism": "tp%d, all-reduce fused into the down GEMM epilogue "
                                  "(peer stores) and the reduce kernel" % world,
                   "l2": "a 256 MB buffer is written between timed steps"},
        "clocks": clk.summary(),
        "gpu_launches": steps * 7,
        "e2e": {"value": ops / e2e_s / 1e12, "unit": "Tint-op/s",
                "h2d_bytes_per_step": 2 * GEMM_M * K * 4, "d2h_bytes_per_step": GEMM_M * K * 4,
                "api": "prism_b200_ffn_chain_tokens (host buffers), every rank"},
        "roofline": {"bound": "tensor", "achieved": ops / world / ms / 1e9, "peak": peak,
                     "unit": "Tint-op/s", "frac": ops / world / ms / 1e9 / peak,
                     "peak_source": peak_src,
                     "kernel": "per GPU: the rank's three GEMMs, quantizations, SwiGLU and "
                               "the all-reduce over the chain's device time",
                     "traffic": None},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def cpu_gemm_baseline(seconds=15.0):
    """Oracle per-token tile dots (reference src/kernels/prefill.rs:48-87) on
    all host cores for a sample of tokens of the gate/up shape."""
    from oracle import oracle
    import synth
    K, N = GEMM_SHAPES[0]
    w = synth.tq2_weights(N, K, 3)
    threads = os.cpu_count()
    n_tok = 8
    x = np.random.default_rng(4).standard_normal((n_tok, K)).astype(np.float32)
    oracle.project_tokens(35, w, N, K, x, threads=threads)
    t0, n = time.perf_counter(), 0
    while time.perf_counter() - t0 < seconds:
        oracle.project_tokens(35, w, N, K, x, threads=threads)
        n += n_tok
    dt = time.perf_counter() - t0
    ops = 2.0 * K * N * n
    return {"value": ops / dt / 1e12, "unit": "Tint-op/s", "cores": threads, "kind": "port",
            "sample": "%d tokens of the (K=%d, N=%d) TQ2_0 projection in 32-token tiles, %.1f s"
                      % (n, K, N, dt)}


def run_gemm(args):
    """multi-token projection on the tensor cores.  2048 tokens,
    (K, N) = (2560, 9216) and (9216, 2560), TQ2_0 and Q2_K weights,
    activations N(0,1) -> Q8_K on the device, f32 outputs."""
    import torch
    import prism_b200 as pb
    import synth
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
        if args.parallel == "tp":
            return run_gemm_tp(args, world, rank, local, dev)
    ex = pb.ProjectionExecutor(local)
    s = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # > 126 MB L2
    steps = min(args.steps, 20)
    results, total_ops, total_ms = {}, 0.0, 0.0
    launches = 0
    for kind, name in ((35, "tq2_0"), (10, "q2_k")):
        for K, N in GEMM_SHAPES:
            w = synth.tq2_weights(N, K, 3) if kind == 35 else synth.q2k_weights(N, K, 3)
            wt = ex.upload(pb.Tensor(kind, K, N, w))
            x = torch.randn(GEMM_M, K, device=dev)
            y = torch.empty(GEMM_M, N, device=dev)
            def run():
                ex.project_f32_tokens_device(wt, GEMM_M, x.data_ptr(), y.data_ptr(),
                                             stream=s.cuda_stream)
            for _ in range(args.warmup):
                run()
            ex.sync()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(steps)]
            with torch.cuda.stream(s):
                for e0, e1 in ev:
                    flush.zero_()
                    e0.record(s)
                    run()
                    e1.record(s)
            torch.cuda.synchronize()
            ex.sync()
            ms = max_over_ranks(float(np.mean([e0.elapsed_time(e1) for e0, e1 in ev])), world,
                                dev)
            ops = 2.0 * GEMM_M * K * N
            results["%s_K%d_N%d" % (name, K, N)] = {"ms": ms, "tops": ops / ms / 1e9}
            total_ops += ops
            total_ms += ms
            launches += 2 * steps
            del wt, x, y
    # end to end through the host-buffer entry point (gate/up, TQ2_0)
    K, N = GEMM_SHAPES[0]
    w = synth.tq2_weights(N, K, 3)
    t = pb.Tensor(35, K, N, w)
    xh = np.random.default_rng(4).standard_normal((GEMM_M, K)).astype(np.float32)
    ex.project_f32_tokens(t, xh)
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        ex.project_f32_tokens(t, xh)
    e2e_s = max_over_ranks((time.perf_counter() - t0) / reps, world, dev)
    peak, peak_src = int8_peak(ex)
    ex.close()
    value = total_ops / total_ms / 1e9  # per GPU, from the max-over-ranks times
    top = results["tq2_0_K2560_N9216"]
    line = {
        "metric": GEMM_METRIC, "value": value * world, "unit": "Tint-op/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": total_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "i8 x u8 -> i32, f32 chain", "data": "synthetic (configs[3] distributions)",
        "config": {"workload": "configs[3]: M=2048 tokens, (K,N) in {(2560,9216),(9216,2560)}, "
                               "TQ2_0 and Q2_K; a step = the four GEMMs",
                   "l2": "a 256 MB buffer is written between timed launches"},
        "gemms": results,
        "roofline": {"bound": "tensor", "achieved": top["tops"], "peak": peak,
                     "unit": "Tint-op/s", "frac": top["tops"] / peak, "peak_source": peak_src,
                     "kernel": "gemm_tokens_kernel<35> (K=2560, N=9216) incl. the Q8_K token "
                               "quantize launch",
                     "traffic": traffic_from_profiles("gemm_tokens_kernel"),
                     "traffic_source": TRAFFIC_SOURCE},
        "gpu_launches": launches,
        "e2e": {"value": world * 2.0 * GEMM_M * K * N / e2e_s / 1e12, "unit": "Tint-op/s",
                "h2d_bytes_per_step": GEMM_M * K * 4, "d2h_bytes_per_step": GEMM_M * N * 4,
                "api": "prism_b200_project_f32_tokens (host buffers), TQ2_0 K=2560 N=9216"},
    }
    if rank == 0 and not args.no_cpu:
        line["cpu_baseline"] = cpu_gemm_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)


PREFILL_TOKENS = 4096
PREFILL_METRIC = "prefill tok/s (batch 1, 4096-token prompt)"


def prefill_launches(cfg, tokens, chunk=2048):
    """Kernels of one prism_b200_model_prefill_async call: per 2048-token pass
    the positions, the embedding and the final position update, then per
    layer norm + quantize + projections + the mixer's kernels + FFN."""
    gdn = 2 + 4 + 4 + 2          # norm, quant, 4 GEMMs, inputs, scan, history, gated, quant, out
    att = 2 + 3 + 3 + 1 + 1      # norm, quant, q/k/v GEMMs, kv rows, query rows, attention, quant, o
    ffn = 2 + 2 + 1 + 1 + 1      # norm, quant, up/gate, swiglu, quant, down
    per_pass = 3 + sum((att if cfg.is_full(l) else gdn) + ffn for l in range(cfg.layers))
    return per_pass * ((tokens + chunk - 1) // chunk)


def projection_ops(cfg):
    """Integer multiply-adds x 2 of every projection of one token (no LM head)."""
    total = 0
    for l in range(cfg.layers):
        for _, rows, cols in cfg.linear_shapes(l):
            total += 2 * rows * cols
    return total


def run_prefill(args):
    """Batched prompt ingestion of the configs[1] model: a step is one
    prefill_async of a PREFILL_TOKENS-token prompt from position 0 (the
    model is reset and the prompt placed outside the timed region)."""
    import dataclasses
    import torch
    import prism_b200 as pb
    import qwen35

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    P = args.prefill_tokens
    cfg = dataclasses.replace(qwen35.CONFIG1, context=P + 8)
    K, W = min(args.steps, 10), args.warmup
    weights = qwen35.synthetic_weights(cfg, seed=0)
    ex = pb.ProjectionExecutor(local)
    model = qwen35.Qwen35Model(ex, cfg)
    model.load(weights)
    prompt = qwen35.prompt_tokens(cfg, P, seed=1)
    stream = torch.cuda.ExternalStream(model.stream(), device=dev)

    def one(timed):
        model.reset()
        model.set_prompt(prompt)
        torch.cuda.synchronize()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record(stream)
        model.prefill_async(P)
        q1.record(stream)
        torch.cuda.synchronize()
        ex.sync()
        return q0.elapsed_time(q1)

    for _ in range(W):
        one(False)
    if world > 1:
        torch.distributed.barrier()
    with Clocks(local) as clk:
        times = [one(True) for _ in range(K)]
    ms = max_over_ranks(float(np.sum(times)), world, dev)
    tps = world * K * P / (ms / 1e3)

    # end to end through the reference-facing block call (host tokens in,
    # device status out, 256-token blocks as Decoder::ingest_block takes)
    model.reset()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for b0 in range(0, P, 256):
        model.ingest_block(prompt[b0:b0 + 256])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    model.close()
    peak, peak_src = int8_peak(ex)
    ex.close()

    ops = projection_ops(cfg) * P
    achieved = ops / (ms / K / 1e3) / 1e12
    line = {
        "metric": PREFILL_METRIC, "value": tps, "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "i8xternary->i32,f32",
        "data": "synthetic (random-init weights, random prompt; no public dataset)",
        "config": {"workload": "configs[1] model (hidden 2560, 32 layers, TQ2_0 seed 0): "
                               "batched ingestion of a %d-token random prompt (seed 1) from "
                               "position 0, 2048-token passes, no LM head" % P,
                   "l2": "each pass streams the ~1 GB of weights (> 126 MB L2)"},
        "clocks": clk.summary(),
        "gpu_launches": K * prefill_launches(cfg, P),
        "e2e": {"value": world * P / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * P, "d2h_bytes_per_step": 4 * ((P + 255) // 256),
                "api": "prism_b200_model_ingest_block, 256-token blocks (host tokens in, "
                       "status out per block)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                     "unit": "Tint-op/s", "frac": achieved / peak, "peak_source": peak_src,
                     "kernel": "all projections of the pass (gemm_tokens_kernel), their "
                               "int-ops over the whole pass time (a lower bound on the GEMM "
                               "kernels' own rate)",
                     "algorithmic_ops_per_step": ops, "traffic": None},
    }
    if rank == 0 and not args.no_cpu:
        cb, _ = cpu_decode_baseline(weights, cfg, prompt, seconds=15.0)
        cb["sample"] = "sequential ingestion (the reference's Decoder::ingest per token): " + \
            cb["sample"]
        line["cpu_baseline"] = cb
    if rank == 0:
        print(json.dumps(line), flush=True)


SERVE_B, SERVE_CTX = 256, 8192
SERVE_TP_STEPS = 8  # steps of the serve_tp sub-object of the decode line
SERVE_METRIC = "batched decode tok/s (256 sequences x 8192-token context, Q8_0 KV)"


def serve_step_bytes(cfg, B, position, tp=1):
    """Algorithmic bytes one GPU moves in a batched step at `position` (every
    sequence): weights once, each sequence's Q8_0 K and V rows of the
    attention layers up to and including the new one, the GDN state read and
    written, the convolution history read and written.  Under `tp`-way
    tensor parallelism a rank holds 1/tp of the weights, GDN heads and
    channels, and max(kv_heads/tp, 1) KV heads (two ranks share a KV head
    when tp exceeds the KV heads)."""
    attn = sum(1 for l in range(cfg.layers) if cfg.is_full(l))
    gdn = cfg.layers - attn
    rec = cfg.head_dim // 32 * 2 + cfg.head_dim
    kv_local = max(cfg.kv_heads // tp, 1)
    kv = attn * 2 * kv_local * rec * (position + 1) * B
    state = gdn * 2 * cfg.ssm_values * cfg.ssm_state * cfg.ssm_state * 4 * B // tp
    conv = gdn * 2 * cfg.conv_channels * (cfg.conv_kernel - 1) * 4 * B // tp
    return cfg.linear_bytes() // tp + kv + state + conv


def serve_measure(args, world, rank, local, dev, K, W, tp, tp_mode):
    """Time the configs[4] batched step on this rank: `tp` ranks split every
    linear, the heads and the KV of the same sequences (tp == world), or each
    rank serves its own sequences (tp == 1).  Returns the measured figures;
    the process group (world > 1) is already up."""
    import torch
    import prism_b200 as pb
    import qwen35
    cfg = replace_ctx(qwen35.CONFIG1, SERVE_CTX)
    weights = qwen35.synthetic_weights(cfg, seed=0)
    ex = pb.ProjectionExecutor(local)
    model = qwen35.Qwen35Model(ex, cfg, kv_policy=qwen35.KV_Q8_0)
    model.load(weights)
    SB = args.sequences
    bt = qwen35.Qwen35Batch(model, SB, SERVE_CTX, tp_rank=rank if tp > 1 else 0, tp_size=tp,
                            tp_mode=tp_mode)
    if tp > 1:
        handles = [None] * world
        torch.distributed.all_gather_object(handles, bt.exchange_handle())
        bt.connect(handles)
    start = SERVE_CTX - (K + W + 4)
    # tensor-parallel ranks serve the same sequences: same seeds everywhere
    seq_seed = 0 if tp > 1 else rank
    bt.fill_context(start, seed=1 + seq_seed)
    toks = np.random.default_rng(2 + seq_seed).integers(0, cfg.vocab, SB).astype(np.uint32)
    if world > 1:
        torch.distributed.barrier()
    bt.step(toks)  # captures the step graph
    stream = torch.cuda.ExternalStream(bt.stream, device=dev)
    bt.decode_async(W)
    torch.cuda.synchronize()
    ex.sync()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        bt.decode_async(K)
        e1.record(stream)
        torch.cuda.synchronize()
    ex.sync()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    served = SB * (world // tp)   # sequences advanced per step by the whole job
    mid = start + 1 + W + K // 2
    step_bytes = serve_step_bytes(cfg, SB, mid, tp)
    # end to end: host tokens in, greedy tokens out, per step
    E = 3
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(E):
        toks = bt.step(toks)
    e2e_s = (time.perf_counter() - t0) / E
    if world > 1:
        torch.distributed.barrier()
    e2e = max_over_ranks(e2e_s, world, dev)
    bt.close()
    model.close()
    ex.close()
    return {"cfg": cfg, "weights": weights, "ms": ms, "K": K, "W": W, "served": served,
            "SB": SB, "start": start, "step_bytes": step_bytes, "e2e_s": e2e,
            "clocks": clk.summary()}


def serve_parallelism(tp, world, tp_mode):
    if tp == 1:
        return "sequences sharded over ranks (dp%d), no exchange" % world if world > 1 else \
            "one GPU"
    if tp_mode == "exact":
        return ("tp%d exact: column-sharded linears, heads and KV; per layer 2 all-gathers of "
                "quantized head/FFN outputs (fused into the quantizer) and 2 of hidden rows "
                "(fused into the GEMM epilogue) over NVLink peer memory; vocabulary-split "
                "output head" % tp)
    return ("tp%d all-reduce: column/row-sharded linears, heads and KV; 2 all-reduces per "
            "layer over NVLink peer memory fused into the GEMM epilogue + next RMSNorm; "
            "vocabulary-split output head" % tp)


def run_serve(args):
    """batched serving of 256 sequences with 8192-token random
    contexts (Q8_0 KV), greedy decode steps.  On N ranks, `--parallel tp`
    (the default, as configs[4] specifies) splits every linear layer, the
    heads and the KV cache of the same 256 sequences over the ranks and
    exchanges the row-parallel outputs over NVLink peer memory (strong
    scaling); `--parallel dp` serves N disjoint batches of 256 instead (weak
    scaling, no exchange)."""
    import torch
    import qwen35
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    tp = world if args.parallel == "tp" else 1
    tp_mode = qwen35.TP_ALLREDUCE if args.tp_mode == "allreduce" else qwen35.TP_EXACT
    r = serve_measure(args, world, rank, local, dev, min(args.steps, 64), args.warmup, tp,
                      tp_mode)
    cfg, K, ms, served, step_bytes = r["cfg"], r["K"], r["ms"], r["served"], r["step_bytes"]
    tps = served * K / (ms / 1e3)
    peak, peak_src = peaks()
    achieved = step_bytes / (ms / K / 1e3) / 1e9
    line = {
        "metric": SERVE_METRIC, "value": tps, "unit": "tok/s", "n_gpus": world, "steps": K,
        "warmup": r["W"], "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "strong" if tp > 1 else "weak",
        "vs_baseline": None, "dtype": "i8xternary->i32,f32; Q8_0 KV",
        "data": "synthetic (random-init weights, seeded random KV/recurrent context)",
        "config": {"workload": "configs[4]: %d sequences%s, 8192-token context filled "
                               "with seeded random Q8_0 KV rows and GDN/conv state, greedy decode "
                               "from position %d; configs[1] geometry"
                               % (r["SB"], " per GPU" if tp == 1 else "", r["start"]),
                   "sequences": served, "context": SERVE_CTX,
                   "parallelism": serve_parallelism(tp, world, args.tp_mode),
                   "l2": "each step reads %.1f GB (> 126 MB L2)" % (step_bytes / 1e9)},
        "clocks": r["clocks"],
        # embed; per attention layer 15 and per GDN layer 16 kernels (norm,
        # quantize, projections, attention or GDN, quantize, out-projection,
        # norm, quantize, up, gate, SwiGLU, quantize, down); norm, quantize,
        # output head, finish
        "gpu_launches": K * (1 + sum(15 if cfg.is_full(l) else 16 for l in range(cfg.layers))
                             + 4),
        "e2e": {"value": served / r["e2e_s"], "unit": "tok/s", "h2d_bytes_per_step": r["SB"] * 4,
                "d2h_bytes_per_step": r["SB"] * 4,
                "api": "prism_b200_batch_step per step (host tokens in, greedy tokens out)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "kernel": "whole batched step, per GPU (this rank's KV + GDN state + "
                               "weight bytes / step time)",
                     "algorithmic_bytes_per_step": step_bytes, "traffic": None},
    }
    if rank == 0 and not args.no_cpu:
        cb, _ = cpu_decode_baseline(r["weights"], qwen35.CONFIG1,
                                    qwen35.prompt_tokens(qwen35.CONFIG1, 64, seed=1), seconds=15.0)
        cb["sample"] = ("per-sequence oracle decode (the CPU serves sequences one at a time): " +
                        cb["sample"] + "; contexts near position 0, so the 8192-token attention "
                        "cost is not included (favours the CPU)")
        line["cpu_baseline"] = cb
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def serve_tp_summary(args, world, rank, local, dev):
    """The configs[4] tensor-parallel serving figure at this N (tp == N, the
    exact exchange form): the sub-object the decode line carries so that a
    1..8-GPU run of the default workload also measures the serving curve."""
    import qwen35
    r = serve_measure(args, world, rank, local, dev, SERVE_TP_STEPS, 3, world, qwen35.TP_EXACT)
    K, ms, served, step_bytes = r["K"], r["ms"], r["served"], r["step_bytes"]
    peak, peak_src = peaks()
    achieved = step_bytes / (ms / K / 1e3) / 1e9
    return {"metric": SERVE_METRIC, "value": served * K / (ms / 1e3), "unit": "tok/s",
            "n_gpus": world, "tp": world, "steps": K, "warmup": r["W"], "ms_per_step": ms / K,
            "scaling": "strong", "sequences": served, "context": SERVE_CTX,
            "parallelism": serve_parallelism(world, world, "exact"),
            "roofline": {"bound": "hbm", "achieved_per_gpu": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_src,
                         "algorithmic_bytes_per_step_per_gpu": step_bytes},
            "e2e": {"value": served / r["e2e_s"], "unit": "tok/s",
                    "h2d_bytes_per_step": r["SB"] * 4, "d2h_bytes_per_step": r["SB"] * 4,
                    "api": "prism_b200_batch_step per step"},
            "clocks": r["clocks"]}


def replace_ctx(cfg, context):
    from dataclasses import replace
    return replace(cfg, context=context)


def run_reference(args):
    world, rank, local = dist_setup(args.gpus)
    if rank != 0:
        return
    if args.workload == "matvec":
        cb = cpu_matvec_baseline(seconds=20.0)
        metric, unit = MATVEC_METRIC, "GB/s"
    elif args.workload == "gemm":
        cb = cpu_gemm_baseline(seconds=20.0)
        metric, unit = GEMM_METRIC, "Tint-op/s"
    elif args.workload == "gdn":
        cb = cpu_gdn_baseline(seconds=20.0)
        metric, unit = GDN_METRIC, "GB/s"
    elif args.workload == "kvq":
        cb = cpu_kvq_baseline(seconds=20.0, n=8192)
        metric, unit = KVQ_METRIC, "positions/s"
    else:
        import qwen35
        from oracle import oracle
        cfg = qwen35.CONFIG1
        weights = oracle_weights(cfg, seed=0)
        prompt = qwen35.prompt_tokens(cfg, PROMPT, seed=1)
        threads = os.cpu_count()
        metric, unit = DECODE_METRIC, "tok/s"
        if args.workload == "prefill":
            # the reference ingests a prompt token by token (Decoder::ingest)
            cb, _ = cpu_decode_baseline(weights, cfg, prompt, seconds=30.0, logits=False)
            metric = PREFILL_METRIC
            cb["sample"] = "sequential ingestion from position 0: " + cb["sample"]
        else:
            # the benchmarked positions: ingest the same prompt (untimed),
            # then W warm-up and up to K timed decode steps (at most ~30 s)
            om = oracle.Qwen35(cfg, weights)
            t_ing = time.perf_counter()
            for t in prompt[:-1]:
                om.step(int(t), logits=False, threads=threads)
            t_ing = time.perf_counter() - t_ing
            cont = [int(prompt[-1])] + [int(t) for t in qwen35.prompt_tokens(cfg, 600, seed=2)]
            for i in range(args.warmup):
                om.step(cont[i], threads=threads)
            n, t0 = 0, time.perf_counter()
            while n < args.steps and time.perf_counter() - t0 < 30.0:
                om.step(cont[args.warmup + n], threads=threads)
                n += 1
            dt = time.perf_counter() - t0
            om.close()
            cb = {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
                  "sample": "%d decode steps of the oracle Qwen35 at positions %d..%d after "
                            "ingesting the %d-token prompt (%.0f s, untimed), %.1f s, "
                            "projections row-chunked over %d threads as reference "
                            "RowParallelism" % (n, PROMPT - 1 + args.warmup,
                                                PROMPT - 2 + args.warmup + n, PROMPT - 1,
                                                t_ing, dt, threads)}
            if args.workload == "serve":
                # the reference serves each sequence with its own decoder
                metric = SERVE_METRIC
                cb["sample"] = ("per-sequence decode at context ~%d (the 8192-token "
                                "attention cost is not included): " % PROMPT) + cb["sample"]
    if unit == "tok/s":
        ms_per_step = 1e3 / cb["value"]
    elif unit == "positions/s":
        ms_per_step = 8192 * 16 / cb["value"] * 1e3
    elif unit == "Tint-op/s":
        ms_per_step = 2.0 * GEMM_M * GEMM_SHAPES[0][0] * GEMM_SHAPES[0][1] / (cb["value"] * 1e9)
    elif args.workload == "gdn":
        ms_per_step = 64 * 16 * 2 * 128 * 128 * 4 / (cb["value"] * 1e9) * 1e3
    else:
        ms_per_step = MV_BYTES / (cb["value"] * 1e9) * 1e3
    line = {
        "impl": "reference", "metric": metric, "value": cb["value"], "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.workload == "gdn" else "i8xternary->i32,f32", "data": "synthetic",
        "config": {"workload": "same as the ours arm, on the host cores",
                   "note": "the Rust reference cannot be built here (no cargo/rustc); the "
                           "oracle/ C restatement of its Source arithmetic is timed"},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "product_library_mapped": product_library_mapped(),
    }
    print(json.dumps(line), flush=True)


def product_library_mapped():
    """Whether this process mapped libprism_b200.so (the reference arm must
    not)."""
    try:
        with open("/proc/self/maps") as f:
            return "libprism_b200" in f.read()
    except OSError:
        return None


TRAFFIC_SOURCE = ("profiles/traffic.json: dram__bytes_read.sum + dram__bytes_write.sum per "
                  "launch from a committed ncu capture of the same kernel, not measured in "
                  "this run")


def traffic_from_profiles(key):
    """DRAM bytes per launch of the named kernel from the committed ncu
    summary (profiles/traffic.json), or None before one exists."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(key)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "matvec", "gdn", "gemm", "serve",
                                                                "prefill", "kvq"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-matvec", action="store_true", help="skip the configs[0] sub-benchmark")
    ap.add_argument("--phase-trace", action="store_true",
                    help="print the dataflow step's per-phase critical path to stderr")
    ap.add_argument("--no-serve", action="store_true",
                    help="skip the decode line's serve_tp (configs[4] at tp = N) sub-object")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens (profiling runs)")
    ap.add_argument("--prefill-tokens", type=int, default=PREFILL_TOKENS,
                    help="prefill workload: prompt tokens (profiling runs use fewer)")
    ap.add_argument("--parallel", default="tp", choices=["tp", "dp"],
                    help="serve workload on N GPUs: tensor-parallel (default) or sequence-sharded")
    ap.add_argument("--tp-mode", default="exact", choices=["exact", "allreduce"],
                    help="serve workload, tensor-parallel: gathered (bit-exact) or all-reduced "
                         "row-parallel projections")
    ap.add_argument("--sequences", type=int, default=SERVE_B,
                    help="serve workload: sequences per GPU (profiling runs use fewer)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "gdn":
        run_gdn(args)
    elif args.workload == "gemm":
        run_gemm(args)
    elif args.workload == "serve":
        run_serve(args)
    elif args.workload == "matvec":
        run_matvec(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "kvq":
        run_kvq(args)
    else:
        run_decode(args)
    import torch
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
