"""Benchmark of the B200 quantized decode hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0).  Workload (configs[0] of the benchmark
configuration): one packed TQ2_0 projection y = W x, W 4096 x 4096 ternary
(seed 0) with fp16 block scales in U(0.01, 0.05), x 4096 N(0,1) quantized
to Q8_K on the device.  A step is quantize + project.  The timed region
rotates through 64 device-resident copies of W (277 MB > 126 MB L2), so
every step streams its weights from HBM.

``--impl reference`` times the reference's CPU arithmetic on the host cores
(the C restatement in oracle/, since the Rust reference cannot be built
here) on the same workload and prints the same line with
"impl": "reference".

Multi-GPU: the batch-1 projection does not shard, so N ranks run N
independent replicas (one per GPU, launched by torchrun); `value` is the
sum of all ranks' bytes over the max-over-ranks device time.
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

ROWS = COLS = 4096
COPIES = 64
# algorithmic bytes of one projection: packed W + Q8_K x + f32 y
W_BYTES = ROWS * (COLS // 256) * 66
ACT_BYTES = (COLS // 256) * 292
Y_BYTES = ROWS * 4
STEP_BYTES = W_BYTES + ACT_BYTES + Y_BYTES
METRIC = "packed-matvec HBM GB/s (TQ2_0 x Q8_K, batch 1)"
WORKLOAD = {
    "workload": "configs[0]: TQ2_0 matvec W 4096x4096 ternary seed 0, fp16 scales U(0.01,0.05), "
                "x 4096 N(0,1) -> Q8_K on device",
    "rows": ROWS, "cols": COLS, "bytes_per_step": STEP_BYTES,
    "l2": "64 rotating device copies of W (277 MB > 126 MB L2)",
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
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


def cpu_baseline(seconds=10.0, threads=None):
    """The reference CPU arithmetic (oracle restatement) on the host cores:
    Q8_K quantization + row-parallel TQ2_0 matvec, repeated on the same
    workload for about `seconds`."""
    from oracle import oracle
    import synth
    threads = threads or os.cpu_count()
    w = synth.tq2_weights(ROWS, COLS, 0)
    x = synth.activations(COLS, 0)
    oracle.matvec(35, w, ROWS, COLS, oracle.q8k_quantize(x), threads=threads)  # warm
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        act = oracle.q8k_quantize(x)
        oracle.matvec(35, w, ROWS, COLS, act, threads=threads)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": reps * STEP_BYTES / dt / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": "%d x (Q8_K quantize + 4096x4096 TQ2_0 matvec), %.1f s, row chunks over %d "
                      "threads as reference RowParallelism" % (reps, dt, threads)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit("--gpus %d but WORLD_SIZE=%d" % (n_gpus, world))
    return world, rank, local


def run_reference(args):
    world, rank, local = dist_setup(args.gpus)
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_baseline(seconds=0.5)
    per = []
    for _ in range(args.steps):
        per.append(cpu_baseline(seconds=max(1.0, 20.0 / max(1, args.steps))))
    value = float(np.mean([p["value"] for p in per]))
    cb = dict(per[-1])
    cb["value"] = value
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": STEP_BYTES / (value * 1e9) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "i8xternary->i32,f32",
        "data": "synthetic", "config": WORKLOAD, "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import prism_b200 as pb
    import synth

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    ex = pb.ProjectionExecutor(local)
    w_host = synth.tq2_weights(ROWS, COLS, 0)
    x_host = synth.activations(COLS, 0)
    t = pb.Tensor(pb.KIND_TQ2_0, COLS, ROWS, w_host)
    weights = [ex.upload(t) for _ in range(COPIES)]
    dev = torch.device("cuda", local)
    x_dev = torch.from_numpy(x_host).to(dev)
    act_dev = torch.empty(ACT_BYTES, dtype=torch.uint8, device=dev)
    y_dev = torch.empty(ROWS, dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(ex.stream(), device=dev)
    s_ptr = ex.stream()
    torch.cuda.synchronize()

    def step(i, ev=None):
        ex.quantize_q8k_device(x_dev.data_ptr(), COLS, act_dev.data_ptr(), stream=s_ptr)
        if ev is not None:
            ev[0].record(stream)
        ex.project_device(weights[i % COPIES], act_dev.data_ptr(), y_dev.data_ptr(), stream=s_ptr)
        if ev is not None:
            ev[1].record(stream)

    for i in range(args.warmup):
        step(i)
    ex.sync()

    # device-timed region (barrier + synchronize on both sides, max over ranks)
    kern_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            step(args.warmup + i, kern_ev[i])
        stop.record(stream)
        torch.cuda.synchronize()
    ex.sync()
    total_ms = start.elapsed_time(stop)
    kern_ms = float(np.mean([a.elapsed_time(b) for a, b in kern_ev]))
    if world > 1:
        t_all = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t_all, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t_all.item())
    value = world * args.steps * STEP_BYTES / (total_ms / 1e3) / 1e9

    # parity spot check of the timed output against the oracle (untimed)
    from oracle import oracle
    y_ref = oracle.matvec(35, w_host, ROWS, COLS, oracle.q8k_quantize(x_host), threads=8)
    y = y_dev.cpu().numpy()
    parity = bool(np.array_equal(y.view(np.uint32), y_ref.view(np.uint32)))

    # end to end through the public host API: pinned x in, y out, per step
    x_pin = torch.from_numpy(x_host).pin_memory()
    y_pin = torch.empty(ROWS, dtype=torch.float32).pin_memory()
    x_np, y_np = x_pin.numpy(), y_pin.numpy()
    for i in range(args.warmup):
        ex.project_f32(weights[i % COPIES], x_np, out=y_np)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(args.steps):
        ex.project_f32(weights[i % COPIES], x_np, out=y_np)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t_all = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t_all, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t_all.item())
    e2e = world * args.steps * STEP_BYTES / (e2e_ms / 1e3) / 1e9

    peak, peak_kind = peaks()
    achieved = STEP_BYTES / (kern_ms / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)"
            if peak_kind == "measured" else "fallback 6650 GB/s",
            "kernel": "matvec_kernel<35> (tq2 projection)",
            "algorithmic_bytes_per_launch": STEP_BYTES,
            "traffic": traffic_from_profiles()}
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "i8xternary->i32,f32",
        "data": "synthetic", "config": WORKLOAD, "parity_bit_exact": parity,
        "clocks": clk.summary(), "gpu_launches": 2 * args.steps,
        "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": COLS * 4,
                "d2h_bytes_per_step": ROWS * 4, "api": "prism_b200_project_f32 (host buffers)"},
        "roofline": roof,
    }
    if rank == 0 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(seconds=10.0)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    for w in weights:
        w.release()
    ex.close()
    if rank == 0:
        print(json.dumps(line), flush=True)


def traffic_from_profiles():
    """DRAM bytes per launch of the projection kernel from the committed ncu
    summary (profiles/matvec_tq2_4096.md), or None before one exists."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("matvec_tq2_4096")
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
