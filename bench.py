"""Benchmark of the nutllm token loop on B200.

Workload (default): BASELINE config 2 — TinyLlama-1.1B shape, INT4 block-32
linears with fp16 scales, fp32 embedding and classifier, seeded synthetic
weights N(0, 0.02), a 5-token prompt and 16 greedy decode steps, batch 1.
One step = one generation (prefill of the prompt + 16 greedy tokens), the
whole loop on the device.

  value     decode tok/s of the device-resident loop (CUDA events on the
            library's stream), prompt and weights already in HBM
  e2e       generated tok/s through the C ABI call a user makes
            (nut_generate_greedy: prompt from host memory in, ids out)
  roofline  the dominant kernel against the measured HBM copy bandwidth
  cpu_baseline  the reference's own CPU token loop (oracle/_ref) on this
            host, on a bounded sample of the same workload

`--impl reference` times the reference CPU implementation instead.
Multi-GPU: batch-1 decode of a model that fits one GPU does not shard;
`--gpus N` runs N independent replicas (weak scaling, no collective).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEED = 1234


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="tinyllama-int4")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,"
             "clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device),
                 f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ ours


def run_ours(args, rank, world, local):
    import nutllm_b200 as nb
    from nutllm_b200 import synthetic as syn

    wl = syn.WORKLOADS[args.workload]
    c = wl.model_config()
    w = syn.build_model(c, wl.qtype, SEED)
    prompt = syn.prompt_ids(c, SEED, wl.prompt)
    model = nb.DeviceModel(w, local)
    kv = nb.KVCache(model)

    def step():
        ids, _, st = nb.generate_greedy(model, kv, prompt, wl.steps,
                                        stop_at_eos=False)
        return ids, st

    for _ in range(max(args.warmup, 3)):
        ids, _ = step()

    barrier = _barrier(world)
    barrier()
    dec_s, pre_s, wall = 0.0, 0.0, 0.0
    with Clocks(local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ids, st = step()
            dec_s += st.decode_seconds
            pre_s += st.prefill_seconds
        wall = time.perf_counter() - t0
    barrier()
    dec_s = _max_over_ranks(dec_s, world)
    pre_s = _max_over_ranks(pre_s, world)
    wall = _max_over_ranks(wall, world)

    decoded = wl.steps * args.steps * world
    value = decoded / dec_s
    prefill_tps = wl.prompt * args.steps * world / pre_s
    e2e = wl.steps * args.steps * world / wall

    roofline = qmatvec_roofline(nb, local) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl, c)
    # kernels per generation step (v1: 7 per layer + embed per token,
    # lm_head + argmax reset per generated token)
    per_token = 7 * c.layers + 1
    launches = args.steps * ((wl.prompt + wl.steps) * per_token + 2 * wl.steps)
    if rank == 0:
        line = {
            "metric": "decode tok/s (TinyLlama-1.1B INT4, batch 1)",
            "value": round(value, 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(1e3 * (dec_s + pre_s) / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int4xfp32",
            "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids)",
            "config": {"workload": wl.name, "prompt": wl.prompt,
                       "decode_steps": wl.steps, "batch": wl.batch,
                       "parallelism": f"replicas{world}",
                       "l2": "inputs larger than L2 (807 MB of weights per token)"},
            "prefill_tok_s": round(prefill_tps, 2),
            "e2e": {"value": round(e2e, 2),
                    "unit": "generated tok/s via nut_generate_greedy (incl. prefill)",
                    "h2d_bytes_per_step": int(prompt.nbytes),
                    "d2h_bytes_per_step": int(wl.steps * 4)},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)


def qmatvec_roofline(nb, device):
    """Dominant kernel: the quantised matvec at the gate/up shape, timed with
    CUDA events on the stream it is launched on."""
    import torch
    rows, cols = 5632, 2048
    w = nb.synth_normal(SEED, 7, rows * cols, 0.02).reshape(rows, cols)
    q = nb.QuantizedMatrix.quantize(w, nb.INT4)
    dev = nb.DeviceQMatrix(q, device)
    torch.cuda.set_device(device)
    x = torch.randn(cols, device=f"cuda:{device}")
    y = torch.empty(rows, device=f"cuda:{device}")
    s = torch.cuda.current_stream()
    for _ in range(10):
        dev.matvec_async(x.data_ptr(), y.data_ptr(), s.cuda_stream)
    reps = 200
    # read (not write) a buffer larger than L2 between launches, so the
    # timed kernel finds the weights in HBM and no dirty lines to evict
    flush = torch.ones(512 << 20, dtype=torch.uint8, device=x.device)
    times = []
    for _ in range(reps):
        flush.sum()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(s)
        dev.matvec_async(x.data_ptr(), y.data_ptr(), s.cuda_stream)
        b.record(s)
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e-3)
    t = statistics.median(times)
    bytes_ = rows * cols // 2 + 2 * (rows * cols // 32) + 4 * cols + 4 * rows
    peak, src = measured_peaks()
    ach = bytes_ / t / 1e9
    return {"kernel": "qmatvec_kernel<int4> 5632x2048", "bound": "hbm",
            "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
            "frac": round(ach / peak, 4), "peak_source": src,
            "bytes_per_launch": bytes_, "us_per_launch": round(t * 1e6, 3),
            "traffic": None}


def cpu_baseline(wl, c):
    """The reference's own CPU loop on a bounded sample (prompt + 2 greedy
    tokens) of the same workload, all host threads."""
    import oracle
    threads = os.cpu_count() or 1
    sample_steps = 2
    try:
        if oracle.reference_available():
            r = oracle.Reference()
            rm = r.model(c, wl.qtype, SEED)
            from nutllm_b200 import synthetic as syn
            prompt = syn.prompt_ids(c, SEED, wl.prompt)
            _, _, _, ps, ds = rm.generate(prompt, sample_steps, threads,
                                          want_logits=False)
            kind = "reference"
        else:
            return {"value": None, "unit": "tok/s", "cores": threads,
                    "kind": "port", "sample": "reference build missing"}
    except Exception as e:  # pragma: no cover - reported, not fatal
        return {"value": None, "unit": "tok/s", "cores": threads,
                "kind": "reference", "sample": f"failed: {e}"}
    return {"value": round(sample_steps / ds, 3), "unit": "decode tok/s",
            "cores": threads, "kind": kind,
            "prefill_tok_s": round(wl.prompt / ps, 3),
            "sample": f"{wl.prompt}-token prompt + {sample_steps} greedy "
                      f"decode steps of {wl.name}, {threads} threads"}


# ------------------------------------------------------------- reference


def run_reference(args, rank, world):
    if rank != 0:
        return
    import oracle
    from nutllm_b200 import synthetic as syn
    wl = syn.WORKLOADS[args.workload]
    c = wl.model_config()
    if not oracle.reference_available():
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref not built (reference "
                                         "sources absent at build time)"}))
        return
    threads = os.cpu_count() or 1
    r = oracle.Reference()
    rm = r.model(c, wl.qtype, SEED)
    prompt = syn.prompt_ids(c, SEED, wl.prompt)
    sample_steps = min(wl.steps, 4)
    for _ in range(min(args.warmup, 1)):
        rm.generate(prompt, 1, threads, want_logits=False)
    dec, pre = 0.0, 0.0
    for _ in range(args.steps):
        _, _, _, ps, ds = rm.generate(prompt, sample_steps, threads,
                                      want_logits=False)
        dec += ds
        pre += ps
    value = sample_steps * args.steps / dec
    print(json.dumps({
        "impl": "reference",
        "metric": "decode tok/s (TinyLlama-1.1B INT4, batch 1)",
        "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * (dec + pre) / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4xfp32", "data": "synthetic",
        "config": {"workload": wl.name, "prompt": wl.prompt,
                   "decode_steps": sample_steps, "batch": 1},
        "prefill_tok_s": round(wl.prompt * args.steps / pre, 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s",
                         "cores": threads, "kind": "reference",
                         "sample": f"{wl.prompt}-token prompt + {sample_steps} "
                                   f"greedy steps per step"},
        "e2e": {"value": round(value, 3), "unit": "tok/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------- plumbing


_pg = None


def _init_dist(world):
    global _pg
    if world > 1 and _pg is None:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
        _pg = dist


def _barrier(world):
    def b():
        if world > 1:
            _pg.barrier()
    return b


def _max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    _pg.all_reduce(t, op=_pg.ReduceOp.MAX)
    return float(t.item())


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    _init_dist(world)
    run_ours(args, rank, world, local)
    if world > 1:
        _pg.barrier()
        _pg.destroy_process_group()


if __name__ == "__main__":
    main()
