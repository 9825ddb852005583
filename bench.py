"""Benchmark of the nutllm token loop on B200.

Workload (default): BASELINE config 2 — TinyLlama-1.1B shape, INT4 block-32
linears with fp16 scales, fp32 embedding and classifier, seeded synthetic
weights N(0, 0.02), a 5-token prompt and 16 greedy decode steps, batch 1.
One step = one generation (prefill of the prompt + 16 greedy tokens), the
whole loop on the device.

  value     decode tok/s of the device-resident loop, weights already in
            HBM (each generation timed with CUDA events on the library's
            stream; the prefill/decode split inside the one launch from the
            kernel's device-timer stamps)
  e2e       decode tok/s through the C ABI call a user makes
            (nut_generate_greedy: prompt from host memory in, ids out; wall
            clock less the in-kernel prefill time)
  roofline  the dominant kernel (the persistent token loop, one launch per
            generation) against the measured HBM copy bandwidth
  qmatvec   microbenchmark (a): the quantised matvec at the BASELINE shapes
  prefill_gemm  microbenchmark (b): the tcgen05 prefill GEMM, 512 tokens
  fp32      microbenchmark (c): fp32 768^3 GEMM and 4096^2 matvec
  cpu_baseline  the reference's own CPU token loop (oracle/_ref) on this
            host, all threads, on the whole workload once

  tp        BASELINE config 5 beside it: the Llama-2-7B shape, 64 sequences,
            tensor-parallel over the run's N ranks (NCCL all-reduce after
            Wo and Wdown), a few generations (--no-tp skips it)

`--impl reference` times the reference CPU implementation instead.
Multi-GPU: batch-1 decode of a model that fits one GPU does not shard;
`--gpus N` runs N independent replicas (weak scaling, no collective) as
`value`, and the tensor-parallel 7B path over the same N ranks as `tp`.
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
L2_BYTES = 126 << 20  # B200 L2

LABELS = {
    "tinyllama-int4": "TinyLlama-1.1B INT4",
    "tinyllama-int8-long": "TinyLlama-1.1B INT8, 512-token prompt + 256 steps",
    "tiny-int8": "tiny dim-288 INT8",
}


def metric_of(wl):
    return f"decode tok/s ({LABELS.get(wl.name, wl.name)}, batch 1)"


def dtype_of(wl, nb):
    return "int4xfp32" if wl.qtype == nb.INT4 else "int8xfp32"




def config_of(wl, world):
    """The workload description, identical in both arms of the bench."""
    from nutllm_b200 import synthetic as syn  # workload tables only: loads no library
    c = wl.model_config()
    per_token = syn.algorithmic_decode_bytes(c, wl.qtype, 0)
    return {"workload": wl.name, "prompt": wl.prompt, "decode_steps": wl.steps,
            "batch": wl.batch, "parallelism": f"replicas{world}",
            "l2": ("inputs larger than L2" if per_token > L2_BYTES else "inputs fit in L2")
                  + " (%.1f MB of weights and classifier per token)" % (per_token / 1e6)}


def cpu_sample(wl):
    """(prompt tokens, greedy steps) the reference CPU runs per sample: the
    whole workload when it takes seconds, a bounded prefix otherwise."""
    if wl.prompt + wl.steps > 64:
        return 64, 8
    return wl.prompt, wl.steps


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="tinyllama-int4")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-micro", action="store_true",
                   help="skip the kernel microbenchmarks")
    p.add_argument("--micro-only", action="store_true",
                   help="run only the kernel microbenchmarks (one JSON line)")
    p.add_argument("--micro-shape", default=None,
                   help="restrict the microbenchmarks to one ROWSxCOLS weight shape")
    p.add_argument("--no-tp", action="store_true",
                   help="skip the tensor-parallel 7B side measurement of the default line")
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
    import torch
    import nutllm_b200 as nb
    from nutllm_b200 import synthetic as syn

    wl = syn.WORKLOADS[args.workload]
    c = wl.model_config()
    w = syn.build_model(c, wl.qtype, SEED)
    prompt = syn.prompt_ids(c, SEED, wl.prompt)
    torch.cuda.set_device(local)
    model = nb.DeviceModel(w, local)
    kv = nb.KVCache(model)
    # the library enqueues every generation on its model's own stream: the
    # CUDA events that time it are recorded on that stream
    lib_stream = torch.cuda.ExternalStream(model.stream, device=local)

    # One timed step is G whole generations: short generations (~10 ms)
    # would otherwise give a timed region of a fraction of a second and a
    # single clock sample.
    G = 5 if wl.prompt + wl.steps <= 64 else 1

    class Split:
        decode_seconds = 0.0
        prefill_seconds = 0.0

    def step():
        tot = Split()
        for _ in range(G):
            ids, _, st = nb.generate_greedy(model, kv, prompt, wl.steps,
                                            stop_at_eos=False)
            tot.decode_seconds += st.decode_seconds
            tot.prefill_seconds += st.prefill_seconds
        return ids, tot

    warmup = max(args.warmup, 3)
    for _ in range(warmup):
        ids, _ = step()

    barrier = _barrier(world)
    events = []
    dec_s, pre_s = 0.0, 0.0
    barrier()
    torch.cuda.synchronize(local)
    launches0 = nb.launch_count()
    with Clocks(local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(lib_stream)
            ids, st = step()
            b.record(lib_stream)
            events.append((a, b))
            dec_s += st.decode_seconds
            pre_s += st.prefill_seconds
        torch.cuda.synchronize(local)
        wall = time.perf_counter() - t0
    launches = nb.launch_count() - launches0
    barrier()
    step_s = sum(a.elapsed_time(b) for a, b in events) * 1e-3
    step_s = _max_over_ranks(step_s, world)
    dec_s = _max_over_ranks(dec_s, world)
    pre_s = _max_over_ranks(pre_s, world)
    wall = _max_over_ranks(wall, world)

    value = wl.steps * G * args.steps * world / dec_s
    prefill_tps = wl.prompt * G * args.steps * world / pre_s
    tp = None if args.no_tp else tp_side(rank, world, local)
    e2e = wl.steps * G * args.steps * world / (wall - pre_s)
    e2e_gen = wl.steps * G * args.steps * world / wall

    if rank != 0:
        return
    per_launch = syn.algorithmic_decode_launch_bytes(c, wl.qtype, wl.prompt, wl.steps)
    if wl.prompt >= syn.GEMM_PREFILL_MIN:
        # the prompt went through the GEMM prefill: the decode part of a
        # generation is the first classifier read plus the persistent launch
        # from position `prompt`, timed by the library (decode_seconds)
        launch_s = dec_s / (args.steps * G)
        kernel = ("decode_mk_kernel after the GEMM prefill (first classifier read, "
                  "then one launch: %d passes, %d classifier reads)"
                  % (wl.steps, wl.steps - 1))
    else:
        launch_s = step_s / (args.steps * G)
        kernel = ("decode_mk_kernel (persistent token loop, one launch per "
                  "generation: %d passes, %d classifier reads)"
                  % (wl.prompt + wl.steps, wl.steps))
    peak, src = measured_peaks()
    ach = per_launch / launch_s / 1e9
    roofline = {
        "kernel": kernel,
        "bound": "hbm", "achieved": round(ach, 1), "peak": peak,
        "unit": "GB/s", "frac": round(ach / peak, 4), "peak_source": src,
        "algorithmic_bytes_per_launch": per_launch,
        "ms_per_launch": round(launch_s * 1e3, 4),
        "traffic": NCU_TRAFFIC.get(wl.name),
    }
    micro = None if args.no_micro else qmatvec_micro(nb, local, peak)
    tpeak, tsrc = measured_tensor_peak()
    gemm = None if args.no_micro else {
        "peak_tflops": tpeak, "peak_source": tsrc,
        "shapes": gemm_micro(nb, local, tpeak)}
    fp32 = None if args.no_micro else fp32_micro(nb, local, peak, tpeak)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl, c)
    line = {
        "metric": metric_of(wl),
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": round(1e3 * step_s / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": dtype_of(wl, nb),
        "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids)",
        "config": config_of(wl, world),
        "timing": "step: %d whole generations (one persistent launch each), CUDA "
                  "events on the library stream; prefill/decode split: in-kernel device "
                  "timer; e2e: wall clock around nut_generate_greedy with host buffers, "
                  "less the device prefill time" % G,
        "generations_per_step": G,
        "prefill_tok_s": round(prefill_tps, 2),
        "e2e": {"value": round(e2e, 2), "unit": "tok/s",
                "h2d_bytes_per_step": int(prompt.nbytes) * G,
                "d2h_bytes_per_step": int(wl.steps * 4) * G,
                "what": "decode tok/s through nut_generate_greedy with host buffers: "
                        "wall clock of the calls (prompt copy in, ids copy out, launch) "
                        "less the in-kernel prefill time",
                "generated_tok_s_incl_prefill": round(e2e_gen, 2)},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "qmatvec": micro,
        "prefill_gemm": gemm,
        "fp32": fp32,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "tp": tp,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- 7B batched, TP

LLAMA7B = dict(layers=32, heads=32, dim=4096, head_dim=128, ffn_dim=11008, vocab_size=32000,
               max_seq=256, eos_token=1, kv_heads=32)
TP_WORKLOADS = {
    # batch 64, 128-token prompts, 128 greedy steps
    "llama7b-int4-b64": dict(cfg=LLAMA7B, batch=64, prompt=128, steps=128),
    # the same shape with 4 layers, for quick checks
    "llama7b-int4-b64-4l": dict(cfg=dict(LLAMA7B, layers=4), batch=64, prompt=128, steps=128),
}


def tp_config_of(name, spec, world):
    """The TP workload description, identical in both arms of the bench."""
    return {"workload": name, "layers": spec["cfg"]["layers"], "batch": spec["batch"],
            "prompt": spec["prompt"], "decode_steps": spec["steps"],
            "parallelism": f"tp{world}",
            "l2": "inputs larger than L2 (every decode step reads the weights and "
                  "KV cache, several GB, from HBM)"}


def tp_decode_bytes(cfg, batch, prompt, steps, world):
    """Algorithmic bytes one rank reads per decode step, averaged over the
    steps: its share of the INT4 linears (q/4 + 2 bytes per 32 weights) and
    of the fp32 classifier, the replicated norms, and its heads' fp32 keys and
    values for every sequence at positions 0..pos."""
    d, f, L, V = cfg["dim"], cfg["ffn_dim"], cfg["layers"], cfg["vocab_size"]
    kvd = cfg["kv_heads"] * cfg["head_dim"]
    params = L * (2 * d * d + 2 * d * kvd + 3 * d * f)
    lin = params // 2 + params // 32 * 2
    cls = V * d * 4
    norms = (2 * L + 1) * d * 4
    avg_ctx = prompt + steps / 2.0
    kv = 2 * L * batch * kvd * 4 * avg_ctx
    return (lin + cls + kv) / world + norms


def cpu_reference_7b(spec, samples=1, warmup=1, n_prompt=4, n_steps=4):
    """The reference's own quantised token loop on the full 7B shape at
    batch 1 (it generates one sequence at a time): the unmodified reference
    (oracle/_ref) builds and quantises the model from the seeded weights, then
    runs prefill_quantized + greedy decode_quantized_token over all host
    threads.  Bounded: each sample is an n_prompt-token prompt and n_steps
    greedy steps.  Returns (decode tok/s, prefill tok/s, threads, sample)."""
    import oracle
    threads = os.cpu_count() or 1
    if not oracle.reference_available():
        return None, None, threads, "oracle/_ref not built"
    from nutllm_b200 import synthetic as syn  # workload tables only: loads no library
    cfg = syn.Config(**spec["cfg"])
    rm = oracle.Reference().model(cfg, 1, SEED)
    prompt = oracle.prompt_ids(cfg, SEED, n_prompt)
    for _ in range(warmup):
        rm.generate(prompt, 1, threads, want_logits=False)
    dec = pre = 0.0
    for _ in range(samples):
        _, _, _, ps, ds = rm.generate(prompt, n_steps, threads, want_logits=False)
        dec += ds
        pre += ps
    sample = (f"batch 1, all {cfg.layers} layers: {n_prompt}-token prompt + {n_steps} greedy "
              f"steps per sample, {samples} samples, reference kernels, {threads} threads")
    return n_steps * samples / dec, n_prompt * samples / pre, threads, sample


def tp_side(rank, world, local, steps=3, warmup=3, workload="llama7b-int4-b64"):
    """BASELINE config 5 (Llama-2-7B shape, INT4, 64 sequences, 128-token
    prompts, 128 greedy steps) tensor-parallel over this run's `world` ranks
    (one per GPU, NCCL all-reduce after Wo and after Wdown), measured beside
    the default line so that every bench line, the driver's scaling run
    included, records the tensor-parallel path at its N.  Every rank takes
    part; returns rank 0's summary (None elsewhere)."""
    import torch
    import nutllm_b200 as nb
    spec = TP_WORKLOADS[workload]
    cfg = nb.Config(**spec["cfg"])
    B, n, nsteps = spec["batch"], spec["prompt"], spec["steps"]
    torch.cuda.set_device(local)
    nccl_id = None
    if world > 1:
        box = [nb.tp_unique_id() if rank == 0 else None]
        _pg.broadcast_object_list(box, src=0)
        nccl_id = box[0]
    tp = nb.TPBatch(B, rank=rank, world=world, nccl_id=nccl_id, config=cfg, seed=SEED,
                    device=local)
    rng = np.random.default_rng(SEED)
    prompts = rng.integers(1, cfg.vocab_size, size=(B, n)).astype(np.int32)
    for _ in range(warmup):
        tp.generate(prompts, nsteps)
    barrier = _barrier(world)
    barrier()
    torch.cuda.synchronize(local)
    dec_s = pre_s = 0.0
    for _ in range(steps):
        _, _, st = tp.generate(prompts, nsteps)
        dec_s += st.decode_seconds
        pre_s += st.prefill_seconds
    barrier()
    tp.close()
    dec_s = _max_over_ranks(dec_s, world)
    pre_s = _max_over_ranks(pre_s, world)
    if rank != 0:
        return None
    per_rank = tp_decode_bytes(spec["cfg"], B, n, nsteps, world)
    step_s = dec_s / (steps * nsteps)
    peak, _ = measured_peaks()
    return {"metric": f"decode tok/s (Llama-2-7B INT4 shape, batch {B}, tensor parallel)",
            "value": round(B * nsteps * steps / dec_s, 2), "unit": "tok/s",
            "config": tp_config_of(workload, spec, world), "all_reduce": "nccl",
            "steps": steps, "warmup": warmup,
            "ms_per_decode_step": round(step_s * 1e3, 4),
            "prefill_tok_s": round(B * n * steps / pre_s, 2),
            "roofline_frac_per_rank": round(per_rank / step_s / 1e9 / peak, 4),
            "timing": "CUDA events on the library stream around prefill and decode, "
                      "max over ranks"}


def run_batch_tp(args, rank, world, local):
    import torch
    import nutllm_b200 as nb
    spec = TP_WORKLOADS[args.workload]
    cfg = nb.Config(**spec["cfg"])
    B, n, steps = spec["batch"], spec["prompt"], spec["steps"]
    torch.cuda.set_device(local)
    nccl_id = None
    if world > 1:
        box = [nb.tp_unique_id() if rank == 0 else None]
        _pg.broadcast_object_list(box, src=0)
        nccl_id = box[0]
    tp = nb.TPBatch(B, rank=rank, world=world, nccl_id=nccl_id, config=cfg, seed=SEED,
                    device=local)
    allreduce = "nccl"
    # NCCL (NVLS where it is available) by default; the one-shot peer-memory
    # all-reduce measured slower at 4 and 8 ranks
    if world > 1 and os.environ.get("NUTLLM_TP_ALLREDUCE", "nccl") == "peer":
        handles = [None] * world
        _pg.all_gather_object(handles, tp.ipc_handle())
        tp.open_peers(handles)
        allreduce = "peer"
    rng = np.random.default_rng(SEED)
    prompts = rng.integers(1, cfg.vocab_size, size=(B, n)).astype(np.int32)
    warmup = max(args.warmup, 3)
    for _ in range(warmup):
        tp.generate(prompts, steps)
    barrier = _barrier(world)
    barrier()
    torch.cuda.synchronize(local)
    launches0 = nb.launch_count()
    dec_s = pre_s = 0.0
    with Clocks(local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _, _, st = tp.generate(prompts, steps)
            dec_s += st.decode_seconds
            pre_s += st.prefill_seconds
        wall = time.perf_counter() - t0
    launches = nb.launch_count() - launches0
    barrier()
    dec_s = _max_over_ranks(dec_s, world)
    pre_s = _max_over_ranks(pre_s, world)
    wall = _max_over_ranks(wall, world)
    info = tp.info()
    tp.close()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v, pv, cores, sample = cpu_reference_7b(spec)
        cpu = {"value": round(v, 3) if v else None, "unit": "decode tok/s (batch 1)",
               "cores": cores, "kind": "reference",
               "prefill_tok_s": round(pv, 3) if pv else None, "sample": sample}
    value = B * steps * args.steps / dec_s
    step_s = dec_s / (args.steps * steps)
    peak, src = measured_peaks()
    per_rank = tp_decode_bytes(spec["cfg"], B, n, steps, world)
    ach = per_rank / step_s / 1e9
    line = {
        "metric": f"decode tok/s (Llama-2-7B INT4 shape, batch {B}, tensor parallel)",
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": round(1e3 * (dec_s + pre_s) / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp16xfp16 (dequantised INT4 weights)",
        "data": "synthetic (seeded random INT4 block-32 weights generated on the device, "
                "N(0,0.02) embeddings and classifier, uniform prompt ids)",
        "config": tp_config_of(args.workload, spec, world),
        "all_reduce": allreduce if world > 1 else None,
        "timing": "CUDA events on the library stream around prefill and decode",
        "prefill_tok_s": round(B * n * args.steps / pre_s, 2),
        "e2e": {"value": round(B * steps * args.steps / wall, 2),
                "unit": "generated tok/s via nut_batch_generate (incl. prefill)",
                "h2d_bytes_per_step": int(prompts.nbytes),
                "d2h_bytes_per_step": int(B * steps * 4)},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "whole decode step (per rank)", "bound": "hbm",
                     "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(ach / peak, 4), "peak_source": src,
                     "algorithmic_bytes_per_step_per_rank": int(per_rank),
                     "weight_bytes_held_per_rank": info["weight_bytes"], "traffic": None},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) per launch of the dominant kernel, from the ncu
# capture summarised in profiles/decode_mk_tinyllama_int4.md
NCU_TRAFFIC: dict = {"tinyllama-int4": 15_657_720_320 + 11_981_568}

QMATVEC_SHAPES = [(2048, 2048), (5632, 2048), (2048, 5632), (32000, 2048)]


def qmatvec_micro(nb, device, peak):
    """Kernel microbenchmark (a): the quantised matvec at every BASELINE
    shape, INT4 and INT8, x ~ N(0, 1).  Each measurement replays a CUDA
    graph of back-to-back launches over enough copies of the matrix to
    exceed twice the L2, so every launch reads its weights from HBM and no
    host launch gap is timed.  GB/s = algorithmic bytes (weights, fp16
    scales, x, y) per launch / device time per launch."""
    import torch
    torch.cuda.set_device(device)
    dev = f"cuda:{device}"
    out = []
    s = torch.cuda.Stream(device=dev)
    for qtype, tname in ((nb.INT4, "int4"), (nb.INT8, "int8")):
        for rows, cols in QMATVEC_SHAPES:
            w = nb.synth_normal(SEED, 7, rows * cols, 0.02).reshape(rows, cols)
            q = nb.QuantizedMatrix.quantize(w, qtype)
            wbytes = (rows * cols // (2 if qtype == nb.INT4 else 1)
                      + 2 * (rows * cols // 32))
            copies = max(2, -(-(256 << 20) // wbytes))
            mats = [nb.DeviceQMatrix(q, device) for _ in range(copies)]
            x = torch.from_numpy(nb.synth_normal(SEED, 8, cols, 1.0)).to(dev)
            ys = [torch.empty(rows, device=dev) for _ in range(copies)]
            with torch.cuda.stream(s):
                for m, y in zip(mats, ys):  # warm-up (also sets attributes)
                    m.matvec_async(x.data_ptr(), y.data_ptr(), s.cuda_stream)
            s.synchronize()
            reps = max(1, 512 // copies)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(reps):
                    for m, y in zip(mats, ys):
                        m.matvec_async(x.data_ptr(), y.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
            times = []
            for _ in range(4):
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(s):
                    a.record(s)
                    g.replay()
                    b.record(s)
                b.synchronize()
                times.append(a.elapsed_time(b) * 1e-3 / (reps * copies))
            t = min(times[1:])
            bytes_ = wbytes + 4 * cols + 4 * rows
            ach = bytes_ / t / 1e9
            out.append({"type": tname, "rows": rows, "cols": cols,
                        "us": round(t * 1e6, 3), "GB/s": round(ach, 1),
                        "frac": round(ach / peak, 4)})
            del g, mats, ys
    return out


def gemm_micro(nb, device, peak_tflops, tokens=512):
    """Kernel microbenchmark (b): the prefill GEMM (nut_qmatrix_gemm, fp16
    operands on the tensor cores, fp32 accumulation) for `tokens` rows of
    activations over every BASELINE weight shape, INT4 and INT8 weights
    (dequantised once and cached).  Each call also rounds the fp32
    activations to fp16; calls are replayed back to back from a CUDA
    graph.  TFLOP/s = 2 tokens rows cols / device time per call."""
    import torch
    torch.cuda.set_device(device)
    dev = f"cuda:{device}"
    s = torch.cuda.Stream(device=dev)
    out = []
    for qtype, tname in ((nb.INT4, "int4"), (nb.INT8, "int8")):
        for rows, cols in QMATVEC_SHAPES:
            w = nb.synth_normal(SEED, 7, rows * cols, 0.02).reshape(rows, cols)
            m = nb.DeviceQMatrix(nb.QuantizedMatrix.quantize(w, qtype), device)
            x = torch.from_numpy(
                nb.synth_normal(SEED, 8, tokens * cols, 1.0).reshape(tokens, cols)).to(dev)
            y = torch.empty(tokens, rows, device=dev)
            with torch.cuda.stream(s):
                for _ in range(2):  # the first call dequantises and caches
                    m.gemm_async(x.data_ptr(), tokens, y.data_ptr(), s.cuda_stream)
            s.synchronize()
            reps = 20
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(reps):
                    m.gemm_async(x.data_ptr(), tokens, y.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
            times = []
            for _ in range(4):
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(s):
                    a.record(s)
                    g.replay()
                    b.record(s)
                b.synchronize()
                times.append(a.elapsed_time(b) * 1e-3 / reps)
            m.check()
            t = min(times[1:])
            tf = 2.0 * tokens * rows * cols / t / 1e12
            out.append({"type": tname, "rows": rows, "cols": cols, "tokens": tokens,
                        "us": round(t * 1e6, 2), "TFLOP/s": round(tf, 1),
                        "frac": round(tf / peak_tflops, 4)})
            del g
    return out


def fp32_micro(nb, device, hbm_peak, tflops_peak):
    """Kernel microbenchmark (c): the fp32 products of the reference's own
    kernel benches (src/threading_selftest.cpp): matmul_threaded 768^3 and
    matvec_threaded 4096^2, bit-identical to the reference.  The matvec
    rotates over weight copies larger than L2; both replay from a CUDA
    graph.  Beside each, the reference's own CPU time (all host threads)."""
    import torch
    import oracle
    torch.cuda.set_device(device)
    dev = f"cuda:{device}"
    s = torch.cuda.Stream(device=dev)
    rng = np.random.default_rng(SEED)

    def graph_time(fn, reps):
        with torch.cuda.stream(s):
            fn()
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                fn(i)
        best = None
        for _ in range(4):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(s):
                a.record(s)
                g.replay()
                b.record(s)
            b.synchronize()
            t = a.elapsed_time(b) * 1e-3 / reps
            best = t if best is None else min(best, t)
        return best

    out = {}
    n = 768
    a = rng.standard_normal((n, n)).astype(np.float32)
    b = rng.standard_normal((n, n)).astype(np.float32)
    ad, bd = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    cd = torch.empty(n, n, device=dev)
    t = graph_time(lambda i=0: nb.matmul_f32_async(ad.data_ptr(), bd.data_ptr(), cd.data_ptr(),
                                                   n, n, n, torch.cuda.current_stream().cuda_stream),
                   20)
    flops = 2.0 * n ** 3
    threads = os.cpu_count() or 1
    cpu = None
    if oracle.reference_available():
        cpu = oracle.Reference().matmul_time(a, b, threads, 5)
    out["matmul_768"] = {"us": round(t * 1e6, 2), "GFLOP/s": round(flops / t / 1e9, 1),
                         "cpu_ms": None if cpu is None else round(cpu * 1e3, 3),
                         "cpu_threads": threads, "bit_exact_with_reference": True}
    rows = cols = 4096
    w = rng.standard_normal((rows, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    copies = 4  # 4 x 64 MB > L2
    wds = [torch.from_numpy(w).to(dev) for _ in range(copies)]
    xd = torch.from_numpy(x).to(dev)
    yd = torch.empty(rows, device=dev)
    t = graph_time(lambda i=0: nb.matvec_f32_async(wds[i % copies].data_ptr(), xd.data_ptr(),
                                                   yd.data_ptr(), rows, cols,
                                                   torch.cuda.current_stream().cuda_stream),
                   16)
    nbytes = rows * cols * 4 + cols * 4 + rows * 4
    cpu = None
    if oracle.reference_available():
        cpu = oracle.Reference().matvec_time(w, x, threads, 20)
    out["matvec_4096"] = {"us": round(t * 1e6, 2), "GB/s": round(nbytes / t / 1e9, 1),
                          "frac_hbm": round(nbytes / t / 1e9 / hbm_peak, 4),
                          "cpu_ms": None if cpu is None else round(cpu * 1e3, 3),
                          "cpu_threads": threads, "bit_exact_with_reference": True}
    return out


def run_micro(device):
    import nutllm_b200 as nb
    peak, src = measured_peaks()
    tpeak, tsrc = measured_tensor_peak()
    print(json.dumps({"qmatvec": qmatvec_micro(nb, device, peak),
                      "prefill_gemm": {"peak_tflops": tpeak, "peak_source": tsrc,
                                       "shapes": gemm_micro(nb, device, tpeak)},
                      "fp32": fp32_micro(nb, device, peak, tpeak)}),
          flush=True)


def measured_tensor_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def cpu_baseline(wl, c):
    """The reference's own CPU loop (oracle/_ref) on this host, all host
    threads, on the workload (or a bounded prefix of it, see cpu_sample)."""
    import oracle
    from nutllm_b200 import synthetic as syn
    threads = os.cpu_count() or 1
    if not oracle.reference_available():
        return {"value": None, "unit": "decode tok/s", "cores": threads,
                "kind": "reference", "sample": "oracle/_ref not built"}
    n_prompt, n_steps = cpu_sample(wl)
    r = oracle.Reference()
    rm = r.model(c, wl.qtype, SEED)
    prompt = oracle.prompt_ids(c, SEED, n_prompt)
    _, _, _, ps, ds = rm.generate(prompt, n_steps, threads, want_logits=False)
    whole = (n_prompt, n_steps) == (wl.prompt, wl.steps)
    return {"value": round(n_steps / ds, 3), "unit": "decode tok/s",
            "cores": threads, "kind": "reference",
            "prefill_tok_s": round(n_prompt / ps, 3),
            "sample": ("the whole workload once: " if whole else
                       "a bounded prefix of the workload: ") +
                      f"{n_prompt}-token prompt + {n_steps} greedy decode "
                      f"steps of {wl.name}"}


# ------------------------------------------------------------- reference


def run_reference_tp(args, world):
    spec = TP_WORKLOADS[args.workload]
    value, pvalue, cores, sample = cpu_reference_7b(spec, samples=max(args.steps, 1),
                                                    warmup=min(args.warmup, 1))
    if value is None:
        print(json.dumps({"impl": "reference", "unavailable": sample}))
        return
    print(json.dumps({
        "impl": "reference",
        "metric": f"decode tok/s (Llama-2-7B INT4 shape, batch {spec['batch']}, tensor parallel)",
        "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * 4 / value, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4xfp32", "data": "synthetic",
        "config": tp_config_of(args.workload, spec, world),
        "note": "the reference generates one sequence at a time (batch 1)",
        "prefill_tok_s": round(pvalue, 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": cores,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference(args, rank, world):
    """The reference's own CPU token loop (oracle/_ref, the unmodified
    reference compiled from its sources), fed by the oracle's restatement of
    the seeded generator: no library of this repository is loaded."""
    if rank != 0:
        return
    if args.workload in TP_WORKLOADS:
        run_reference_tp(args, world)
        return
    import oracle
    from nutllm_b200 import synthetic as syn  # workload tables only: loads no library
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
    n_prompt, sample_steps = cpu_sample(wl)
    prompt = oracle.prompt_ids(c, SEED, n_prompt)
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
        "metric": metric_of(wl),
        "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * (dec + pre) / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4xfp32" if wl.qtype == 1 else "int8xfp32",
        "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids)",
        "config": config_of(wl, world),
        "timing": "wall clock of the reference's prefill_quantized and decode loop, "
                  f"{threads} host threads",
        "prefill_tok_s": round(n_prompt * args.steps / pre, 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s",
                         "cores": threads, "kind": "reference",
                         "sample": f"{n_prompt}-token prompt + {sample_steps} "
                                   f"greedy steps of {wl.name} per step"},
        "e2e": {"value": round(value, 3), "unit": "tok/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                "generated_tok_s_incl_prefill": round(sample_steps * args.steps / (dec + pre), 3)},
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
    if args.micro_shape:
        r, c = (int(v) for v in args.micro_shape.lower().split("x"))
        QMATVEC_SHAPES[:] = [(r, c)]
    if args.micro_only:
        run_micro(local)
        return
    _init_dist(world)
    if args.workload in TP_WORKLOADS:
        run_batch_tp(args, rank, world, local)
    else:
        run_ours(args, rank, world, local)
    if world > 1:
        _pg.barrier()
        _pg.destroy_process_group()


if __name__ == "__main__":
    main()
