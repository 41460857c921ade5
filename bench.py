#!/usr/bin/env python
"""Embedding-generation benchmark: BERT-base on B200, embeddings/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one forward of one length-ragged batch (256 rows x seq 256, valid
lengths U[32, 256]) through the library: token ids in, pooled + L2-normalised
f32 embeddings out.  Inputs are seeded synthetic token batches and the
weights are random-init N(0, 0.02) (no dataset or checkpoint exists offline).

Under torchrun each rank drives one GPU and processes its own shard of
batches (replicas, no collective on the data path); value is the whole-job
rows/s over the max-over-ranks device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "jammi-ai_b200"))

import numpy as np  # noqa: E402

WORKLOADS = {
    "bert-base-int8-s256": dict(arch="bert-base", fmt="int8", batch=256, seq=256, len_lo=32, len_hi=256),
    "bert-base-bf16-s256": dict(arch="bert-base", fmt="bf16", batch=256, seq=256, len_lo=32, len_hi=256),
}
DEFAULT_WORKLOAD = "bert-base-int8-s256"
POOL_BATCHES = 8  # distinct input batches cycled through the timed steps
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attention", default="mma", choices=["mma", "tcgen05"],
                    help="attention kernel for rows of <= 256 keys (jb_set_attention_tcgen05)")
    ap.add_argument("--quick", action="store_true",
                    help="device-timed steps only (no clock sampler, e2e loop or CPU leg); "
                         "for profiler captures")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.marks = []

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def mark(self):
        self.marks.append(sum(1 for _ in open(self.path)) if self.path else 0)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if len(self.marks) >= 2:
            sel = rows[self.marks[0]:self.marks[1]] or rows
        else:
            sel = rows
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in sel if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in sel if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in sel for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sel)}


def linear_flops(cfg: dict, tokens: int) -> float:
    """Algorithmic FLOPs of the six per-layer linears over `tokens` valid
    tokens: L * 2 * (4 H^2 + 2 H F) per token."""
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    return float(L) * 2.0 * (4 * H * H + 2 * H * F) * tokens


def cpu_sample(cfg: dict, lens_all, ids_all, budget_s: float, max_rows: int):
    """Time the CPU oracle (numpy f32 restatement of the reference forward;
    BLAS uses every host core) on rows of the same workload, one row per
    forward at its own length -- the reference pipeline pads to the longest
    row of its batch, so a one-row forward never computes padding."""
    from oracle import bert as ob
    w = _cpu_weights(cfg)
    bc = ob.BertConfig.from_dict(cfg)
    rows = 0
    t0 = time.perf_counter()
    for ids, n in zip(ids_all, lens_all):
        n = int(n)
        ob.bert_forward(w, bc, ids[None, :n], np.ones((1, n), np.uint32), dtype=np.float32)
        rows += 1
        if rows >= max_rows or time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return rows, dt


_CPU_W = {}


def _cpu_weights(cfg):
    from jammi_b200.synthetic import bert_weights
    key = json.dumps(cfg, sort_keys=True)
    if key not in _CPU_W:
        _CPU_W[key] = bert_weights(cfg, seed=0)
    return _CPU_W[key]


def arch_cfg(name):
    from jammi_b200 import synthetic
    return {"bert-base": synthetic.BERT_BASE, "bert-large": synthetic.BERT_LARGE,
            "minilm-l6": synthetic.MINILM_L6}[name]


def inputs(wl, seed, n_batches):
    from jammi_b200.synthetic import token_batch, uniform_lengths
    rng = np.random.default_rng(seed)
    lens = np.stack([uniform_lengths(rng, wl["batch"], wl["len_lo"], wl["len_hi"]) for _ in range(n_batches)])
    ids = np.stack([token_batch(rng, l, wl["seq"]) for l in lens])
    return ids, lens


def run_reference(args, wl):
    """The reference arm: the reference's CPU forward, restated (it cannot be
    built here), timed on the host cores over bounded samples of the same
    workload; rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cfg = arch_cfg(wl["arch"])
    ids, lens = inputs(wl, 1234, 1)
    rows_per_step = 2
    cursor = 0
    total_rows, total_t = 0, 0.0
    for step in range(args.warmup + args.steps):
        sl = slice(cursor, cursor + rows_per_step)
        r, dt = cpu_sample(cfg, lens[0][sl], ids[0][sl], 1e9, rows_per_step)
        cursor = (cursor + rows_per_step) % wl["batch"]
        if step >= args.warmup:
            total_rows += r
            total_t += dt
    value = total_rows / total_t
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": "embeddings/sec", "value": value, "unit": "embeddings/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total_t / args.steps, "higher_is_better": True,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "arch": wl["arch"], "rows_per_step": rows_per_step,
                   "seq": wl["seq"], "lengths": f"U[{wl['len_lo']},{wl['len_hi']}]"},
        "cpu_baseline": {"value": value, "unit": "embeddings/s", "cores": cores, "kind": "port",
                         "sample": f"{rows_per_step} rows per step, one row per forward at its own length, "
                                   "numpy f32 restatement of the reference CPU forward"},
        "e2e": {"value": value, "unit": "embeddings/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per GEMM launch,
# averaged over the four linears of one layer, from the ncu capture recorded
# in profiles/bert_base_int8_b256_s256_launches.md (same workload).
GEMM_TRAFFIC_PER_LAUNCH = {"bert-base-int8-s256": 158.9e6}


def main():
    args = parse()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
        return
    import torch
    import torch.distributed as dist
    from jammi_b200 import Bert, ops
    from jammi_b200.synthetic import bert_weights

    ops.set_attention_tcgen05(args.attention == "tcgen05")
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from jammi_b200.sharding import init_replica_group
        init_replica_group("nccl", timeout_s=180.0, device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = arch_cfg(wl["arch"])
    model = Bert.from_weights(bert_weights(cfg, seed=0), cfg, device=local, fmt=wl["fmt"])
    B, S = wl["batch"], wl["seq"]
    ids_np, lens_np = inputs(wl, 1000 + rank, POOL_BATCHES)
    d_ids = torch.from_numpy(ids_np.astype(np.int32)).to(dev)
    d_lens = torch.from_numpy(lens_np.astype(np.int32)).to(dev)
    out = torch.empty((B, cfg["hidden_size"]), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        j = i % POOL_BATCHES
        model.encode_device(d_ids[j], d_lens[j], out, stream=stream)

    for i in range(args.warmup):
        step(i)
    model.sync(stream)

    clocks = ClockSampler(local)
    if not args.quick:
        clocks.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(dev)
    clocks.mark()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks.mark()
    barrier()
    model.sync(stream)
    ms_dev = e0.elapsed_time(e1)
    ms = max_over_ranks(ms_dev)
    clk = clocks.stop()
    value = world * args.steps * B / (ms / 1000.0)
    # Kernel breakdown: a separate pass with per-launch CUDA events (which
    # run the forward launch by launch instead of as one CUDA graph, so they
    # stay out of the timed region above).
    prof_steps = min(args.steps, 10)
    model.profile_enable(True)
    for i in range(prof_steps):
        step(i)
    model.sync(stream)
    prof = model.profile_read()
    model.profile_enable(False)
    tokens = sum(int(lens_np[i % POOL_BATCHES].sum()) for i in range(prof_steps))

    if args.quick:
        if rank == 0:
            print(json.dumps({"quick": True, "value": value, "ms_per_step": ms / args.steps,
                              "kernel_ms_per_step": {k: v["ms"] / prof_steps for k, v in prof.items()}}))
        model.close()
        if world > 1:
            dist.destroy_process_group()
        return
    # e2e through the public host API: pinned host ids/lens in, host f32 out
    h_ids = torch.from_numpy(ids_np.astype(np.uint32).view(np.int32)).pin_memory().numpy().view(np.uint32)
    h_lens = torch.from_numpy(lens_np.astype(np.uint32).view(np.int32)).pin_memory().numpy().view(np.uint32)
    h_out = torch.empty((B, cfg["hidden_size"]), dtype=torch.float32).pin_memory().numpy()
    for i in range(min(args.warmup, 3)):
        model.encode(h_ids[i % POOL_BATCHES], h_lens[i % POOL_BATCHES], stream=stream, out=h_out)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        emb = model.encode(h_ids[i % POOL_BATCHES], h_lens[i % POOL_BATCHES], stream=stream, out=h_out)
    t_e2e = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e_value = world * args.steps * B / t_e2e
    assert emb.shape == (B, cfg["hidden_size"]) and np.isfinite(emb).all()

    peaks, peak_src = load_peaks()
    lin = prof["linear"]
    flops_per_step_avg = linear_flops(cfg, tokens) / prof_steps
    achieved_tflops = linear_flops(cfg, tokens) / (lin["ms"] / 1000.0) / 1e12 if lin["ms"] > 0 else None
    if wl["fmt"] == "int8":
        peak = 2.0 * peaks["bf16_tflops_sustained"]
        peak_note = f"int8 dense peak taken as 2 x {peak_src} bf16 sustained ({peaks['bf16_tflops_sustained']})"
    else:
        peak = peaks["bf16_tflops_sustained"]
        peak_note = f"{peak_src} bf16 sustained"
    launches_per_step = sum(v["launches"] for v in prof.values()) / prof_steps

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n_rows, dt = cpu_sample(cfg, lens_np[0], ids_np[0], 15.0, 64)
        cpu = {"value": n_rows / dt, "unit": "embeddings/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{n_rows} rows of batch 0 of this workload, one row per forward at its own "
                         "length, numpy f32 restatement of the reference CPU forward (BLAS on all cores)"}

    if rank == 0:
        line = {
            "metric": "embeddings/sec", "value": value, "unit": "embeddings/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8/bf16" if wl["fmt"] == "int8" else "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "arch": wl["arch"], "weights": wl["fmt"],
                       "global_batch": B * world, "batch_per_gpu": B, "seq_len": S,
                       "lengths": f"U[{wl['len_lo']},{wl['len_hi']}]",
                       "valid_tokens_per_step": tokens / prof_steps,
                       "parallelism": f"replicas{world}",
                       "l2": "inputs+activations per step exceed L2 (>1 GB streamed per step)"},
            "e2e": {"value": e2e_value, "unit": "embeddings/s",
                    "h2d_bytes_per_step": int(B * S * 4 + B * 4),
                    "d2h_bytes_per_step": int(B * cfg["hidden_size"] * 4)},
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "roofline": {"bound": "tensor", "kernel": "gemm_tc_kernel (all six linears)",
                         "achieved": achieved_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved_tflops / peak) if achieved_tflops else None,
                         "traffic": GEMM_TRAFFIC_PER_LAUNCH.get(args.workload),
                         "traffic_unit": "bytes per launch (mean of one layer's four linears)",
                         "traffic_source": "ncu --set full capture, "
                                           "profiles/bert_base_int8_b256_s256_launches.md",
                         "peak_source": peak_note,
                         "flops_per_step": flops_per_step_avg},
            "kernel_ms_per_step": {k: v["ms"] / prof_steps for k, v in prof.items()},
            "kernel_ms_source": f"separate {prof_steps}-step pass with per-launch CUDA events",
            "forward": "CUDA graph replay (captured on the second call of a shape)",
            "attention": args.attention,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
