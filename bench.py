#!/usr/bin/env python
"""Embedding-generation benchmark on B200: embeddings/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl ours|reference] [--rows R]

Default workload (the metric's "BERT-base int8 seq256"): BERT-base with int8
weights (per-output-channel scales) and per-token int8 activations, bf16
attention; a step is one forward of one length-ragged batch of 256 rows x
seq 256, valid lengths U[32, 256]: token ids in, pooled + L2-normalised f32
embeddings out.  Inputs are seeded synthetic token batches and the weights
are random-init N(0, 0.02) (no dataset or checkpoint exists offline).

One process drives all N devices (the rows are independent: no collective
exists on the data path).  Under torchrun, rank 0 does the work and the
other ranks exit at once; nothing initialises NCCL.

* ``value``: device-resident throughput.  Each device holds its own input
  batches; K steps are queued on every device, timed with CUDA events on
  each device's stream; value = N * K * B / the slowest device's time.
* ``e2e``: the product driver, ``jb_generate_embeddings`` over the N devices:
  N * K * B rows of the same workload as host token ids in, host f32
  [rows, H] out in row order plus the validity bitmap -- length bucketing,
  packing into pinned staging, H2D, forward, D2H and the scatter into row
  order all inside the timed region.

Other workloads: ``bert-base-bf16-s256`` (bf16 weights and activations),
``bert-large-int8-s512`` (24 layers, B 128, lengths lognormal(5.0, 0.6)
clipped to [8, 512], pre-quantised int8 weights with scales log-uniform in
[1e-3, 1e-1]), ``clip-vit-b32-bf16`` (CLIP ViT-B/32 vision tower, 512 images
of 224x224x3, pixels N(0, 1)), and ``sharded-job-int8``: 4,194,304 rows
(``--rows``) of lengths lognormal(4.5, 0.8) clipped to [8, 512] through the
driver in one call over N devices (value = e2e = rows/s host to host).
``sidecar-binary-1m``: the ANN sidecar insert on one device -- 1,048,576
unit-norm 768-wide f32 embedding rows (1% null in the validity bitmap) into
a Binary sidecar (jb_sidecar_add, then jb_sidecar_build: median threshold and
sign-packing); value = rows/s of create + add + build from device-resident
rows, e2e = the same from pinned host rows.  search_final for 64 queries
(k 10, oversample 32) is timed on one built sidecar.  The sidecar calls return when their work is done, so each
phase is timed on the host clock around a synchronised call.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "jammi-ai_b200"))

import numpy as np  # noqa: E402

WORKLOADS = {
    "bert-base-int8-s256": dict(kind="text", arch="bert-base", fmt="int8", batch=256, seq=256,
                                dist=("uniform", 32, 256)),
    "bert-base-bf16-s256": dict(kind="text", arch="bert-base", fmt="bf16", batch=256, seq=256,
                                dist=("uniform", 32, 256)),
    "bert-base-f16-s256": dict(kind="text", arch="bert-base", fmt="f16", batch=256, seq=256,
                               dist=("uniform", 32, 256)),
    "bert-large-int8-s512": dict(kind="text", arch="bert-large", fmt="int8", batch=128, seq=512,
                                 dist=("lognormal", 5.0, 0.6, 8, 512), prequantised=True),
    "clip-vit-b32-bf16": dict(kind="image", arch="vit-b32", fmt="bf16", batch=512),
    "sharded-job-int8": dict(kind="job", arch="bert-base", fmt="int8", batch=256, seq=512,
                             dist=("lognormal", 4.5, 0.8, 8, 512), rows=4_194_304),
    "sidecar-binary-1m": dict(kind="sidecar", rows=1_048_576, dim=768, null_frac=0.01, queries=64,
                              k=10, oversample=32),
}
DEFAULT_WORKLOAD = "bert-base-int8-s256"
POOL_BATCHES = 8      # distinct resident input batches cycled through the timed steps
PAD_MULTIPLE = 32     # the driver pads each batch's width to a multiple of 32 (few graph shapes)

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per GEMM launch,
# averaged over one layer's four linears, from an ncu capture of this
# workload (the capture's summary, command and date are in profiles/).
GEMM_TRAFFIC = {"bert-base-int8-s256": (160.0e6, "2026-12-02",
                                        "profiles/bert_base_int8_b256_s256_launches.md")}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--rows", type=int, default=None, help="rows of the sharded-job workload")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attention", default="default", choices=["default", "mma", "tcgen05"],
                    help="attention kernel (jb_set_attention_tcgen05); default: the library's")
    ap.add_argument("--quick", action="store_true",
                    help="device-timed steps only (no clock sampler, e2e or CPU leg); "
                         "for profiler captures")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p)), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of the benchmark's GPUs, every 100 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = ",".join(str(g) for g in gpus)
        self.proc = None
        self.path = None
        self.marks = []

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpus, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)

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
        sel = rows[self.marks[0]:self.marks[1]] if len(self.marks) >= 2 else rows
        sel = sel or rows
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        num = lambda v: v.replace(".", "").isdigit()
        sm = [float(r[1]) for r in sel if num(r[1])]
        mx = [float(r[2]) for r in sel if num(r[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in sel for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sel), "gpus": self.gpus}


# ── workload definitions ─────────────────────────────────────────────────────

def arch_cfg(name):
    from jammi_b200 import synthetic
    return {"bert-base": synthetic.BERT_BASE, "bert-large": synthetic.BERT_LARGE,
            "minilm-l6": synthetic.MINILM_L6}[name]


def lengths(rng, wl, n):
    from jammi_b200.synthetic import lognormal_lengths, uniform_lengths
    d = wl["dist"]
    if d[0] == "uniform":
        return uniform_lengths(rng, n, d[1], d[2])
    return lognormal_lengths(rng, n, d[1], d[2], d[3], d[4])


def dist_name(wl):
    d = wl.get("dist")
    if not d:
        return "50 tokens (49 patches + CLS)"
    return f"U[{d[1]},{d[2]}]" if d[0] == "uniform" else f"clip(lognormal({d[1]},{d[2]}),{d[3]},{d[4]})"


def text_batches(wl, seed, n_batches):
    from jammi_b200.synthetic import token_batch
    rng = np.random.default_rng(seed)
    lens = np.stack([lengths(rng, wl, wl["batch"]) for _ in range(n_batches)])
    ids = np.stack([token_batch(rng, l, wl["seq"]) for l in lens])
    return ids, lens


def job_rows(wl, rows, seed):
    """``rows`` rows of the workload's length distribution, packed as the
    driver takes them: (values u32, offsets u64[rows + 1]); ids uniform in
    [1000, 30521], [CLS]=101 first, [SEP]=102 last."""
    rng = np.random.default_rng(seed)
    lens = lengths(rng, wl, rows).astype(np.uint64)
    offsets = np.zeros(rows + 1, dtype=np.uint64)
    np.cumsum(lens, out=offsets[1:])
    values = rng.integers(1000, 30522, size=int(offsets[-1]), dtype=np.uint32)
    values[offsets[:-1].astype(np.int64)] = 101
    two = lens > 1
    values[(offsets[1:][two] - 1).astype(np.int64)] = 102
    return values, offsets, lens


def bert_weights(wl, cfg):
    """Random-init weights; for a pre-quantised workload the six linears of
    every layer are int8 with per-output-channel scales log-uniform in
    [1e-3, 1e-1] (``weight_q`` / ``weight_scale``)."""
    from jammi_b200.synthetic import bert_weights as bw
    w = bw(cfg, seed=0)
    if wl.get("prequantised"):
        from oracle.quant import LINEARS
        rng = np.random.default_rng(1)
        H, F = cfg["hidden_size"], cfg["intermediate_size"]
        for n in range(cfg["num_hidden_layers"]):
            for lin, (o, i) in zip(LINEARS, [(H, H)] * 4 + [(F, H), (H, F)]):
                k = f"encoder.layer.{n}.{lin}"
                s = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), size=o)).astype(np.float32)
                q = np.clip(np.rint(w[k + ".weight"] / s[:, None]), -127, 127).astype(np.int8)
                del w[k + ".weight"]
                w[k + ".weight_q"] = q
                w[k + ".weight_scale"] = s
    return w


def float_weights(w):
    """The f32 weights a CPU forward uses for a pre-quantised checkpoint: q * s."""
    out = {}
    for k, v in w.items():
        if k.endswith(".weight_q"):
            out[k[:-2]] = v.astype(np.float32) * w[k[:-2] + "_scale"][:, None]
        elif not k.endswith(".weight_scale"):
            out[k] = v
    return out


def vit_cfg():
    from oracle import clip as oc
    return oc.ClipVisionConfig()


# ── algorithmic work ─────────────────────────────────────────────────────────

def linear_flops(cfg, tokens):
    """L * 2 * (4 H^2 + 2 H F) per valid token: the six per-layer linears."""
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    return float(L) * 2.0 * (4 * H * H + 2 * H * F) * tokens


def attention_flops(cfg, sum_n2):
    """L * 4 * H * n^2 per row (QK^T and PV over the valid keys)."""
    return float(cfg["num_hidden_layers"]) * 4.0 * cfg["hidden_size"] * sum_n2


def memory_bytes(cfg, fmt, tokens, rows):
    """Algorithmic DRAM bytes of the memory-bound kernels of one forward,
    bf16 activations: embeddings + LN (read word and position rows, write the
    row, + its int8 copy and scale), per layer two LayerNorms (read 2H, write
    2H [+ H + 4]), for int8 the attention-output quantiser (read 2H, write
    H + 4) and the GELU quantiser (read 2F, write F + 4); the pool reads 2H
    per token and writes 4H per row."""
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    q = fmt == "int8"
    emb = 4 * H + 2 * H + (H + 4 if q else 0)
    ln = 2 * H + 2 * H + (H + 4 if q else 0)
    per_layer = 2 * ln + ((2 * H + H + 4) + (2 * F + F + 4) if q else 0)
    return float(tokens) * (emb + L * per_layer + 2 * H) + float(rows) * 4 * H


def vit_flops(cfg):
    """Per image: the 12 blocks' linears over 50 tokens, attention over 50
    keys, the patch embedding (a [49, 3072] x [3072, 768] GEMM) and the
    [768 -> 512] projection."""
    W, L, T = cfg.width, cfg.layers, cfg.tokens
    F = cfg.mlp
    patch_k = 3 * cfg.patch_size * cfg.patch_size
    lin = L * 2.0 * (4 * W * W + 2 * W * F) * T
    att = L * 4.0 * W * T * T
    return lin, att, 2.0 * (T - 1) * patch_k * W + 2.0 * W * cfg.embed_dim


# ── CPU baseline (the reference's CPU forward, restated) ────────────────────

def cpu_sample_text(wl, cfg, w_cpu, lens_all, ids_all, budget_s, max_rows):
    """The oracle's numpy f32 forward (BLAS on every host core), one row per
    forward at its own length: the reference pipeline pads to the longest
    row of its batch, so a one-row forward computes no padding."""
    from oracle import bert as ob
    bc = ob.BertConfig.from_dict(cfg)
    rows = 0
    t0 = time.perf_counter()
    for ids, n in zip(ids_all, lens_all):
        n = int(n)
        ob.bert_forward(w_cpu, bc, ids[None, :n], np.ones((1, n), np.uint32), dtype=np.float32)
        rows += 1
        if rows >= max_rows or time.perf_counter() - t0 > budget_s:
            break
    return rows, time.perf_counter() - t0


def cpu_sample_image(w, cfg, px, budget_s, max_rows):
    from oracle import clip as oc
    rows = 0
    t0 = time.perf_counter()
    while rows < max_rows and time.perf_counter() - t0 <= budget_s:
        oc.clip_vision_forward(w, cfg, px[rows % len(px):rows % len(px) + 1], dtype=np.float32)
        rows += 1
    return rows, time.perf_counter() - t0


def cpu_baseline(wl, budget_s=15.0):
    """The CPU baseline leg: rows of this workload through the oracle."""
    if wl["kind"] == "image":
        from oracle import clip as oc
        cfg = vit_cfg()
        w = oc.random_clip_weights(cfg, seed=0)
        px = np.random.default_rng(7).standard_normal((4, 3, 224, 224)).astype(np.float32)
        n, dt = cpu_sample_image(w, cfg, px, budget_s, 64)
        what = f"{n} images, one per forward"
    else:
        cfg = arch_cfg(wl["arch"])
        w = float_weights(bert_weights(wl, cfg))
        ids, lens = text_batches(wl, 1234, 1)
        n, dt = cpu_sample_text(wl, cfg, w, lens[0], ids[0], budget_s, 64)
        what = f"{n} rows of one batch of this workload, one row per forward at its own length"
    return {"value": n / dt, "unit": "embeddings/s", "cores": os.cpu_count(), "kind": "port",
            "cpu": cpu_model(),
            "sample": what + "; numpy f32 restatement of the reference CPU forward "
                             "(oracle/), BLAS on all host cores"}


def run_reference(args, wl):
    """The reference arm: the reference's CPU forward, restated (it cannot be
    built here), timed on the host cores over bounded samples of the same
    workload; rank 0 only."""
    rows_per_step = 2
    total_rows, total_t = 0, 0.0
    if wl["kind"] == "image":
        from oracle import clip as oc
        cfg = vit_cfg()
        w = oc.random_clip_weights(cfg, seed=0)
        px = np.random.default_rng(7).standard_normal((4, 3, 224, 224)).astype(np.float32)
        for step in range(args.warmup + args.steps):
            r, dt = cpu_sample_image(w, cfg, px, 1e9, rows_per_step)
            if step >= args.warmup:
                total_rows += r
                total_t += dt
    else:
        cfg = arch_cfg(wl["arch"])
        w = float_weights(bert_weights(wl, cfg))
        ids, lens = text_batches(wl, 1234, 1)
        cursor = 0
        for step in range(args.warmup + args.steps):
            sl = slice(cursor, cursor + rows_per_step)
            r, dt = cpu_sample_text(wl, cfg, w, lens[0][sl], ids[0][sl], 1e9, rows_per_step)
            cursor = (cursor + rows_per_step) % wl["batch"]
            if step >= args.warmup:
                total_rows += r
                total_t += dt
    value = total_rows / total_t
    line = {
        "impl": "reference", "metric": "embeddings/sec", "value": value, "unit": "embeddings/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total_t / args.steps, "higher_is_better": True,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "arch": wl["arch"], "rows_per_step": rows_per_step,
                   "lengths": dist_name(wl)},
        "cpu_baseline": {"value": value, "unit": "embeddings/s", "cores": os.cpu_count(), "kind": "port",
                         "cpu": cpu_model(),
                         "sample": f"{rows_per_step} rows per step, one row per forward at its own "
                                   "length, numpy f32 restatement of the reference CPU forward"},
        "e2e": {"value": value, "unit": "embeddings/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)


# ── the timed GPU arms ───────────────────────────────────────────────────────

def save_weights(w):
    from safetensors.numpy import save_file
    fd, path = tempfile.mkstemp(suffix=".safetensors")
    os.close(fd)
    save_file({k: np.ascontiguousarray(v) for k, v in w.items()}, path)
    return path


def device_timed(torch, n, steps, warmup, step_fn, streams):
    """Queues `warmup` then `steps` steps on every device (round robin from
    one thread: every call only enqueues), timing each device's steps with
    CUDA events on its stream; returns the slowest device's milliseconds."""
    for i in range(warmup):
        for d in range(n):
            step_fn(d, i)
    for d in range(n):
        torch.cuda.synchronize(d)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for d in range(n):
        with torch.cuda.device(d):
            ev[d][0].record(streams[d])
    for i in range(steps):
        for d in range(n):
            step_fn(d, i)
    for d in range(n):
        with torch.cuda.device(d):
            ev[d][1].record(streams[d])
    for d in range(n):
        torch.cuda.synchronize(d)
    ms = [ev[d][0].elapsed_time(ev[d][1]) for d in range(n)]
    return max(ms), ms


def run_text(args, wl, n, torch):
    from jammi_b200 import Bert, ops
    from jammi_b200.driver import generate_embeddings

    cfg = arch_cfg(wl["arch"])
    w = bert_weights(wl, cfg)
    path = save_weights(w)
    try:
        models = [Bert(path, cfg, device=d, fmt=wl["fmt"]) for d in range(n)]
    finally:
        os.unlink(path)
    B, S, H = wl["batch"], wl["seq"], cfg["hidden_size"]
    streams, d_ids, d_lens, outs, host = [], [], [], [], []
    for d in range(n):
        dev = torch.device("cuda", d)
        ids_np, lens_np = text_batches(wl, 1000 + d, POOL_BATCHES)
        host.append((ids_np, lens_np))
        d_ids.append(torch.from_numpy(ids_np.astype(np.int32)).to(dev))
        d_lens.append(torch.from_numpy(lens_np.astype(np.int32)).to(dev))
        outs.append(torch.empty((B, H), dtype=torch.float32, device=dev))
        streams.append(torch.cuda.Stream(device=dev))

    def step(d, i):
        j = i % POOL_BATCHES
        models[d].encode_device(d_ids[d][j], d_lens[d][j], outs[d], stream=streams[d])

    clocks = ClockSampler(range(n))
    if not args.quick:
        clocks.start()
    clocks.mark()
    ms, ms_dev = device_timed(torch, n, args.steps, args.warmup, step, streams)
    clocks.mark()
    # the sampler stops before the driver leg: nvidia-smi's queries take the
    # driver's locks, which stall a host loop that synchronises every batch
    clk = clocks.stop() if not args.quick else None
    for d in range(n):
        models[d].sync(streams[d])
    value = n * args.steps * B / (ms / 1000.0)

    # kernel classes: a separate pass on device 0 with per-launch CUDA events
    # (it runs the forward launch by launch instead of as one CUDA graph, so
    # it stays out of the timed region above)
    prof_steps = min(args.steps, 10)
    models[0].profile_enable(True)
    for i in range(prof_steps):
        step(0, i)
    models[0].sync(streams[0])
    prof = models[0].profile_read()
    models[0].profile_enable(False)
    lens0 = host[0][1]
    tokens = sum(int(lens0[i % POOL_BATCHES].sum()) for i in range(prof_steps))
    sum_n2 = sum(float((lens0[i % POOL_BATCHES].astype(np.float64) ** 2).sum()) for i in range(prof_steps))

    e2e = None
    if not args.quick:
        # the driver over the N devices: N * K * B rows of the same workload
        rows = n * args.steps * B
        values, offsets, _ = job_rows(wl, rows, seed=77)
        out = np.empty((rows, H), dtype=np.float32)            # caller-owned, pages mapped by
        validity = np.zeros((rows + 7) // 8, dtype=np.uint8)   # the warm-up call
        kw = dict(batch_rows=B, pad_multiple=PAD_MULTIPLE, out=out, validity=validity)
        # warm-up: a width is run eagerly the first time a handle sees it and
        # captured as a CUDA graph the second time (the steady state of a
        # long job, or of a service that calls the driver repeatedly)
        for _ in range(2):
            generate_embeddings(models, values, offsets, **kw)
        t0 = time.perf_counter()
        _, _, st = generate_embeddings(models, values, offsets, **kw)
        t_e2e = time.perf_counter() - t0
        assert np.isfinite(out).all() and st["valid_rows"] == rows
        e2e = {"value": rows / t_e2e, "unit": "embeddings/s",
               "h2d_bytes_per_step": int(st["h2d_bytes"] / args.steps),
               "d2h_bytes_per_step": int(st["d2h_bytes"] / args.steps),
               "path": f"jb_generate_embeddings over {n} device(s): host ids in, host f32 [rows, {H}] "
                       "+ validity bitmap out in row order; length bucketing, pinned staging, "
                       "H2D, forward, D2H and scatter inside the timed region",
               "rows": rows,
               "driver": {k: st[k] for k in ("seconds", "prepare_seconds", "pack_seconds",
                                             "scatter_seconds", "wait_seconds", "enqueue_seconds",
                                             "setup_seconds", "worker_seconds_max",
                                             "worker_seconds_min", "batches", "tokens")}}

    peaks, src = load_peaks()
    lin_ms, att_ms, mem_ms = (prof[k]["ms"] for k in ("linear", "attention", "memory"))
    lin_f = linear_flops(cfg, tokens)
    att_f = attention_flops(cfg, sum_n2)
    int8 = wl["fmt"] == "int8"
    peak = (2.0 if int8 else 1.0) * peaks["bf16_tflops"]
    mem_b = memory_bytes(cfg, wl["fmt"], tokens, prof_steps * B)
    ach = lin_f / (lin_ms / 1e3) / 1e12 if lin_ms > 0 else None
    traffic = GEMM_TRAFFIC.get(args.workload)
    roofline = {
        "bound": "tensor", "kernel": "gemm_tc_kernel (the six linears of every layer)",
        "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak if ach else None,
        "traffic": traffic[0] if traffic else None,
        "traffic_note": (f"bytes per GEMM launch, mean of one layer's four linears: a constant from "
                         f"the ncu capture of {traffic[1]} ({traffic[2]}), not re-measured by this run"
                         if traffic else "no capture of this workload"),
        "peak_source": (f"2 x {src} bf16 burst ({peaks['bf16_tflops']} TF/s; B200's dense int8 rate is "
                        "twice bf16): the linears are timed one launch at a time in a short pass"
                        if int8 else f"{src} bf16 burst ({peaks['bf16_tflops']} TF/s"
                        + ("; B200's dense f16 rate equals bf16's)" if wl["fmt"] == "f16" else ")")),
        "flops_per_step": lin_f / prof_steps,
        "attention": {"achieved": att_f / (att_ms / 1e3) / 1e12 if att_ms > 0 else None,
                      "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                      "frac": (att_f / (att_ms / 1e3) / 1e12) / peaks["bf16_tflops"] if att_ms > 0 else None,
                      "flops_per_step": att_f / prof_steps},
        "memory": {"bound": "hbm", "kernels": "embeddings+LN, LayerNorm(+quant), quantisers, pooling",
                   "achieved": mem_b / (mem_ms / 1e3) / 1e9 if mem_ms > 0 else None,
                   "peak": peaks["hbm_gbs"], "unit": "GB/s",
                   "frac": (mem_b / (mem_ms / 1e3) / 1e9) / peaks["hbm_gbs"] if mem_ms > 0 else None,
                   "bytes_per_step": mem_b / prof_steps},
    }
    line = {
        "metric": "embeddings/sec", "value": value, "unit": "embeddings/s", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "ms_per_step_per_device": [m / args.steps for m in ms_dev],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8/bf16" if int8 else wl["fmt"], "data": "synthetic",
        "config": {"workload": args.workload, "arch": wl["arch"], "weights": wl["fmt"],
                   "global_batch": B * n, "batch_per_gpu": B, "seq_len": S, "lengths": dist_name(wl),
                   "valid_tokens_per_step": tokens / prof_steps, "parallelism": f"replicas{n}",
                   "process": "one process drives every device; no collective",
                   "l2": "inputs + activations per step exceed L2 (> 1 GB streamed per step)"},
        "e2e": e2e,
        "gpu_launches": int(round(sum(v["launches"] for v in prof.values()) / prof_steps * args.steps * n)),
        "roofline": roofline,
        "kernel_ms_per_step": {k: v["ms"] / prof_steps for k, v in prof.items()},
        "kernel_ms_source": f"separate {prof_steps}-step pass on device 0 with per-launch CUDA events",
        "forward": "CUDA graph replay (captured on the second call of a shape)",
        "attention": args.attention,
        "clocks": clk,
    }
    for m in models:
        m.close()
    return line


def run_image(args, wl, n, torch):
    from jammi_b200 import OpenClipVisionTransformer
    from oracle import clip as oc
    cfg = vit_cfg()
    path = save_weights(oc.random_clip_weights(cfg, seed=0))
    try:
        models = [OpenClipVisionTransformer(path, cfg.to_open_clip_config(), device=d, fmt=wl["fmt"])
                  for d in range(n)]
    finally:
        os.unlink(path)
    B, E = wl["batch"], cfg.embed_dim
    pool = 2  # two resident batches of 308 MB per device
    streams, d_px, outs = [], [], []
    for d in range(n):
        dev = torch.device("cuda", d)
        g = torch.Generator(device=dev).manual_seed(1000 + d)
        d_px.append(torch.randn((pool, B, 3, 224, 224), generator=g, device=dev, dtype=torch.float32))
        outs.append(torch.empty((B, E), dtype=torch.float32, device=dev))
        streams.append(torch.cuda.Stream(device=dev))

    def step(d, i):
        models[d].forward_image_device(d_px[d][i % pool], outs[d], stream=streams[d])

    clocks = ClockSampler(range(n))
    if not args.quick:
        clocks.start()
    clocks.mark()
    ms, ms_dev = device_timed(torch, n, args.steps, args.warmup, step, streams)
    clocks.mark()
    clk = clocks.stop() if not args.quick else None
    value = n * args.steps * B / (ms / 1000.0)
    prof_steps = min(args.steps, 10)
    models[0].profile_enable(True)
    for i in range(prof_steps):
        step(0, i)
    models[0].sync(streams[0])
    prof = models[0].profile_read()
    models[0].profile_enable(False)
    e2e = None
    if not args.quick:
        # jb_encode_image per device from one host thread each: pinned host
        # pixels in (H2D inside the call), host f32 embeddings out
        h_px = [torch.from_numpy(np.random.default_rng(d).standard_normal((B, 3, 224, 224))
                                 .astype(np.float32)).pin_memory().numpy() for d in range(n)]
        steps_e2e = max(3, args.steps // 10)
        with cf.ThreadPoolExecutor(n) as ex:
            # two warm-up calls: each chunk's forward graph is captured on the
            # second call a handle sees it
            for _ in range(2):
                list(ex.map(lambda d: models[d].forward_image(h_px[d], stream=streams[d]), range(n)))
            t0 = time.perf_counter()
            list(ex.map(lambda d: [models[d].forward_image(h_px[d], stream=streams[d])
                                   for _ in range(steps_e2e)], range(n)))
            t = time.perf_counter() - t0
        e2e = {"value": n * steps_e2e * B / t, "unit": "embeddings/s",
               "h2d_bytes_per_step": B * 3 * 224 * 224 * 4, "d2h_bytes_per_step": B * E * 4,
               "path": "jb_encode_image: pinned host f32 pixels in, host f32 embeddings out, "
                       f"one host thread per device, {steps_e2e} steps"}
    peaks, src = load_peaks()
    lin, att, extra = vit_flops(cfg)
    lin_ms, att_ms = prof["linear"]["ms"], prof["attention"]["ms"]
    ach = (lin + extra) * B * prof_steps / (lin_ms / 1e3) / 1e12 if lin_ms > 0 else None
    line = {
        "metric": "embeddings/sec", "value": value, "unit": "embeddings/s", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "ms_per_step_per_device": [m / args.steps for m in ms_dev],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": args.workload, "arch": "CLIP ViT-B/32 vision tower", "weights": "bf16",
                   "global_batch": B * n, "batch_per_gpu": B, "image": "224x224x3, pixels N(0,1)",
                   "parallelism": f"replicas{n}", "process": "one process drives every device",
                   "l2": "308 MB of pixels per step, larger than L2"},
        "e2e": e2e,
        "gpu_launches": int(round(sum(v["launches"] for v in prof.values()) / prof_steps * args.steps * n)),
        "roofline": {"bound": "tensor", "kernel": "gemm_tc_kernel (patch embedding, block linears, projection)",
                     "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": ach / peaks["bf16_tflops"] if ach else None, "traffic": None,
                     "peak_source": f"{src} bf16 burst",
                     "flops_per_step": (lin + extra) * B,
                     "attention": {"achieved": att * B * prof_steps / (att_ms / 1e3) / 1e12 if att_ms > 0 else None,
                                   "unit": "TFLOP/s", "flops_per_step": att * B}},
        "kernel_ms_per_step": {k: v["ms"] / prof_steps for k, v in prof.items()},
        "kernel_ms_source": f"separate {prof_steps}-step pass on device 0 with per-launch CUDA events",
        "clocks": clk,
    }
    for m in models:
        m.close()
    return line


def run_job(args, wl, n, torch):
    """The sharded job: all rows through jb_generate_embeddings in one call."""
    from jammi_b200 import Bert
    from jammi_b200.driver import generate_embeddings
    cfg = arch_cfg(wl["arch"])
    path = save_weights(bert_weights(wl, cfg))
    try:
        models = [Bert(path, cfg, device=d, fmt=wl["fmt"]) for d in range(n)]
    finally:
        os.unlink(path)
    H, B = cfg["hidden_size"], wl["batch"]
    rows = args.rows or wl["rows"]
    values, offsets, lens = job_rows(wl, rows, seed=4242)
    out = np.empty((rows, H), dtype=np.float32)                 # caller-owned: its pages are
    out.fill(0.0)                                               # mapped before the timed call
    validity = np.zeros((rows + 7) // 8, dtype=np.uint8)
    kw = dict(batch_rows=B, pad_multiple=PAD_MULTIPLE)
    # warm-up: a 1/64 sample of the rows (every width class twice or more,
    # so each device captures its graphs before the timed call)
    ws = max(1, rows // 64)
    generate_embeddings(models, values[: int(offsets[ws])], offsets[: ws + 1], **kw)
    clocks = ClockSampler(range(n))
    clocks.start()
    clocks.mark()
    t0 = time.perf_counter()
    _, _, st = generate_embeddings(models, values, offsets, out=out, validity=validity, **kw)
    t = time.perf_counter() - t0
    clocks.mark()
    clk = clocks.stop()
    assert st["valid_rows"] == rows and np.isfinite(out[:: max(1, rows // 4096)]).all()
    value = rows / t
    peaks, src = load_peaks()
    tokens = float(lens.sum())
    lin_f = linear_flops(cfg, tokens)
    line = {
        "metric": "embeddings/sec", "value": value, "unit": "embeddings/s", "n_gpus": n,
        "steps": 1, "warmup": 1, "ms_per_step": 1000.0 * t,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8/bf16",
        "data": "synthetic",
        "config": {"workload": args.workload, "arch": wl["arch"], "weights": wl["fmt"], "rows": rows,
                   "lengths": dist_name(wl), "batch_rows": B, "valid_tokens": tokens,
                   "parallelism": f"length-bucketed batches pulled by one worker per device ({n})",
                   "value": "host ids in -> host f32 [rows, 768] + validity out, one driver call"},
        "e2e": {"value": value, "unit": "embeddings/s", "h2d_bytes_per_step": st["h2d_bytes"],
                "d2h_bytes_per_step": st["d2h_bytes"]},
        "driver": st,
        "linear_tflops_whole_job": lin_f / t / 1e12,
        "linear_frac_whole_job": lin_f / t / 1e12 / (2.0 * peaks["bf16_tflops"]),
        "clocks": clk,
    }
    for m in models:
        m.close()
    return line


def _sidecar_insert(L, lib, vectors_ptr, bits_ptr, rows, dim, keep=False):
    """One insert step through the C ABI (create, add, build); seconds of
    (add, build), the valid row count and the handle when kept."""
    import ctypes
    h = ctypes.c_void_p()
    L.check(lib.jb_sidecar_create(0, dim, 3, ctypes.byref(h)))
    try:
        added = ctypes.c_int64()
        t0 = time.perf_counter()
        L.check(lib.jb_sidecar_add(h, vectors_ptr, bits_ptr, rows, None, ctypes.byref(added)))
        t1 = time.perf_counter()
        L.check(lib.jb_sidecar_build(h, 1, None))
        t2 = time.perf_counter()
    except BaseException:
        lib.jb_sidecar_free(h)
        raise
    if not keep:
        lib.jb_sidecar_free(h)
        h = None
    return t1 - t0, t2 - t1, added.value, h


def _sidecar_search(L, lib, h, q_ptr, nq, k, over, keys, dist, steps, warmup):
    """Median seconds of one search_final call of nq queries on a built handle."""
    ts = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        L.check(lib.jb_sidecar_search_final(h, q_ptr, nq, k, over, keys.ctypes.data, dist.ctypes.data))
        if i >= warmup:
            ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def run_sidecar(args, wl, n, torch):
    """The ANN sidecar insert (write_batch -> add -> build) and search_final."""
    from jammi_b200 import _lib as L
    if n != 1:
        raise SystemExit("the sidecar workload runs on one device")
    lib = L.lib()
    rows, dim, nq, k, over = wl["rows"], wl["dim"], wl["queries"], wl["k"], wl["oversample"]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    vec = torch.randn((rows, dim), generator=g, device=dev, dtype=torch.float32)
    vec /= vec.norm(dim=1, keepdim=True)
    ok = np.random.default_rng(12).random(rows) >= wl["null_frac"]
    bits = np.packbits(ok, bitorder="little")
    bits_d = torch.from_numpy(bits).to(dev)
    q = (vec[:nq] + 0.05 * torch.randn((nq, dim), generator=g, device=dev)).contiguous()
    keys = np.empty((nq, k), np.int64)
    dist = np.empty((nq, k), np.float32)
    torch.cuda.synchronize()

    def leg(vp, bp, steps, warmup):
        out = []
        for i in range(warmup + steps):
            r = _sidecar_insert(L, lib, vp, bp, rows, dim)
            if i >= warmup:
                out.append(r)
        return out

    clocks = ClockSampler([0])
    clocks.start()
    clocks.mark()
    dev_leg = leg(vec.data_ptr(), bits_d.data_ptr(), args.steps, args.warmup)
    clocks.mark()
    clk = clocks.stop()
    valid = dev_leg[0][2]
    assert valid == int(ok.sum())
    h_vec = vec.cpu().pin_memory()
    h_bits = torch.from_numpy(bits).pin_memory()
    h_q = q.cpu().pin_memory()
    e2e_steps = max(3, min(args.steps, 10))
    host_leg = leg(h_vec.data_ptr(), h_bits.data_ptr(), e2e_steps, 2)
    med = lambda xs: statistics.median(xs)
    t_add, t_build = (med([r[i] for r in dev_leg]) for i in range(2))
    h_add, h_build = (med([r[i] for r in host_leg]) for i in range(2))
    # search_final on one built sidecar (a service's steady state): device
    # queries and host results, then host queries and host results
    _, _, _, h = _sidecar_insert(L, lib, vec.data_ptr(), bits_d.data_ptr(), rows, dim, keep=True)
    try:
        t_search = _sidecar_search(L, lib, h, q.data_ptr(), nq, k, over, keys, dist, 20, 3)
        h_search = _sidecar_search(L, lib, h, h_q.data_ptr(), nq, k, over, keys, dist, 20, 3)
    finally:
        lib.jb_sidecar_free(h)
    # algorithmic bytes of add + build: read every input row, write the valid
    # ones to the store, read the store back for the codes, write the codes,
    # read the threshold sample once
    nb = (dim + 7) // 8
    sample = min(valid, 100_000)
    alg = rows * 4 * dim + valid * (4 * dim + 4 * dim + nb) + sample * 4 * dim
    peaks, src = load_peaks()
    ach = alg / (t_add + t_build) / 1e9
    line = {
        "metric": "sidecar rows/sec", "value": rows / (t_add + t_build), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * (t_add + t_build),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32/u8",
        "data": "synthetic",
        "config": {"workload": args.workload, "rows": rows, "dim": dim, "valid_rows": valid,
                   "precision": "binary", "threshold": "median", "queries": nq, "k": k, "oversample": over,
                   "l2": f"{rows * dim * 4 / 1e9:.1f} GB of rows per step, larger than L2",
                   "timing": "host clock around each synchronised C-ABI call; median over steps"},
        "phases_ms": {"add": 1e3 * t_add, "build": 1e3 * t_build, "search_final": 1e3 * t_search},
        "search_final_queries_per_s": nq / t_search,
        "e2e": {"value": rows / (h_add + h_build), "unit": "rows/s", "h2d_bytes_per_step": rows * dim * 4 +
                len(bits) + nq * dim * 4, "d2h_bytes_per_step": nq * k * 12,
                "phases_ms": {"add": 1e3 * h_add, "build": 1e3 * h_build, "search_final": 1e3 * h_search},
                "path": "jb_sidecar_add from pinned host rows + bitmap, jb_sidecar_build, "
                        "jb_sidecar_search_final with host queries and results"},
        # per insert step: add = one counter reset + (compaction, counter
        # commit) per chunk of 131072 rows (device-resident rows are read in
        # place); build = the median threshold (init, four passes of histogram
        # + select, final) + packing
        "gpu_launches": args.steps * (1 + 2 * -(-rows // 131072) + (1 + 4 * 2 + 1) + 1),
        "roofline": {"bound": "hbm", "kernel": "add + build (compaction, threshold, sign-packing)",
                     "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": ach / peaks["hbm_gbs"], "traffic": None,
                     "peak_source": f"{src} copy bandwidth",
                     "bytes_per_step": alg},
        "clocks": clk,
    }
    return line


def sidecar_cpu_baseline(wl, sample_rows=65536):
    """The oracle's insert + build (numpy, one thread for the sort) on a sample."""
    from oracle import index as oi
    rng = np.random.default_rng(3)
    v = rng.standard_normal((sample_rows, wl["dim"])).astype(np.float32)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    bits = np.packbits(rng.random(sample_rows) >= wl["null_frac"], bitorder="little")
    t0 = time.perf_counter()
    store = oi.sidecar_add(v, bits)
    tau = oi.fit_binary_threshold(store, "median")
    oi.pack_threshold_bits(store, tau)
    dt = time.perf_counter() - t0
    return {"value": sample_rows / dt, "unit": "rows/s", "cores": 1, "kind": "port", "cpu": cpu_model(),
            "sample": f"{sample_rows} rows: oracle sidecar_add + median threshold + sign-packing (numpy)"}


def main():
    args = parse()
    wl = WORKLOADS[args.workload]
    rank, world, _ = dist_env()
    if rank != 0:
        return  # one process drives every device; the other ranks have no work
    n = max(args.gpus, 1)
    if args.impl == "reference":
        if wl["kind"] == "sidecar":
            cb = sidecar_cpu_baseline(wl)
            print(json.dumps({"impl": "reference", "metric": "sidecar rows/sec", "value": cb["value"],
                              "unit": "rows/s", "n_gpus": args.gpus, "steps": 1, "warmup": 0,
                              "higher_is_better": True, "dtype": "f32/u8", "data": "synthetic",
                              "config": {"workload": args.workload}, "cpu_baseline": cb, "vs_baseline": None,
                              "e2e": {"value": cb["value"], "unit": "rows/s", "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}), flush=True)
            return
        run_reference(args, wl)
        return
    import torch
    from jammi_b200 import ops
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        raise SystemExit(f"needs {n} CUDA device(s), found {torch.cuda.device_count()}")
    if args.attention != "default":
        ops.set_attention_tcgen05(args.attention == "tcgen05")
    if wl["kind"] == "text":
        line = run_text(args, wl, n, torch)
    elif wl["kind"] == "image":
        line = run_image(args, wl, n, torch)
    elif wl["kind"] == "sidecar":
        line = run_sidecar(args, wl, n, torch)
        line["cpu_baseline"] = sidecar_cpu_baseline(wl) if not args.no_cpu_baseline else None
        print(json.dumps(line), flush=True)
        return
    else:
        line = run_job(args, wl, n, torch)
    if args.quick:
        print(json.dumps({"quick": True, "value": line["value"], "ms_per_step": line["ms_per_step"],
                          "kernel_ms_per_step": line.get("kernel_ms_per_step")}), flush=True)
        return
    line["cpu_baseline"] = (cpu_baseline(wl) if n == 1 and not args.no_cpu_baseline
                            and wl["kind"] != "job" else None)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
