#!/usr/bin/env python
"""Benchmark of the palettized SAM3 ViT encoder hot path on B200.

Workload (one "step"): 64 seeded 1008x1008x3 fp16 images through the 32-block
palettized ViT encoder (D 1024, 16 heads, MLP 4096; every QKV / proj / fc1 /
fc2 weight uint8 indices + a 256-entry fp16 palette per output channel;
pruned to 2592 tokens by L2 norm after block 16), sharded by image over the
GPUs (64/N images per rank, no collectives on the data path), processed in
calls of --batch images. Synthetic data with the spec's distributions, random
weights of the spec's architecture.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torch.distributed.run (one rank per GPU). Rank 0 prints
one JSON line:
  value   images/s of the whole job, device-timed (CUDA events on the library's
          stream, inputs resident in HBM), max over ranks;
  e2e     the same through the host-buffer C-ABI entry point
          (sam3_encoder_forward_host_pipelined over all of the rank's images:
          pinned host images in, pruned features and indices out, every copy
          inside the timed region, overlapped with the encoder of the
          neighbouring call);
  roofline  the palette-dequant GEMM (dominant kernel): algorithmic FLOPs
          (2*M*N*K) / its summed CUDA-event launch time, measured in a second
          pass over the same steps with events around every launch (kept out
          of `value`: the events stop each kernel's start from overlapping
          the previous kernel's tail), against the measured sustained bf16
          tensor peak;
  cpu_baseline  the CPU oracle (a C++ restatement of the path) on a bounded
          sample, rank 0 at N=1 only.
--impl reference times the reference path's CPU restatement (the reference
itself is Swift/Metal and cannot run here) on the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "metal-sam-ios-experiments_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "encoder images/s at 1008^2 (32-block uint8-palettized ViT, prune to 2592 after block 16)"
UNIT = "images/s"
IMAGE = 1008
GRID = IMAGE // 14
SEQ = GRID * GRID
KEEP = SEQ // 2
DIM, HEADS, HIDDEN, BLOCKS = 1024, 16, 4096, 32


def workload_config(args, world):
    return {
        "workload": "c4 batched encoder: 64 seeded 1008x1008 images, 32-block uint8-palettized "
                    "ViT (D 1024, 16 heads, MLP 4096, per-output-channel 256-entry fp16 "
                    "palettes), 5184 tokens pruned to 2592 by L2 norm after block 16, "
                    "sharded by image",
        "images": args.images,
        "images_per_gpu": args.images // world,
        "batch_per_call": min(args.batch, args.images // world),
        "parallelism": f"dp{world} (image sharding, no collectives)",
        "l2": "inputs larger than L2: 554 MB of palettized weights and >126 MB of "
              "activations per call are streamed every step",
    }


def image_shard(rank, world, images):
    """Contiguous block of images owned by `rank`: (first global index, count).
    Images are independent, so the ranks exchange nothing."""
    if world <= 0 or images % world:
        raise ValueError(f"{images} images do not split evenly over {world} ranks")
    per = images // world
    return rank * per, per


def encoder_flops_per_image():
    lin_pre = 2.0 * SEQ * DIM * (3 * DIM + DIM + 2 * HIDDEN)
    lin_post = 2.0 * KEEP * DIM * (3 * DIM + DIM + 2 * HIDDEN)
    att_pre = 4.0 * HEADS * SEQ * SEQ * 64
    att_post = 4.0 * HEADS * KEEP * KEEP * 64
    patch = 2.0 * SEQ * DIM * 588
    return {"gemm": 16 * (lin_pre + lin_post), "attention": 16 * (att_pre + att_post),
            "patch": patch}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p["bf16_tflops_sustained"]),
                "hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0,
                "source": "fallback"}


def load_traffic():
    """Per-launch DRAM traffic of the GEMM from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "gemm_palette_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clock/throttle samples taken while the timed region runs."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            self.file.close()
            os.unlink(self.file.name)
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(", ") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        mine = [r for r in rows if len(r) >= 10 and (self.uuid is None or r[1].strip() == self.uuid)]
        if not mine:
            mine = [r for r in rows if len(r) >= 10]
        if not mine:
            return None
        sm = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in mine if r[3].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in mine for i in range(4) if r[6 + i].strip() == "Active"})
        loaded = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(mine)}


# ---------------------------------------------------------------- CPU oracle sample
def cpu_oracle_sample(repeats=1):
    """Per-image time of the CPU oracle on one 1008^2 image, extrapolated from a
    bounded sample: patch embedding + block 1 (5184 tokens) + prune + block 17
    (2592 tokens), with the two blocks weighted x16 each."""
    import numpy as np
    from oracle import oracle as O
    O.build()
    # every host core this process may run on (torch.distributed.run sets
    # OMP_NUM_THREADS=1 for each rank, which would time a single core)
    O.set_num_threads(len(os.sched_getaffinity(0)))
    blk_a = O.SyntheticBlock(7, 0)
    blk_b = O.SyntheticBlock(7, 16)
    img = O.gen_uniform(7, 1, (1, IMAGE, IMAGE, 3), -1.0, 1.0)
    pw = O.gen_normal(7, 2, (DIM, 3, 14, 14), 0.0, 0.02)
    pb = O.gen_normal(7, 3, (DIM,), 0.0, 0.02)
    table = O.rope_table(GRID, GRID)
    best = None
    for _ in range(repeats):
        t0 = time.perf_counter()
        x = O.patch_embed(img, pw, pb, 14)
        t1 = time.perf_counter()
        x = O.vit_block(x, 1, SEQ, HEADS, blk_a, table, SEQ)
        t2 = time.perf_counter()
        xp, rope_p, _ = O.prune(x, 1, SEQ, KEEP, rope=table, rope_period=SEQ)
        t3 = time.perf_counter()
        O.vit_block(xp, 1, KEEP, HEADS, blk_b, rope_p, KEEP)
        t4 = time.perf_counter()
        per_image = (t1 - t0) + 16 * (t2 - t1) + (t3 - t2) + 16 * (t4 - t3)
        best = per_image if best is None else min(best, per_image)
    return {"seconds_per_image": best, "cores": O.num_threads(),
            "sample": "1 image 1008^2: patch embed + block 1 (5184 tokens) + prune + block 17 "
                      "(2592 tokens) timed, blocks extrapolated x16 each to 32 blocks"}


# ---------------------------------------------------------------- synthetic weights
def make_weights(torch, sam3, device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    keep = []

    def t(x):
        keep.append(x)
        return x

    def lin(n, k):
        idx = t(torch.randint(0, 256, (n, k), generator=g, device=device, dtype=torch.uint8))
        pal = torch.randn((n, 256), generator=g, device=device) * 0.02
        pal = t(pal.half().float().sort(dim=1).values.half().contiguous())
        bias = t((torch.randn((n,), generator=g, device=device) * 0.01).half())
        return sam3.palette_linear(idx, pal, bias, n, k)

    ones = t(torch.ones(DIM, dtype=torch.float16, device=device))
    zeros = t(torch.zeros(DIM, dtype=torch.float16, device=device))
    blocks = [sam3.block_weights(ones, zeros, lin(3 * DIM, DIM), lin(DIM, DIM), ones, zeros,
                                 lin(HIDDEN, DIM), lin(DIM, HIDDEN)) for _ in range(BLOCKS)]
    pw = t((torch.randn((DIM, 3, 14, 14), generator=g, device=device) * 0.02).half())
    pb = t((torch.randn((DIM,), generator=g, device=device) * 0.02).half())
    w = sam3.encoder_weights(pw, pb, blocks)
    w._tensors = keep
    return w


# ---------------------------------------------------------------- arms
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    """CPU restatement of the reference path (the reference's Swift/Metal code
    cannot run here), timed on the host cores on the same workload and metric."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    samples = []
    for i in range(args.warmup + args.steps):
        r = cpu_oracle_sample(1)
        if i >= args.warmup:
            samples.append(r["seconds_per_image"])
    spi = statistics.median(samples)
    value = 1.0 / spi
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": spi * args.images * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16 storage, fp32 accumulate",
        "data": "synthetic", "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": r["sample"] + "; each step = one such sample"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    import sam3cuda as sam3

    world, rank, local = dist_env()
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    first, per_rank = image_shard(rank, world, args.images)
    batch = min(args.batch, per_rank)
    dev = torch.device("cuda", local)
    ctx = sam3.Context(local, max_batch=batch)
    w = make_weights(torch, sam3, dev, 1234)
    gen = torch.Generator(device=dev)
    imgs = torch.empty((per_rank, IMAGE, IMAGE, 3), dtype=torch.float16, device=dev)
    for i in range(per_rank):  # image i of the job is seeded by its global index
        gen.manual_seed(1000 + first + i)
        imgs[i] = (torch.rand((IMAGE, IMAGE, 3), generator=gen, device=dev) * 2 - 1).half()
    keep = ctx.out_tokens
    feats = torch.empty((per_rank, keep, DIM), dtype=torch.float16, device=dev)
    idx = torch.empty((per_rank, keep), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)

    def step():
        for c0 in range(0, per_rank, batch):
            n = min(batch, per_rank - c0)
            ctx.encoder_forward(imgs[c0].data_ptr(), n, w, feats[c0].data_ptr(),
                                idx[c0].data_ptr())

    def barrier():
        torch.cuda.synchronize()
        ctx.sync()
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    barrier()

    # ---- device-timed region (inputs resident in HBM)
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    launches0 = ctx.launches
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    ev1.synchronize()
    ctx.sync()
    launches = ctx.launches - launches0
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    barrier()
    ms_max = max_over_ranks(ms)
    launches_all = sum_over_ranks(launches)

    # ---- per-kernel device time: the same steps again with CUDA events
    # around every launch on the library's stream (these events keep each
    # kernel from overlapping the next one's start, so this pass is timed
    # separately from `value`)
    ctx.profile_enable(True)
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(args.steps):
        step()
    p1.record(stream)
    p1.synchronize()
    ctx.sync()
    prof = ctx.profile_read()
    ctx.profile_enable(False)
    prof_ms = p0.elapsed_time(p1)
    barrier()

    # ---- end to end through the host-buffer entry point
    h_imgs = torch.empty(imgs.shape, dtype=torch.float16, pin_memory=True)
    h_imgs.copy_(imgs)
    h_feats = torch.empty(feats.shape, dtype=torch.float16, pin_memory=True)
    h_idx = torch.empty(idx.shape, dtype=torch.int32, pin_memory=True)

    def step_e2e():
        # every image of this rank through the pipelined host entry point:
        # uploads of the next call and downloads of the previous one overlap
        # the encoder
        ctx.encoder_forward_host_pipelined(h_imgs.data_ptr(), per_rank, w, h_feats.data_ptr(),
                                           h_idx.data_ptr())

    step_e2e()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_e2e()
    e1.record(stream)
    e1.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()
    # the host-path result must equal the device-path result
    same = bool(torch.equal(h_idx.to(dev), idx)) and bool(torch.equal(h_feats.to(dev), feats))

    peaks = load_peaks()
    g = prof["gemm"]
    gemm_tflops = g["flops"] / (g["ms"] * 1e-3) / 1e12 if g["ms"] > 0 else 0.0
    a = prof["attention"]
    att_tflops = a["flops"] / (a["ms"] * 1e-3) / 1e12 if a["ms"] > 0 else 0.0
    traffic = load_traffic()
    result = None
    if rank == 0:
        value = args.images * args.steps / (ms_max * 1e-3)
        flops = encoder_flops_per_image()
        total_flops = sum(flops.values()) * args.images
        step_ms = ms_max / args.steps
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16 (uint8-palette weights expanded to fp16 on chip, fp32 accumulate)",
            "data": "synthetic", "config": workload_config(args, world),
            "e2e": {"value": args.images * args.steps / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": args.images * IMAGE * IMAGE * 3 * 2,
                    "d2h_bytes_per_step": args.images * keep * (DIM * 2 + 4),
                    "matches_device_path": same},
            "roofline": {
                "kernel": "gemm_ws_kernel + gemm_wsc_kernel (palette-dequant tcgen05 pair GEMMs: "
                          "QKV/proj/fc1/fc2, averaged over their launches)",
                "bound": "tensor", "achieved": gemm_tflops,
                "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": gemm_tflops / peaks["bf16_tflops_sustained"],
                "peak_kind": f"bf16_tflops_sustained ({peaks['source']})",
                "frac_of_burst_peak": gemm_tflops / peaks["bf16_tflops"],
                "traffic": traffic.get("bytes_per_launch_weighted") if traffic else None,
                "launches": g["launches"], "kernel_ms": g["ms"],
                "share_of_step": g["ms"] / prof_ms if prof_ms > 0 else None,
                "timing": "per-launch CUDA events in a second pass over the same steps "
                          f"({prof_ms / args.steps:.2f} ms per step with the events)",
            },
            "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 3),
                            "tflops": (v["flops"] / (v["ms"] * 1e-3) / 1e12) if v["ms"] and v["flops"] else None,
                            "gbs": (v["bytes"] / (v["ms"] * 1e-3) / 1e9) if v["ms"] and v["bytes"] else None}
                        for k, v in prof.items()},
            "attention_tflops": att_tflops,
            "whole_step_tflops": total_flops * args.steps / (ms_max * 1e-3) / 1e12,
            "gpu_launches": int(launches_all),
            "clocks": clk,
        }
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            r = cpu_oracle_sample(1)
            result["cpu_baseline"] = {"value": 1.0 / r["seconds_per_image"], "unit": UNIT,
                                      "cores": r["cores"], "kind": "port", "sample": r["sample"]}
        print(json.dumps(result), flush=True)
    ctx.close()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--images", type=int, default=64)
    ap.add_argument("--batch", type=int, default=16,
                    help="images per encoder call (16: the post-prune GEMMs and attention "
                         "fill the GPU better than at 8; a rank with fewer images uses them all)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("note: warm-up raised to the minimum of 3 steps", file=sys.stderr)
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
