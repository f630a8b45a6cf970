"""Benchmark of the Gemma 3 Q8_0 token loop on B200 (bs=1 greedy decode).

Default workload: the 27B-shaped decoder (vocab
262144, d 5376, 62 layers, 32 q / 16 KV heads of 128, ffn 21504, window 1024,
5:1 local:global) with seeded synthetic Q8_0 weights generated on the device,
a 2048-token seeded prompt prefilled in one batched pass on the tensor cores
(tcgen05 GEMMs; NCCL sums of the row-parallel partials under tensor
parallelism), then greedy decode.
`--workload 270m` runs config 0's 270M shape (8-token prompt) instead, and
`--workload 270m-long` config 2 (270M, 4096-token prompt, decode past the
512-token window).  Batched decode of independent sequences (tensor-core
GEMMs with M = sequences, per-sequence KV caches): `--workload 270m-batch`
is config 3 (256 sequences x 1024-token prompts, split evenly over the N
ranks as replicas with no collective), `--workload 27b-bs32` config 4 at
batch 32 on one GPU.

One step = one decoded token (batch 1).  Under torchrun (N > 1) the model is
tensor-parallel over N GPUs (Q/K/V, gate, up column-sharded; o-proj, down
row-sharded with an NCCL all-reduce; vocab-sharded LM head with an NCCL max
of the argmax keys), so the N ranks decode the same tokens: value = tokens /
max-over-ranks time ("scaling": "strong").

Printed JSON line:
  value          decode tok/s, K steps device-resident (graph replays, token fed
                 back on the device), CUDA events on the model stream
  e2e            tok/s through vrt_decode_step (the C ABI call a caller makes):
                 host token + position copied in, argmax result copied out, per step
  roofline       the dominant kernel (layer gate/up mat-vec: RMSNorm prologue,
                 gelu*up epilogue) timed alone on the same stream; algorithmic
                 bytes / time vs the measured HBM peak
  cpu_baseline   the CPU oracle (C restatement of the reference token loop,
                 GQA-generalised; the reference itself refuses head_count_kv != 1)
                 on a bounded sample, extrapolated to one token
  prefill        the prompt's prefill, device-timed (CUDA events), tokens/s
  clocks         nvidia-smi samples taken during the timed region
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
sys.path[:0] = [os.path.join(ROOT, "vortex-rt_b200"), os.path.join(ROOT, "oracle")]

import synth_gguf as sg  # noqa: E402

PROMPT_LEN = {"27b": 2048, "270m": 8, "270m-long": 4096, "270m-batch": 1024, "27b-bs32": 2048}
BATCH_SEQS = {"270m-batch": 256, "27b-bs32": 32}
METRIC = "decode tok/s (Gemma3-shaped Q8_0, bs=1 greedy)"


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic(workload: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(workload)
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows: list[list[str]] = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def shape_for(workload: str) -> sg.Gemma3Shape:
    return sg.SHAPES["27b" if workload.startswith("27b") else "270m"]


def bytes_per_token(shape: sg.Gemma3Shape, pos: int) -> int:
    """Q8_0 weight bytes + norm vectors + embedding row + KV read/write at `pos`."""
    d, hd = shape.embedding_length, shape.head_dim
    q8 = lambda r, c: r * c // 32 * 34  # noqa: E731
    layer = (q8(shape.q_width + 2 * shape.kv_width, d) + q8(d, shape.q_width) + 2 * q8(shape.feed_forward_length, d)
             + q8(d, shape.feed_forward_length))
    w = layer * shape.block_count + q8(shape.vocab_size, d)
    norms = (4 * d + 2 * hd) * 4 * shape.block_count + 4 * d
    kv = 0
    for l in range(shape.block_count):
        n = pos + 1 if (l + 1) % 6 == 0 else min(pos + 1, shape.sliding_window)
        kv += n * shape.head_count_kv * hd * 4 * 2
    return w + norms + d // 32 * 34 + kv


def cpu_baseline(workload: str, threads: int) -> dict:
    """Oracle port timed on a bounded sample of one decode token."""
    import oracle as O

    shape = shape_for(workload)
    if not workload.startswith("27b"):
        sample_layers, sample_vocab = shape.block_count, shape.vocab_size
    else:
        sample_layers, sample_vocab = 2, 16384
    small = shape.with_(block_count=sample_layers, vocab_size=sample_vocab)
    o = O.Oracle(shape=small, seed=11, threads=threads, max_positions=8)
    o.decode(2, 0, 1)  # warm caches / page in
    o.reset()
    t0 = time.perf_counter()
    steps = 2
    for p in range(steps):
        o.decode(2 + p, p, 1)
    t_tok = (time.perf_counter() - t0) / steps
    # LM head slice alone, to split head vs layer time
    raw = O.synth_q8(11, "token_embd.weight", sample_vocab, shape.embedding_length)
    x = np.random.default_rng(0).standard_normal(shape.embedding_length).astype(np.float32)
    t1 = time.perf_counter()
    O.q8_matvec(raw, x, sample_vocab, lanes=64 if shape.embedding_length > 1024 else 8, threads=threads)
    t_head = time.perf_counter() - t1
    per_layer = max(t_tok - t_head, 1e-9) / sample_layers
    full = per_layer * shape.block_count + t_head * (shape.vocab_size / sample_vocab)
    o.close()
    return {"value": 1.0 / full, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{steps} decode tokens of a {sample_layers}-layer, {sample_vocab}-row-vocab slice of the "
                      f"{workload} shape + one LM-head slice mat-vec, extrapolated to {shape.block_count} layers and "
                      f"vocab {shape.vocab_size}; C restatement of src/gemma3.cpp (the reference itself refuses "
                      f"head_count_kv != 1), {threads} host threads"}


def run_reference_arm(args, rank: int, world: int):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    vals = []
    for _ in range(args.warmup):
        cpu_baseline(args.workload, threads)
    for _ in range(args.steps):
        vals.append(cpu_baseline(args.workload, threads))
    v = statistics.median([x["value"] for x in vals])
    cb = dict(vals[-1])
    cb["value"] = v
    shape = shape_for(args.workload)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "q8_0*f32", "data": "synthetic",
        "config": {"workload": f"{args.workload}-shaped Gemma 3 Q8_0 decode, bs=1", "d_model": shape.embedding_length,
                   "layers": shape.block_count, "vocab": shape.vocab_size},
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_batched(args, rank: int, world: int, local: int):
    """Configs 3 / 4-bs32: independent sequences decoded together (vrt_batch).
    Under torchrun, config 3 splits the sequences evenly over the ranks, each
    rank a full replica with no collective on the data path ("replicas");
    config 4 at batch 32 is tensor parallel (every rank holds all sequences
    and 1/N of every projection, NCCL all-reduce after o-proj and down)."""
    import datetime

    import torch
    import torch.distributed as dist

    import vrt

    dist_on = world > 1
    if dist_on:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    tp = args.workload == "27b-bs32" and world > 1
    shape = shape_for(args.workload)
    if args.layers:
        shape = shape.with_(block_count=args.layers)
    if args.vocab:
        shape = shape.with_(vocab_size=args.vocab)
    total = BATCH_SEQS[args.workload]
    M = total if tp else total // world
    prompt_len = args.prompt_len or PROMPT_LEN[args.workload]
    e2e_steps = max(4, args.steps // 4)
    P = prompt_len + args.warmup + args.steps + e2e_steps + 8
    nccl_id = None
    if tp:
        obj = [vrt.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    ctx = vrt.Context(local)
    model = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=1234, max_positions=P,
                      tp_rank=rank if tp else 0, tp_world=world if tp else 1, nccl_id=nccl_id)
    b = vrt.Batch(model, M, P)
    stream = torch.cuda.ExternalStream(ctx.stream)

    def barrier():
        if dist_on:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        if dist_on:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rng = np.random.default_rng(3 if tp else 3 + rank)  # tensor parallel: the same prompts on every rank
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    barrier()
    ev[0].record(stream)
    for i in range(M):
        b.prefill(i, [2] + rng.integers(3, shape.vocab_size, prompt_len - 1).tolist())
    ev[1].record(stream)
    ctx.sync()
    t_pf = max_over_ranks(ev[0].elapsed_time(ev[1]) / 1000.0)
    b.decode_steps(M, args.warmup)
    ctx.sync()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    ctx.sync()
    barrier()
    ev[2].record(stream)
    b.decode_steps(M, args.steps)
    ev[3].record(stream)
    ctx.sync()
    barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(ev[2].elapsed_time(ev[3]))
    tok_s = total * args.steps / (ms / 1000.0)
    # e2e: the public call per step plus the read-back of every sequence's new id
    ids = np.zeros(M, np.uint32)
    barrier()
    ctx.sync()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        b.decode_steps(M, 1)
        b.last_ids(M, ids)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = total * e2e_steps / e2e_s
    _, pos = b.read(0, 1)
    status = model.device_status()
    b.close()
    model.close()
    ctx.close()
    if rank == 0:
        peak, peak_kind = measured_peaks()
        mid = prompt_len + args.warmup + args.steps // 2
        weights = bytes_per_token(shape, 0)  # weights + norms (+ one position of KV)
        step_bytes = weights + M * (bytes_per_token(shape, mid) - weights)
        if tp:
            step_bytes /= world  # per GPU: weights and KV heads are both sharded
        achieved = step_bytes / (ms / 1000.0 / args.steps) / 1e9
        cpu = None if args.no_cpu_baseline else cpu_baseline(args.workload, os.cpu_count() or 1)
        line = {
            "metric": METRIC.replace("bs=1", f"batched, {total} sequences"), "value": tok_s, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "q8_0*fp16x2->f32",
            "data": "synthetic (seeded Q8_0 weights generated on device, seeded uniform prompt ids)",
            "config": {"workload": {"270m-batch": f"config 3: 270M-shaped Gemma 3 Q8_0, {total} sequences x "
                                                  f"{prompt_len}-token prompts, greedy decode, sequences split over "
                                                  f"{world} replica(s)",
                                    "27b-bs32": f"config 4 at batch {total}: 27B-shaped, {prompt_len}-token prompts"
                                                + (f", tensor parallel over {world} GPUs" if tp else "")
                                    }[args.workload],
                       "d_model": shape.embedding_length, "layers": shape.block_count, "vocab": shape.vocab_size,
                       "global_batch": total, "sequences_per_gpu": M,
                       "parallelism": (f"tp{world}" if tp else f"replicas x{world}") if world > 1 else "single GPU",
                       "positions": f"{prompt_len + args.warmup}..{prompt_len + args.warmup + args.steps}",
                       "l2": f"inputs larger than L2 ({step_bytes / 1e9:.1f} GB per step)"},
            "gpu_launches": (7 * shape.block_count + 3) * args.steps,
            "kernels_per_step": 7 * shape.block_count + 3,
            "roofline": {"bound": "hbm", "kernel": "whole batched step: Q8_0 weights once + every sequence's KV",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_step": step_bytes, "traffic": None},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4 * M,
                    "note": "tokens stay on the device; each step reads back every sequence's new id"},
            "prefill": {"tokens": total * prompt_len, "s": t_pf, "tok_s": total * prompt_len / t_pf,
                        "method": "batched tensor-core prefill per sequence"},
            "final_position": pos,
            "device_status": status,
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="27b", choices=["27b", "270m", "270m-long", "270m-batch", "27b-bs32"])
    ap.add_argument("--prompt-len", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="profiling: fewer layers of the same shape")
    ap.add_argument("--vocab", type=int, default=0, help="profiling: smaller vocabulary of the same shape")
    ap.add_argument("--tp-exchange", default="peer", choices=["peer", "nccl"],
                    help="tensor parallelism: peer-memory exchange fused into the consumer kernels, or NCCL all-reduce")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist

    import vrt

    if args.workload in BATCH_SEQS:
        return run_batched(args, rank, world, local)

    dist_on = world > 1
    if dist_on:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    shape = shape_for(args.workload)
    if args.layers:
        shape = shape.with_(block_count=args.layers)
    if args.vocab:
        shape = shape.with_(vocab_size=args.vocab)
    prompt_len = args.prompt_len or PROMPT_LEN[args.workload]
    e2e_steps = args.steps
    positions = prompt_len + args.warmup + args.steps + e2e_steps + 8
    prompt = [2] + np.random.default_rng(4).integers(3, shape.vocab_size, prompt_len - 1).tolist()

    nccl_id = None
    if dist_on:
        obj = [vrt.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    ctx = vrt.Context(local)
    cfg = vrt.Gemma3Config.from_shape(shape)
    m = vrt.Model(ctx, None, config=cfg, seed=1234, max_positions=positions, tp_rank=rank, tp_world=world,
                  nccl_id=nccl_id, tp_exchange=args.tp_exchange)
    kernels = m.step_kernels()

    def barrier():
        if dist_on:
            dist.barrier()

    # prefill: batched tensor-core passes (NCCL sums of the row-parallel partials under TP)
    stream = torch.cuda.ExternalStream(ctx.stream)
    pf0 = torch.cuda.Event(enable_timing=True)
    pf1 = torch.cuda.Event(enable_timing=True)
    barrier()
    pf0.record(stream)
    m.prefill(prompt)
    pf1.record(stream)
    ctx.sync()
    t_pf = pf0.elapsed_time(pf1) / 1000.0
    tpf = torch.tensor([t_pf], dtype=torch.float64, device="cuda")
    if dist_on:
        dist.all_reduce(tpf, op=dist.ReduceOp.MAX)
    t_pf = float(tpf.item())

    # warmup
    m.decode_steps_async(args.warmup)
    ctx.sync()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ctx.sync()
    barrier()
    ev0.record(stream)
    m.decode_steps_async(args.steps)
    ev1.record(stream)
    ctx.sync()
    barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if dist_on:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tok_s = args.steps / (ms / 1000.0)
    status = m.device_status()
    tok, pos = m.next_token()

    # e2e through the C ABI call with host buffers (vrt_decode_step)
    barrier()
    ctx.sync()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        _, ids, _ = m.decode(tok, pos, 1, want_hidden=False)
        tok, pos = int(ids[0]), pos + 1
    ctx.sync()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if dist_on:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_tok_s = e2e_steps / float(te.item())

    # dominant kernel alone: layer-0 gate/up mat-vec
    k_ms, k_bytes = m.time_kernel(0, 2, iters=20)
    peak, peak_kind = measured_peaks()
    achieved = k_bytes / (k_ms / 1000.0) / 1e9
    step_bytes = bytes_per_token(shape, prompt_len + args.warmup + args.steps // 2)
    m.close()
    ctx.close()

    if rank == 0:
        cpu = None if args.no_cpu_baseline else cpu_baseline(args.workload, os.cpu_count() or 1)
        tr = committed_traffic(args.workload)
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "q8_0*f32",
            "data": "synthetic (seeded Q8_0 weights generated on device, seeded uniform prompt ids)",
            "config": {"workload": {"27b": f"config 4: 27B-shaped Gemma 3 Q8_0, bs=1 greedy decode after a "
                                           f"{prompt_len}-token prefill",
                                    "270m": f"config 0: 270M-shaped Gemma 3 Q8_0, bs=1 greedy decode after "
                                            f"{prompt_len} prompt tokens",
                                    "270m-long": f"config 2: 270M-shaped Gemma 3 Q8_0, {prompt_len}-token batched "
                                                 "prefill, then bs=1 greedy decode past the 512-token window"
                                    }[args.workload],
                       "d_model": shape.embedding_length, "layers": shape.block_count,
                       "heads": f"{shape.head_count}q/{shape.head_count_kv}kv x {shape.head_dim}",
                       "ffn": shape.feed_forward_length, "vocab": shape.vocab_size, "global_batch": 1,
                       "positions": f"{prompt_len + args.warmup}..{prompt_len + args.warmup + args.steps}",
                       "parallelism": f"tp{world}" if world > 1 else "single GPU",
                       "tp_exchange": (("peer memory (partials pushed over NVLink, summed in the consumer kernel)"
                                        if args.tp_exchange == "peer" else "NCCL all-reduce") if world > 1 else None),
                       "l2": f"inputs larger than L2 ({step_bytes / 1e9:.1f} GB streamed per token)"},
            "gpu_launches": kernels * args.steps,
            "kernels_per_step": kernels,
            "step_roofline": {"bytes_per_token": step_bytes, "achieved_gbs": step_bytes * tok_s / 1e9 / world,
                              "peak_gbs": peak, "frac": step_bytes * tok_s / 1e9 / world / peak,
                              "note": "per GPU; weights + norms + KV per token over device time"},
            "roofline": {"bound": "hbm", "kernel": "q8t_gemv_kernel<Resid, GeluPair> (layer gate/up)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_launch": k_bytes,
                         "ms_per_launch": k_ms, "traffic": tr},
            "e2e": {"value": e2e_tok_s, "unit": "tok/s", "h2d_bytes_per_step": 20, "d2h_bytes_per_step": 40},
            "prefill": {"tokens": prompt_len, "s": t_pf, "tok_s": prompt_len / t_pf,
                        "method": "batched: tcgen05 Q8_0 GEMMs + tiled prefill attention, chunks of 2048"
                                  + (", NCCL sums of the row-parallel partials" if world > 1 else "")},
            "device_status": status,
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
