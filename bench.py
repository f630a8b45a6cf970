"""Benchmark of the Gemma 3 Q8_0 token loop on B200.

Default workload: the 27B-shaped decoder (vocab
262144, d 5376, 62 layers, 32 q / 16 KV heads of 128, ffn 21504, window 1024,
5:1 local:global) with seeded synthetic Q8_0 weights generated on the device,
a 2048-token seeded prompt prefilled in one batched pass on the tensor cores
(tcgen05 GEMMs; NCCL sums of the row-parallel partials under tensor
parallelism), then greedy decode at batch 1.  Under torchrun (N > 1) the
model is tensor-parallel over N GPUs (Q/K/V, gate, up column-sharded; o-proj,
down row-sharded, their partial sums exchanged over NVLink peer memory inside
the consuming kernel; vocab-sharded LM head), so the N ranks decode the same
tokens: value = tokens / max-over-ranks time ("scaling": "strong").

Other workloads: `270m` (config 0), `270m-long` (config 2: 4096-token
prefill, decode past the 512 window), `270m-batch` (config 3: 256 sequences x
1024-token prompts, split over the ranks as replicas), `27b-bs32` (config 4 at
batch 32), `sweep` (config 1: the isolated Q8_0 mat-vec / FFN / LM-head
shapes, 1000 iterations each, hot and cold HBM).

Printed JSON line (rank 0):
  value          decode tok/s over K device-resident steps (graph replays,
                 token fed back on the device), CUDA events on the model stream
  e2e            tok/s through vrt_decode_step (the C ABI call a caller makes):
                 token + position copied in, argmax result copied out, per step
  roofline       the dominant kernel (layer gate/up mat-vec) timed alone on the
                 same stream: algorithmic bytes / time vs the measured HBM peak
  step_roofline  whole step: weights + norms + KV bytes per token / step time
  ids            the greedy ids decoded in the timed region (first 8, count,
                 SHA-1) and the smallest top-2 logit margin over them (a
                 teacher-forced replay of the same steps with top-2 logits), so
                 lines at different N can be checked for the same stream
  cpu_baseline   the CPU oracle timed on whole decode tokens of the same model
                 shape on this box's host cores (config 0: the reference's own
                 token loop, oracle/_ref)
  prefill        the prompt's prefill, device-timed, tokens/s
  clocks         SM clock / throttle reasons sampled in-process (NVML, 10 ms)
                 during the timed region
  also           (default workload) configs 0, 1, 2 and 4 at batch 32 on one
                 GPU, and config 3 at every N (its sequences split over the
                 ranks as replicas), measured in the same run
`--impl reference` runs the reference arm: the reference's CPU token loop
(oracle/_ref for the 270M shape; the C restatement of it where the reference
refuses the shape, e.g. 16 KV heads) on whole tokens of the same workload.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "vortex-rt_b200"), os.path.join(ROOT, "oracle")]

import synth_gguf as sg  # noqa: E402

PROMPT_LEN = {"27b": 2048, "270m": 8, "270m-long": 4096, "270m-batch": 1024, "27b-bs32": 2048}
BATCH_SEQS = {"270m-batch": 256, "27b-bs32": 32}
METRIC = "decode tok/s (Gemma3-shaped Q8_0, bs=1 greedy)"
SEED = 1234


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


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """SM clock, power and throttle reasons of this rank's GPU, sampled every
    10 ms in-process through NVML (read-only queries); nvidia-smi at 200 ms
    when NVML is not importable."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, local: int):
        self.local = local
        self.rows = []
        self.stop_ev = threading.Event()
        self.thread = None
        self.source = None
        self.h = None
        self.nv = None

    def _handle(self):
        import pynvml as nv
        import torch
        nv.nvmlInit()
        props = torch.cuda.get_device_properties(self.local)
        tries = [f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0",
                 f"{props.pci_domain_id:04X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"]
        for t in tries:
            try:
                return nv, nv.nvmlDeviceGetHandleByPciBusId(t)
            except Exception:  # noqa: BLE001 - try the next form
                pass
        return nv, nv.nvmlDeviceGetHandleByIndex(self.local)

    def start(self):
        try:
            self.nv, self.h = self._handle()
            self.source = "nvml, 10 ms"
            self.max_mhz = float(self.nv.nvmlDeviceGetMaxClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            get_reasons = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons",
                                  getattr(self.nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))

            def loop():
                while not self.stop_ev.is_set():
                    try:
                        self.rows.append((float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)),
                                          int(get_reasons(self.h)) if get_reasons else 0,
                                          self.nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0))
                    except Exception:  # noqa: BLE001 - a failed sample is skipped
                        pass
                    self.stop_ev.wait(0.010)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            self.source = "nvidia-smi, 200 ms"
            self._smi_start()

    def _smi_start(self):
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.local), "--query-gpu=" + fields,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

        def rd():
            for line in self.proc.stdout:
                r = [x.strip() for x in line.split(",")]
                if len(r) < 7:
                    continue
                try:
                    bits = sum(self.REASONS[n] for n, v in zip(names, r[3:7]) if v.lower() == "active")
                    self.max_mhz = float(r[1])
                    self.rows.append((float(r[0]), bits, float(r[2])))
                except ValueError:
                    pass

        self.thread = threading.Thread(target=rd, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        self.stop_ev.set()
        if getattr(self, "proc", None):
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "source": self.source}
        sm = [r[0] for r in self.rows]
        bits = 0
        for r in self.rows:
            bits |= r[1]
        reasons = sorted(n for n, b in self.REASONS.items() if bits & b)
        return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm), "sm_max_mhz": getattr(self, "max_mhz", None),
                "power_w_max": max(r[2] for r in self.rows), "reasons": reasons, "samples": len(self.rows),
                "source": self.source}


# ------------------------------------------------------------------ shapes

def shape_for(workload: str, layers: int = 0, vocab: int = 0) -> sg.Gemma3Shape:
    s = sg.SHAPES["27b" if workload.startswith("27b") else "270m"]
    if layers:
        s = s.with_(block_count=layers)
    if vocab:
        s = s.with_(vocab_size=vocab)
    return s


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


def prompt_ids(shape: sg.Gemma3Shape, n: int, seed: int = 4) -> list[int]:
    return [2] + np.random.default_rng(seed).integers(3, shape.vocab_size, n - 1).tolist()


def workload_config(workload: str, shape: sg.Gemma3Shape, world: int, prompt_len: int, warmup: int, steps: int,
                    tp_exchange: str) -> dict:
    """The `config` object of the JSON line: identical for both arms."""
    name = {"27b": f"config 4: 27B-shaped Gemma 3 Q8_0, bs=1 greedy decode after a {prompt_len}-token prefill",
            "270m": f"config 0: 270M-shaped Gemma 3 Q8_0, bs=1 greedy decode after {prompt_len} prompt tokens",
            "270m-long": f"config 2: 270M-shaped Gemma 3 Q8_0, {prompt_len}-token batched prefill, then bs=1 "
                         "greedy decode past the 512-token window"}[workload]
    step_bytes = bytes_per_token(shape, prompt_len + warmup + steps // 2)
    return {"workload": name, "d_model": shape.embedding_length, "layers": shape.block_count,
            "heads": f"{shape.head_count}q/{shape.head_count_kv}kv x {shape.head_dim}",
            "ffn": shape.feed_forward_length, "vocab": shape.vocab_size, "global_batch": 1,
            "positions": f"{prompt_len + warmup}..{prompt_len + warmup + steps}",
            "parallelism": f"tp{world}" if world > 1 else "single GPU",
            "tp_exchange": (("peer memory (partials pushed over NVLink, summed in the consumer kernel)"
                             if tp_exchange == "peer" else "NCCL all-reduce") if world > 1 else None),
            "l2": f"inputs larger than L2 ({step_bytes / 1e9:.1f} GB streamed per token)"}


# ------------------------------------------------------------ CPU baselines

def cpu_tokens(shape: sg.Gemma3Shape, threads: int, warm: int, n: int, prompt: list[int]) -> dict:
    """Whole decode tokens of the C restatement of the reference token loop
    (GQA-generalised) on a host copy of the same seeded model."""
    import oracle as O

    t0 = time.perf_counter()
    o = O.Oracle(shape=shape, seed=SEED, threads=threads, max_positions=warm + n + 2)
    create_s = time.perf_counter() - t0
    toks = prompt + [prompt[-1]] * (warm + n)
    for p in range(warm):
        o.decode(toks[p], p, 1)
    times = []
    for p in range(warm, warm + n):
        t = time.perf_counter()
        o.decode(toks[p], p, 1)
        times.append(time.perf_counter() - t)
    o.close()
    return {"tok_s": n / sum(times), "per_token_s": times, "create_s": create_s}


def cpu_reference_270m(threads: int, prompt: list[int], n: int, warm: int = 0) -> dict | None:
    """The reference's own token loop (src/gemma3.cpp via oracle/_ref) on the
    270M synthetic GGUF: greedy tokens after the prompt, timed per token."""
    import oracle as O

    if not O.reference_available():
        return None
    shape = sg.SHAPES["270m"]
    d = os.path.join(tempfile.gettempdir(), "vrt_bench_models")
    path = sg.cached_model(shape, SEED, d)
    r = O.Reference(path, threads=threads)
    for p, t in enumerate(prompt[:-1]):
        r.decode(t, p, 0)
    tok, pos = prompt[-1], len(prompt) - 1
    times = []
    for i in range(warm + n):
        t = time.perf_counter()
        _, ids, _ = r.decode(tok, pos, 1)
        if i >= warm:
            times.append(time.perf_counter() - t)
        tok, pos = int(ids[0]), pos + 1
    r.close()
    return {"tok_s": len(times) / sum(times), "per_token_s": times}


def cpu_baseline(workload: str, shape: sg.Gemma3Shape, threads: int) -> dict:
    prompt = prompt_ids(shape, 8)
    if workload.startswith("270m"):
        r = cpu_reference_270m(threads, prompt, 8, warm=1)
        if r is not None:
            return {"value": r["tok_s"], "unit": "tok/s", "cores": threads, "kind": "reference",
                    "sample": f"8 whole greedy decode tokens (after 1 warm-up) following an 8-token prompt, the "
                              f"reference's own src/gemma3.cpp token loop (oracle/_ref) on the same seeded 270M "
                              f"model, {threads} host threads"}
    r = cpu_tokens(shape, threads, 1, 2, prompt)
    return {"value": r["tok_s"], "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"2 whole decode tokens (after 1 warm-up) of the full {shape.name}-shaped model "
                      f"({shape.block_count} layers, vocab {shape.vocab_size}) at positions 1-2, C restatement of "
                      f"src/gemma3.cpp (the reference itself refuses head_count_kv != 1), {threads} host threads; "
                      f"host model built in {r['create_s']:.0f} s"}


def run_reference_arm(args, rank: int, world: int):
    """The reference's CPU token loop on whole tokens of this workload: one
    step = one decode token (prompt tokens run through the same loop first for
    270M; for 27B the 2048-token prefill is not replayed on the host, where it
    would take about an hour, so the tokens sit at positions 1..K+W)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    workload = args.workload if args.workload in ("27b", "270m", "270m-long") else "27b"
    shape = shape_for(workload, args.layers, args.vocab)
    prompt_len = args.prompt_len or PROMPT_LEN[workload]
    t_all = time.perf_counter()
    if workload.startswith("270m"):
        r = cpu_reference_270m(threads, prompt_ids(shape, 8), args.steps, warm=args.warmup)
        kind, what = "reference", "the reference's own src/gemma3.cpp token loop (oracle/_ref)"
        pos = "positions 8.."
    else:
        r = None
    if r is None:
        r = cpu_tokens(shape, threads, args.warmup, args.steps, prompt_ids(shape, 8))
        kind = "port"
        what = ("the C restatement of src/gemma3.cpp (oracle/liboracle.so; the reference itself refuses "
                "head_count_kv != 1)")
        pos = f"positions {args.warmup}..{args.warmup + args.steps - 1}"
    v = r["tok_s"]
    sample = (f"{args.steps} whole greedy decode tokens (after {args.warmup} warm-up tokens) of the full "
              f"{shape.name}-shaped model, {pos}, {what}, {threads} host threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "q8_0*f32", "data": "synthetic",
        "config": workload_config(workload, shape, world, prompt_len, args.warmup, args.steps, args.tp_exchange),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t_all,
    }), flush=True)


# ------------------------------------------------------------------ sweep

SWEEP = [("qkv_1920x640_triplet", "multi", 640, 640, 3), ("mv_640x1024", "gemv", 640, 1024, 1),
         ("ffn_2048x640x2_640x2048", "ffn", 2048, 640, 1), ("lm_262144x640_argmax", "head", 262144, 640, 1),
         ("mv_21504x5376", "gemv", 21504, 5376, 1)]


def sweep(ctx, iters: int = 1000, cpu: bool = True, only: list[str] | None = None) -> dict:
    """Config 1: each shape's drop-in pipeline kernel (raw GGUF rows:
    vrt_q8_gemv[_multi] / vrt_q8_ffn / vrt_lm_head_argmax) and the packed
    (Q8T) model kernel, `iters` calls each, hot (one weight copy, L2-resident
    when it fits) and cold (copies rotated over >= 2x L2).  GB/s counts
    rows*cols/32*34 + 4*cols + 4*rows per call.  With cpu=True the
    reference's CPU-reference loops are timed on the same shapes (q8_test's
    fp32 loop, src/q8_test_main.cpp:125-128, and ffn_test's fp64 matvec,
    src/ffn_test_main.cpp:217-250, both restated in oracle/) and the GPU
    outputs are checked against the fp64 one (atol/rtol 1e-3)."""
    import ctypes as Cc

    import torch

    import vrt

    L = vrt.lib()
    peak, peak_kind = measured_peaks()
    l2 = ctx.info().l2_bytes
    stream = torch.cuda.ExternalStream(ctx.stream)
    out = {"iterations": iters, "peak_gbs": peak, "peak_source": f"{peak_kind} hbm_gbs", "shapes": {}}
    rng = np.random.default_rng(11)
    for name, kind, rows, cols, count in SWEEP:
        if only and name not in only:
            continue
        if kind == "ffn":
            mats = [sg.q8_matrix_bytes(SEED, f"sweep.{name}.{t}", r, c) for t, r, c in
                    (("gate", rows, cols), ("up", rows, cols), ("down", cols, rows))]
            alg = sum(m.nbytes for m in mats) + 4 * cols + 4 * cols
        else:
            mats = [sg.q8_matrix_bytes(SEED, f"sweep.{name}.{i}", rows, cols) for i in range(count)]
            alg = sum(m.nbytes for m in mats) + 4 * cols + 4 * rows * count + (8 if kind == "head" else 0)
        raw = np.concatenate(mats)
        nbytes = raw.nbytes
        ncopy = max(1, -(-2 * l2 // nbytes))
        x = rng.standard_normal(cols).astype(np.float32)
        dev = torch.cuda.current_device()
        stride = (nbytes + 255) // 256 * 256  # every copy 256-byte aligned
        w = torch.zeros((ncopy, stride), dtype=torch.uint8, device=dev)
        w[:, :nbytes] = torch.from_numpy(raw).to(dev)
        dx = torch.from_numpy(x).to(dev)
        n_out = (rows * count) if kind != "ffn" else cols
        dy = torch.zeros(max(n_out, 1), dtype=torch.float32, device=dev)
        work = torch.zeros(2 * rows, dtype=torch.float32, device=dev)
        res = torch.zeros(2, dtype=torch.int32, device=dev)
        offs = (Cc.c_uint64 * count)(*[i * mats[0].nbytes for i in range(count)])
        dims = (Cc.c_uint32 * count)(*([rows] * count))
        torch.cuda.synchronize()

        def raw_call(i):
            base = w[i].data_ptr()
            if kind == "gemv":
                return L.vrt_q8_gemv(ctx.h, base, nbytes, 0, dx.data_ptr(), dy.data_ptr(), cols, rows, None)
            if kind == "multi":
                return L.vrt_q8_gemv_multi(ctx.h, base, nbytes, offs, dims, count, dx.data_ptr(), dy.data_ptr(), cols,
                                           None)
            if kind == "ffn":
                g, u = mats[0].nbytes, mats[1].nbytes
                return L.vrt_q8_ffn(ctx.h, base, nbytes, 0, g, g + u, dx.data_ptr(), work.data_ptr(), dy.data_ptr(),
                                    cols, rows, cols, None)
            return L.vrt_lm_head_argmax(ctx.h, base, nbytes, 0, dx.data_ptr(), cols, rows, None, res.data_ptr(), None)

        # packed (Q8T) copies of the same matrices, the model kernels' layout
        if kind == "ffn":
            pb_gu, pb_dn = L.vrt_q8t_bytes(2 * rows, cols), L.vrt_q8t_bytes(cols, rows)
            pk = torch.empty((ncopy, pb_gu + pb_dn), dtype=torch.uint8, device=dev)
            for i in range(ncopy):
                g, u = mats[0].nbytes, mats[1].nbytes
                vrt.check(L.vrt_q8t_pack_pair(ctx.h, w[i].data_ptr(), nbytes, 0, g, rows, cols, pk[i].data_ptr(), None))
                vrt.check(L.vrt_q8t_pack(ctx.h, w[i].data_ptr(), nbytes, g + u, cols, rows,
                                         pk[i].data_ptr() + pb_gu, None))
        else:
            pb = L.vrt_q8t_bytes(rows * count, cols)
            pk = torch.empty((ncopy, pb), dtype=torch.uint8, device=dev)
            for i in range(ncopy):
                vrt.check(L.vrt_q8t_pack(ctx.h, w[i].data_ptr(), nbytes, 0, rows * count, cols, pk[i].data_ptr(), None))

        def packed_call(i):
            base = pk[i].data_ptr()
            if kind in ("gemv", "multi"):
                return L.vrt_q8t_gemv(ctx.h, base, rows * count, cols, dx.data_ptr(), dy.data_ptr(), None)
            if kind == "ffn":
                return L.vrt_q8t_ffn(ctx.h, base, base + pb_gu, cols, rows, cols, dx.data_ptr(), work.data_ptr(),
                                     dy.data_ptr(), None)
            return L.vrt_q8t_lm_head_argmax(ctx.h, base, rows, cols, dx.data_ptr(), None, res.data_ptr(), None)

        rec = {"rows": rows * count if kind != "ffn" else f"{rows}x2+{cols}", "cols": cols, "bytes_per_call": alg,
               "weight_copies_cold": ncopy}
        outputs = {}
        for label, call in (("raw", raw_call), ("packed", packed_call)):
            for mode in ("hot", "cold"):
                for i in range(3):
                    vrt.check(call(i % ncopy))
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record(stream)
                for i in range(iters):
                    call(i % ncopy if mode == "cold" else 0)
                ev1.record(stream)
                ev1.synchronize()
                us = ev0.elapsed_time(ev1) * 1000.0 / iters
                rec[f"{label}_{mode}_us"] = us
                rec[f"{label}_{mode}_gbs"] = alg / us / 1e3
                rec[f"{label}_{mode}_frac"] = alg / us / 1e3 / peak
            ctx.sync()
            outputs[label] = (dy.cpu().numpy().copy() if kind != "head" else res.cpu().numpy().copy())
        if cpu:
            rec.update(_sweep_cpu(kind, mats, x, rows, cols, count, outputs))
        out["shapes"][name] = rec
        del w, pk
        torch.cuda.empty_cache()
    return out


def _sweep_cpu(kind, mats, x, rows, cols, count, outputs) -> dict:
    """CPU-reference loops of the reference test programs on the sweep shape
    (all host threads), and the check of the GPU results against fp64."""
    import oracle as O

    threads = os.cpu_count() or 1
    rec = {"cpu_threads": threads}
    if kind == "ffn":
        t = time.perf_counter()
        g = O.q8_matvec(mats[0], x, rows, lanes=0, threads=threads)
        u = O.q8_matvec(mats[1], x, rows, lanes=0, threads=threads)
        a = O.gelu_mul(g, u)
        ref = O.q8_matvec(mats[2], a, cols, lanes=0, threads=threads)
        rec["cpu_ffn_test_fp64_ms"] = (time.perf_counter() - t) * 1e3
    else:
        ref = np.concatenate([O.q8_matvec(m, x, rows, lanes=0, threads=threads) for m in mats])
        t = time.perf_counter()
        for m in mats:
            O.q8_matvec(m, x, rows, lanes=0, threads=threads)
        rec["cpu_ffn_test_fp64_ms"] = (time.perf_counter() - t) * 1e3
        t = time.perf_counter()
        for m in mats:
            O.q8_matvec(m, x, rows, lanes=1, threads=threads)
        rec["cpu_q8_test_fp32_ms"] = (time.perf_counter() - t) * 1e3
    if kind == "head":
        idx, _ = O.argmax(ref)
        rec["check"] = "argmax equal" if all(int(o[0]) == idx for o in outputs.values()) else "ARGMAX MISMATCH"
    else:
        worst = 0.0
        for o in outputs.values():
            err = np.abs(o[:ref.size].astype(np.float64) - ref) / (1e-3 + 1e-3 * np.abs(ref))
            worst = max(worst, float(err.max()))
        rec["check"] = f"within atol/rtol 1e-3 of fp64 (worst err/bound {worst:.3f})" if worst <= 1 else \
            f"MISMATCH (err/bound {worst:.3f})"
    return rec


def run_sweep(args):
    import torch

    import vrt

    ctx = vrt.Context(0)
    t0 = time.perf_counter()
    only = args.sweep_shapes.split(",") if args.sweep_shapes else None
    res = sweep(ctx, iters=args.steps if args.steps >= 100 else 1000, cpu=not args.no_cpu_baseline, only=only)
    shapes = res["shapes"]
    # headline: the largest single mat-vec, cold HBM, packed kernel
    big = shapes.get("mv_21504x5376") or next(iter(shapes.values()))
    line = {"metric": "Q8_0 mat-vec achieved HBM GB/s (21504x5376, cold)", "value": big["packed_cold_gbs"],
            "unit": "GB/s", "n_gpus": 1, "steps": res["iterations"], "warmup": 3,
            "ms_per_step": big["packed_cold_us"] / 1000.0, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q8_0*f32", "data": "synthetic (seeded Q8_0 weights, x ~ N(0,1))",
            "config": {"workload": "config 1: isolated Q8_0 mat-vec / fused FFN / LM head + argmax sweep",
                       "l2": "cold = weight copies rotated over >= 2x L2; hot = one copy"},
            "gpu_launches": res["iterations"] * 4 * len(SWEEP),
            "roofline": {"bound": "hbm", "kernel": "q8t_gemv_kernel (21504x5376, cold)",
                         "achieved": big["packed_cold_gbs"], "peak": res["peak_gbs"], "unit": "GB/s",
                         "frac": big["packed_cold_frac"], "traffic": None},
            "sweep": res, "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)
    ctx.close()
    del torch


# ---------------------------------------------------------- decode (bs=1)

def decode_run(args, workload: str, rank: int, world: int, local: int, dist_on: bool, ctx, steps: int, warmup: int,
               e2e_steps: int, with_margins: bool = True, nccl_id=None) -> dict:
    """Prefill + timed greedy decode of one model; returns the numbers of the line."""
    import torch
    import torch.distributed as dist

    import vrt

    shape = shape_for(workload, args.layers if workload == args.workload else 0,
                      args.vocab if workload == args.workload else 0)
    prompt_len = (args.prompt_len if workload == args.workload else 0) or PROMPT_LEN[workload]
    positions = prompt_len + warmup + steps + e2e_steps + 8
    prompt = prompt_ids(shape, prompt_len)
    m = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=SEED, max_positions=positions,
                  tp_rank=rank, tp_world=world, nccl_id=nccl_id, tp_exchange=args.tp_exchange,
                  step_mode=args.step_mode)
    kernels = m.step_kernels()
    stream = torch.cuda.ExternalStream(ctx.stream)

    def barrier():
        if dist_on:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        if dist_on:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    barrier()
    ev[0].record(stream)
    m.prefill(prompt)
    ev[1].record(stream)
    ctx.sync()
    t_pf = max_over_ranks(ev[0].elapsed_time(ev[1]) / 1000.0)

    m.decode_steps_async(warmup)
    ctx.sync()
    tok_start, pos_start = m.next_token()
    ids_dev = torch.zeros(max(steps, 1), dtype=torch.int32, device="cuda")
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    ctx.sync()
    barrier()
    ev[2].record(stream)
    m.decode_steps_async(steps, ids_dev.data_ptr())
    ev[3].record(stream)
    ctx.sync()
    barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(ev[2].elapsed_time(ev[3]))
    tok_s = steps / (ms / 1000.0)
    status = m.device_status()
    ids = ids_dev.cpu().numpy().astype(np.uint32)[:steps]
    tok, pos = m.next_token()

    # e2e through the C ABI call with host buffers (vrt_decode_step)
    barrier()
    ctx.sync()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        _, out_ids, _ = m.decode(tok, pos, 1, want_hidden=False)
        tok, pos = int(out_ids[0]), pos + 1
    ctx.sync()
    e2e_tok_s = e2e_steps / max_over_ranks(time.perf_counter() - t0)

    # the timed steps again, teacher-forced, with top-2 logits: the margins that
    # tell a legitimate near-tie from a divergence when streams are compared
    margins = None
    agree = None
    if with_margins:
        m.reset()
        m.prefill(prompt)
        m.decode_steps_async(warmup)
        t, p = m.next_token()
        assert (t, p) == (tok_start, pos_start)
        margins, agree = [], 0
        for i in range(steps):
            _, top, lg = m.decode(t, p, 2, want_hidden=False)
            margins.append(float(lg[0] - lg[1]))
            agree += int(top[0]) == int(ids[i])
            t, p = int(ids[i]), p + 1

    # dominant kernel alone: layer-0 gate/up mat-vec
    k_ms, k_bytes = m.time_kernel(0, 2, iters=20)
    m.close()
    return {"shape": shape, "prompt_len": prompt_len, "tok_s": tok_s, "ms": ms, "kernels": kernels,
            "status": status, "clocks": clocks, "e2e": e2e_tok_s, "prefill_s": t_pf, "ids": ids,
            "margins": margins, "agree": agree, "k_ms": k_ms, "k_bytes": k_bytes}


def ids_summary(r: dict) -> dict:
    ids = r["ids"]
    out = {"first8": ids[:8].tolist(), "count": int(ids.size),
           "sha1": hashlib.sha1(ids.astype("<u4").tobytes()).hexdigest()[:16]}
    if r["margins"] is not None:
        out["min_top2_margin"] = min(r["margins"]) if r["margins"] else None
        out["replay_agrees"] = f"{r['agree']}/{ids.size}"
    return out


def line_for(args, workload: str, r: dict, world: int, steps: int, warmup: int, cpu: dict | None) -> dict:
    peak, peak_kind = measured_peaks()
    shape = r["shape"]
    achieved = r["k_bytes"] / (r["k_ms"] / 1000.0) / 1e9
    step_bytes = bytes_per_token(shape, r["prompt_len"] + warmup + steps // 2)
    tr = committed_traffic("27b") if workload == "27b" and not args.layers and not args.vocab else None
    line = {
        "metric": METRIC, "value": r["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": r["ms"] / steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q8_0*f32", "data": "synthetic (seeded Q8_0 weights generated on device, seeded uniform prompt ids)",
        "config": workload_config(workload, shape, world, r["prompt_len"], warmup, steps, args.tp_exchange),
        "gpu_launches": r["kernels"] * steps,
        "kernels_per_step": r["kernels"],
        "step_mode": args.step_mode,
        "step_roofline": {"bytes_per_token": step_bytes, "achieved_gbs": step_bytes * r["tok_s"] / 1e9 / world,
                          "peak_gbs": peak, "frac": step_bytes * r["tok_s"] / 1e9 / world / peak,
                          "note": "per GPU; weights + norms + KV per token over device time"},
        "roofline": {"bound": "hbm", "kernel": "q8t_gemv_kernel<Resid, GeluPair> (layer gate/up)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_launch": r["k_bytes"],
                     "ms_per_launch": r["k_ms"],
                     "traffic": (tr / world) if tr else None,
                     "traffic_source": ("ncu dram bytes of one 1-GPU launch (profiles/traffic.json)"
                                        + (f", divided by {world}: each rank streams 1/{world} of the rows"
                                           if world > 1 else "")) if tr else None},
        "e2e": {"value": r["e2e"], "unit": "tok/s", "h2d_bytes_per_step": 20, "d2h_bytes_per_step": 40},
        "prefill": {"tokens": r["prompt_len"], "s": r["prefill_s"], "tok_s": r["prompt_len"] / r["prefill_s"],
                    "method": "batched: tcgen05 Q8_0 GEMMs + tiled prefill attention, chunks of 2048"
                              + (", NCCL sums of the row-parallel partials" if world > 1 else "")},
        "ids": ids_summary(r),
        "device_status": r["status"],
        "clocks": r["clocks"],
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def also_line(line: dict | None) -> dict | None:
    """A secondary workload's line inside the default line's `also`: the keys
    that repeat the main line's are dropped, the rest is kept as printed."""
    if line is None:
        return None
    for k in ("metric", "n_gpus", "dtype", "data", "higher_is_better", "vs_baseline"):
        line.pop(k, None)
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="27b", choices=["27b", "270m", "270m-long", "270m-batch", "27b-bs32",
                                                          "sweep"])
    ap.add_argument("--prompt-len", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 0 / config 1 results of the default run")
    ap.add_argument("--sweep-shapes", default="", help="sweep workload: comma-separated subset of the shapes")
    ap.add_argument("--layers", type=int, default=0, help="profiling: fewer layers of the same shape")
    ap.add_argument("--vocab", type=int, default=0, help="profiling: smaller vocabulary of the same shape")
    ap.add_argument("--tp-exchange", default="peer", choices=["peer", "nccl"],
                    help="tensor parallelism: peer-memory exchange fused into the consumer kernels, or NCCL all-reduce")
    ap.add_argument("--step-mode", default="launches", choices=["launches", "persistent"],
                    help="decode step as one kernel per op (default) or one persistent kernel per token")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if args.workload == "sweep":
        if rank == 0:
            run_sweep(args)
        return None
    if args.workload in BATCH_SEQS:
        return run_batched(args, rank, world, local)

    import datetime

    import torch
    import torch.distributed as dist

    import vrt

    dist_on = world > 1
    if dist_on:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    nccl_id = None
    if dist_on:
        obj = [vrt.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    ctx = vrt.Context(local)
    e2e_steps = args.steps
    r = decode_run(args, args.workload, rank, world, local, dist_on, ctx, args.steps, args.warmup, e2e_steps,
                   nccl_id=nccl_id)
    extras = {}
    extras_on = args.workload == "27b" and not args.no_extras and not args.layers and not args.vocab
    if world == 1 and extras_on:
        # config 0 on the same GPU in the same run (one GPU: replicas only)
        r0 = decode_run(args, "270m", 0, 1, local, False, ctx, 256, 8, 64)
        c0 = line_for(args, "270m", r0, 1, 256, 8, None if args.no_cpu_baseline else
                      cpu_baseline("270m", r0["shape"], os.cpu_count() or 1))
        extras["config0_270m"] = also_line(c0)
        # config 1: the isolated kernels
        extras["config1_sweep"] = sweep(ctx, iters=1000, cpu=not args.no_cpu_baseline)
        # config 2: 4096-token batched prefill, then decode past the 512 window
        r2 = decode_run(args, "270m-long", 0, 1, local, False, ctx, 512, 8, 32)
        extras["config2_270m_long"] = also_line(line_for(args, "270m-long", r2, 1, 512, 8, None))
        # config 4 at batch 32 (one GPU; under torchrun the default line is the bs=1 tensor-parallel one)
        extras["config4_bs32"] = also_line(batched_run(args, "27b-bs32", 0, 1, local, False, ctx, 16, 3))
    if extras_on:
        # config 3 on every rank: the 256 sequences split over the ranks as replicas, no collective
        r3 = batched_run(args, "270m-batch", rank, world, local, dist_on, ctx, 64, 4)
        if r3 is not None:
            extras["config3_270m_batch"] = also_line(r3)
    ctx.close()
    if rank == 0:
        cpu = None if args.no_cpu_baseline else cpu_baseline(args.workload, r["shape"], os.cpu_count() or 1)
        line = line_for(args, args.workload, r, world, args.steps, args.warmup, cpu)
        if extras:
            line["also"] = extras
        print(json.dumps(line), flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


def run_batched(args, rank: int, world: int, local: int):
    """`--workload 270m-batch` / `27b-bs32` on their own."""
    import datetime

    import torch
    import torch.distributed as dist

    import vrt

    dist_on = world > 1
    if dist_on:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    ctx = vrt.Context(local)
    line = batched_run(args, args.workload, rank, world, local, dist_on, ctx, args.steps, args.warmup,
                       cpu=not args.no_cpu_baseline)
    ctx.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


def batched_run(args, workload: str, rank: int, world: int, local: int, dist_on: bool, ctx, steps: int,
                warmup: int, cpu: bool = False) -> dict | None:
    """Configs 3 / 4-bs32: independent sequences decoded together (vrt_batch).
    Under torchrun, config 3 splits the sequences evenly over the ranks, each
    rank a full replica with no collective on the data path ("replicas");
    config 4 at batch 32 is tensor parallel (every rank holds all sequences
    and 1/N of every projection, NCCL all-reduce after o-proj and down).
    Returns the line on rank 0 (None elsewhere); every rank must call."""
    import torch
    import torch.distributed as dist

    import vrt

    own = workload == args.workload
    tp = workload == "27b-bs32" and world > 1
    shape = shape_for(workload, args.layers if own else 0, args.vocab if own else 0)
    total = BATCH_SEQS[workload]
    M = total if tp else total // world
    prompt_len = (args.prompt_len if own else 0) or PROMPT_LEN[workload]
    e2e_steps = max(4, steps // 4)
    P = prompt_len + warmup + steps + e2e_steps + 8
    nccl_id = None
    if tp:
        obj = [vrt.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    model = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=SEED, max_positions=P,
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
    b.decode_steps(M, warmup)
    ctx.sync()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    ctx.sync()
    barrier()
    ev[2].record(stream)
    b.decode_steps(M, steps)
    ev[3].record(stream)
    ctx.sync()
    barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(ev[2].elapsed_time(ev[3]))
    tok_s = total * steps / (ms / 1000.0)
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
    first_ids, pos = b.read(0, 1 << 12)
    status = model.device_status()
    b.close()
    model.close()
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    mid = prompt_len + warmup + steps // 2
    weights = bytes_per_token(shape, 0)  # weights + norms (+ one position of KV)
    step_bytes = weights + M * (bytes_per_token(shape, mid) - weights)
    if tp:
        step_bytes /= world  # per GPU: weights and KV heads are both sharded
    achieved = step_bytes / (ms / 1000.0 / steps) / 1e9
    cpu_line = cpu_baseline(workload, shape, os.cpu_count() or 1) if cpu else None
    seq0 = np.asarray(first_ids, np.uint32)
    line = {
        "metric": METRIC.replace("bs=1", f"batched, {total} sequences"), "value": tok_s, "unit": "tok/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q8_0*int8/fp16->f32",
        "data": "synthetic (seeded Q8_0 weights generated on device, seeded uniform prompt ids)",
        "config": {"workload": {"270m-batch": f"config 3: 270M-shaped Gemma 3 Q8_0, {total} sequences x "
                                              f"{prompt_len}-token prompts, greedy decode, sequences split over "
                                              f"{world} replica(s)",
                                "27b-bs32": f"config 4 at batch {total}: 27B-shaped, {prompt_len}-token prompts"
                                            + (f", tensor parallel over {world} GPUs" if tp else "")
                                }[workload],
                   "d_model": shape.embedding_length, "layers": shape.block_count, "vocab": shape.vocab_size,
                   "global_batch": total, "sequences_per_gpu": M,
                   "parallelism": (f"tp{world}" if tp else f"replicas x{world}") if world > 1 else "single GPU",
                   "positions": f"{prompt_len + warmup}..{prompt_len + warmup + steps}",
                   "l2": f"inputs larger than L2 ({step_bytes / 1e9:.1f} GB per step)"},
        "gpu_launches": (7 * shape.block_count + 3) * steps,
        "kernels_per_step": 7 * shape.block_count + 3,
        "roofline": {"bound": "hbm", "kernel": "whole batched step: Q8_0 weights once + every sequence's KV",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_step": step_bytes, "traffic": None},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4 * M,
                "note": "tokens stay on the device; each step reads back every sequence's new id"},
        "prefill": {"tokens": total * prompt_len, "s": t_pf, "tok_s": total * prompt_len / t_pf,
                    "method": "batched tensor-core prefill per sequence"},
        "ids": {"sequence0_first8": seq0[:8].tolist(), "sequence0_count": int(seq0.size),
                "sequence0_sha1": hashlib.sha1(seq0.astype("<u4").tobytes()).hexdigest()[:16]},
        "final_position": pos,
        "device_status": status,
        "clocks": clocks,
    }
    if cpu_line is not None:
        line["cpu_baseline"] = cpu_line
    return line


if __name__ == "__main__":
    main()
