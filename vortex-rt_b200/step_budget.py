"""Per-layer time budget of the decode step (launch chain), from the phase
stamps of the timing build.

    make -C vortex-rt_b200 stamps
    VRT_LIB=vortex-rt_b200/libvortexrt_b200_stamps.so python vortex-rt_b200/step_budget.py
    # tensor parallel: the same under torchrun, one rank per GPU
    VRT_LIB=... torchrun --nproc-per-node N --master-addr 127.0.0.1 vortex-rt_b200/step_budget.py

Builds the seeded 27B-shaped model (or --shape 270m), prefills a seeded
prompt, runs warm-up steps, then times single decode steps.  For every mat-vec
and attention launch the timing build records (over the launch's CTAs) the
first start, the first and last release of griddepcontrol.wait, the last CTA
past the tensor-parallel exchange, past its prologue, and the last end
(globaltimer, ns).  Printed per kernel of a layer, medians over layers 1..L-1
and steps, in microseconds:

    total     end of this launch - end of the previous one
    gap       first CTA start - previous end (negative: started early under
              programmatic dependent launch)
    wait      first wait release - previous end
    spread    last - first wait release
    xchg      exchange (peer partial sums + grid barrier), tensor parallel only
    prologue  activation build (norms, quantisation) after the exchange
    main      weight stream / attention after the prologue, to the last CTA end
"""

from __future__ import annotations

import argparse
import ctypes as C
import datetime
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import synth_gguf as sg  # noqa: E402
import vrt  # noqa: E402

NAMES = ["qkv", "attn", "oproj", "gateup", "down"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="27b", choices=["27b", "270m"])
    ap.add_argument("--layers", type=int, default=0, help="fewer layers of the same shape")
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=6)
    ap.add_argument("--seed", type=int, default=1234)
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    nccl_id = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        obj = [vrt.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    L = vrt.lib()
    if not hasattr(L, "vrt_chain_stamps"):
        raise SystemExit("this library has no phase stamps: build `make stamps` and set VRT_LIB to it")
    L.vrt_chain_stamps.argtypes = [C.c_void_p, C.c_uint32]
    L.vrt_chain_stamps.restype = C.c_int
    ctx = vrt.Context(local)
    shape = sg.SHAPES[args.shape]
    if args.layers:
        shape = shape.with_(block_count=args.layers)
    prompt = [2] + np.random.default_rng(4).integers(3, shape.vocab_size, args.prompt_len - 1).tolist()
    m = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=args.seed,
                  max_positions=args.prompt_len + args.steps + 16, tp_rank=rank, tp_world=world, nccl_id=nccl_id,
                  tp_exchange="peer", step_mode="launches")
    m.prefill(prompt)
    m.decode_steps_async(4)
    ctx.sync()
    nl = shape.block_count
    nk = 5 * nl + 2
    buf = np.zeros((2048, 6), np.uint64)
    L.vrt_chain_stamps(buf.ctypes.data, 2048)  # reset
    steps = []
    for _ in range(args.steps):
        if world > 1:
            dist.barrier()
        m.decode_steps_async(1)
        ctx.sync()
        L.vrt_chain_stamps(buf.ctypes.data, 2048)
        steps.append(buf[:nk].astype(np.float64).copy())
    res = {n: {k: [] for k in ("total", "gap", "wait", "spread", "xchg", "pro", "main")} for n in NAMES}
    for r in steps:
        for layer in range(1, nl):
            for j, n in enumerate(NAMES):
                k = 5 * layer + j
                prev_end = r[k - 1, 5]
                s0, s1, s2, s3, s4, s5 = r[k]
                base = s3 if s3 > 0 else s2
                res[n]["total"].append(s5 - prev_end)
                res[n]["gap"].append(s0 - prev_end)
                res[n]["wait"].append(s1 - prev_end)
                res[n]["spread"].append(s2 - s1)
                res[n]["xchg"].append(s3 - s2 if s3 > 0 else 0.0)
                res[n]["pro"].append(s4 - base)
                res[n]["main"].append(s5 - s4)
    step_us = np.median([r[5 * nl, 5] - r[0, 0] for r in steps]) / 1e3
    lines = [f"rank {rank}/{world}, {args.shape} shape, {nl} layers, positions ~{args.prompt_len + 5}: "
             f"QKV0 start -> LM head end {step_us:.1f} us, {step_us / nl:.2f} us per layer",
             "kernel     total     gap    wait  spread    xchg  prologue    main   (us)"]
    for n in NAMES:
        d = {k: float(np.median(v)) / 1e3 for k, v in res[n].items()}
        lines.append(f"{n:8s} {d['total']:7.2f} {d['gap']:7.2f} {d['wait']:7.2f} {d['spread']:7.2f} "
                     f"{d['xchg']:7.2f} {d['pro']:9.2f} {d['main']:7.2f}")
    if rank in (0, world - 1):
        print("\n".join(lines), flush=True)
    m.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
