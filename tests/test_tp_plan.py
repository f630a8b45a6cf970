"""Tensor-parallel partitioning, on CPU: world_size-2 gloo ranks each ask the
library for their shard (vrt_tp_plan, no GPU) and all-gather it; the shards
must tile heads, FFN rows and the vocabulary exactly once, in rank order."""

import os

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import synth_gguf as sg
import vrt


def _worker(rank, world, port, shape_name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    s = vrt.tp_plan(vrt.Gemma3Config.from_shape(sg.SHAPES[shape_name]), world, rank)
    mine = [s.q_head0, s.q_heads, s.kv_head0, s.kv_heads, s.ffn0, s.ffn, s.vocab0, s.vocab]
    out = [None] * world
    dist.all_gather_object(out, mine)
    if rank == 0:
        q.put(out)
    dist.destroy_process_group()


@pytest.mark.parametrize("shape_name,world", [("27b", 2), ("tiny-gqa", 2)])
def test_shards_tile_the_model(shape_name, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + world + len(shape_name)
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = q.get(timeout=120)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    shape = sg.SHAPES[shape_name]
    for field, total in ((0, shape.head_count), (2, shape.head_count_kv), (4, shape.feed_forward_length),
                         (6, shape.vocab_size)):
        at = 0
        for r in out:
            assert r[field] == at
            at += r[field + 1]
        assert at == total


def test_uneven_split_rejected():
    cfg = vrt.Gemma3Config.from_shape(sg.SHAPES["270m"])  # one KV head cannot split
    with pytest.raises(vrt.VrtError, match="split evenly"):
        vrt.tp_plan(cfg, 2, 0)
    for w in (1, 2, 4, 8):
        vrt.tp_plan(vrt.Gemma3Config.from_shape(sg.SHAPES["27b"]), w, w - 1)
