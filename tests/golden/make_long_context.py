"""Regenerates the long-context parity fixtures tests/golden/long_*.json.

They pin the GPU paths at the contexts the benchmark runs, where the sliding
window has been crossed, the global layers attend over thousands of
positions and the decode attention runs many history splits:

* ``long_270m_prefill4096``  config 2: the 270M shape, a 4096-token seeded
  prompt, then 32 greedy steps (positions 4096..4127), from the reference's
  own token loop (oracle/_ref: src/gemma3.cpp decode_token, prompt tokens
  with top_k = 0 as generate_greedy_tokens does, gemma3.cpp:2080-2149).
* ``long_270m_batch1024``    config 3: four seeded 1024-token prompts, each
  followed by 16 greedy steps, from oracle/_ref.
* ``long_27b_slice2048``     config 4 widths (32 q / 16 KV heads of 128,
  ffn 21504, window 1024) on 6 layers with a 16384-entry vocabulary: a
  2048-token prompt, then 16 greedy steps.  Layer 5 is global and attends
  over 2048+ positions.  The reference refuses 16 KV heads
  (gemma3.cpp:252-257), so this one comes from the C restatement
  (oracle/liboracle.so), which tests/test_oracle.py pins bit for bit to the
  reference build on one-KV-head models.

Each step records the reference's top-8 ids and logits; ``stream[i]`` is the
greedy id emitted by step i (step 0 = the last prompt token).  Run from the
repository root in a container that has the reference tree (a few minutes
on 8 cores):
    python tests/golden/make_long_context.py [name ...]
"""

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "vortex-rt_b200"), os.path.join(ROOT, "oracle")]

import oracle as O  # noqa: E402
import synth_gguf as sg  # noqa: E402

TOPK = 8

CASES = {
    "long_270m_prefill4096": dict(shape="270m", overrides={}, seed=2024, source="reference",
                                  prompts=[(4096, 91)], steps=32),
    "long_270m_batch1024": dict(shape="270m", overrides={}, seed=2024, source="reference",
                                prompts=[(1024, 301), (1024, 302), (1024, 303), (1024, 304)], steps=16),
    "long_27b_slice2048": dict(shape="27b", overrides=dict(block_count=6, vocab_size=16384, name="27b-slice"),
                               seed=27, source="restatement", prompts=[(2048, 92)], steps=16),
}


def prompt_ids(n: int, seed: int, vocab: int) -> list[int]:
    """BOS + n-1 seeded uniform ids in [3, vocab) (the benchmark's prompt rule)."""
    return [2] + np.random.default_rng(seed).integers(3, vocab, n - 1).tolist()


def run_stream(model, prompt: list[int], steps: int) -> dict:
    """Prompt through decode_token (LM head only at the last token), then
    greedy steps; top-8 ids/logits of every step."""
    model.reset()
    for pos, t in enumerate(prompt[:-1]):
        model.decode(t, pos, 0)
    tok, pos = prompt[-1], len(prompt) - 1
    stream, top_ids, top_logits = [], [], []
    for _ in range(steps + 1):
        _, ids, lg = model.decode(tok, pos, TOPK)
        stream.append(int(ids[0]))
        top_ids.append([int(i) for i in ids])
        top_logits.append([float(v) for v in lg])
        tok, pos = int(ids[0]), pos + 1
    return dict(stream=stream, top_ids=top_ids, top_logits=top_logits,
                margins=[lg[0] - lg[1] for lg in top_logits])


def make(name: str, tmp: str) -> dict:
    c = CASES[name]
    shape = sg.SHAPES[c["shape"]].with_(**c["overrides"])
    threads = os.cpu_count() or 1
    P = max(n for n, _ in c["prompts"]) + c["steps"] + 8
    if c["source"] == "reference":
        model = O.Reference(sg.cached_model(shape, c["seed"], tmp), threads=threads)
    else:
        model = O.Oracle(shape=shape, seed=c["seed"], threads=threads, max_positions=P)
    seqs = []
    for n, ps in c["prompts"]:
        t0 = time.time()
        prompt = prompt_ids(n, ps, shape.vocab_size)
        rec = dict(prompt_len=n, prompt_seed=ps, prompt=prompt)
        rec.update(run_stream(model, prompt, c["steps"]))
        seqs.append(rec)
        print(f"{name}: prompt {n} (seed {ps}) in {time.time() - t0:.0f} s, stream {rec['stream'][:6]}...",
              flush=True)
    model.close()
    return dict(name=name, shape=c["shape"], overrides=c["overrides"], seed=c["seed"], top_k=TOPK,
                steps=c["steps"], source={"reference": "oracle/_ref (reference src/gemma3.cpp + src/gguf.cpp)",
                                          "restatement": "oracle/liboracle.so (C restatement, GQA)"}[c["source"]],
                generator="tests/golden/make_long_context.py", sequences=seqs)


def main():
    names = sys.argv[1:] or list(CASES)
    O.build()
    with __import__("tempfile").TemporaryDirectory() as d:
        for name in names:
            out = make(name, d)
            path = os.path.join(HERE, name + ".json")
            with open(path, "w") as f:
                json.dump(out, f, separators=(",", ":"))
            print("wrote", path, os.path.getsize(path), "bytes", flush=True)


if __name__ == "__main__":
    main()
