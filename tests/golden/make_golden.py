"""Regenerates tests/golden/reference_streams.json from the reference's own
token loop (oracle/_ref: src/gemma3.cpp + src/gguf.cpp with the host shim).

Run from the repository root in a container that has the reference tree:
    python tests/golden/make_golden.py
The fixture stores greedy token streams, the top-4 logits of a first token
and the checksum sum_i h_i * (i + 1) of its final hidden state (the
checksum printed by src/gemma_main.cpp:346-387).
"""

import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [os.path.join(ROOT, "vortex-rt_b200"), os.path.join(ROOT, "oracle")]

import oracle as O  # noqa: E402
import synth_gguf as sg  # noqa: E402

CASES = [
    dict(name="tiny_s1234_fused_l8", shape="tiny", seed=1234, lanes=0, fusion=-1, prompt=[2, 300, 301, 302],
         max_new=24),
    dict(name="tiny_s7_unfused_l64", shape="tiny", seed=7, lanes=64, fusion=0, prompt=[2, 17, 260, 261, 262],
         max_new=20),
    dict(name="tiny_w4_s3_l16", shape="tiny", seed=3, lanes=16, fusion=1, prompt=[2, 9], max_new=30,
         overrides=dict(sliding_window=4)),
]


def main():
    O.build()
    out = []
    with __import__("tempfile").TemporaryDirectory() as d:
        for c in CASES:
            shape = sg.SHAPES[c["shape"]].with_(**c.get("overrides", {}))
            path = sg.cached_model(shape, c["seed"], d)
            r = O.Reference(path, lanes=c["lanes"], fusion=c["fusion"])
            toks, _ = r.generate(c["prompt"], c["max_new"])
            r.reset()
            h, ids, lg = r.decode(c["prompt"][0], 0, 4, single=True)
            rec = dict(c)
            rec.update(tokens=toks, first_top4_ids=[int(i) for i in ids],
                       first_top4_logits=[float(v) for v in lg],
                       first_hidden_checksum=float(np.sum(h.astype(np.float64) * np.arange(1, h.size + 1))))
            out.append(rec)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_streams.json")
    with open(path, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "source": "oracle/_ref (reference gemma3.cpp)",
                   "cases": out}, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
