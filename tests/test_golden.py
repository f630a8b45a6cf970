"""Committed golden fixtures (tests/golden/*.json, made by tests/golden/make_golden.py
from the reference's own token loop, oracle/_ref).  They pin the oracle on any
machine, including ones without the reference tree."""

import json
import os

import numpy as np
import pytest

import oracle as O
import synth_gguf as sg

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_streams.json")


def cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_oracle_matches_golden(case, model_dir):
    shape = sg.SHAPES[case["shape"]].with_(**case.get("overrides", {}))
    path = sg.cached_model(shape, case["seed"], model_dir)
    o = O.Oracle(path, lanes=case["lanes"], fusion=case["fusion"])
    assert o.generate(case["prompt"], case["max_new"]) == case["tokens"]
    o.reset()
    h, ids, lg = o.decode(case["prompt"][0], 0, 4)
    assert [int(i) for i in ids] == case["first_top4_ids"]
    assert np.allclose(lg, case["first_top4_logits"], rtol=0, atol=0)
    chk = float(np.sum(h.astype(np.float64) * np.arange(1, h.size + 1)))
    assert chk == case["first_hidden_checksum"]
