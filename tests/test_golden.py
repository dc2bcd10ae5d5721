"""The CPU oracle pinned against the reference's known answers.

tests/golden/sampler_golden.json was produced by the reference sample.c
(compiled unmodified, tests/golden/make_golden.py). The plain-C restatement
must reproduce every field of every row bit for bit; so must the reference
build itself when it is present (a check of the harness and the recipe)."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden.make_golden import OUT, case_inputs

with open(OUT) as f:
    GOLDEN = json.load(f)["cases"]


def _check(case, res, rng):
    exp = case["expected"]
    assert res["id"].tolist() == exp["id"], case["name"]
    assert res["n_window"].tolist() == exp["n_window"], case["name"]
    assert res["n_kept"].tolist() == exp["n_kept"], case["name"]
    assert res["greedy"].tolist() == exp["greedy"], case["name"]
    assert res["p_chosen"].view(np.uint32).tolist() == exp["p_chosen_bits"], case["name"]
    assert res["inv_sum"].view(np.uint32).tolist() == exp["inv_sum_bits"], case["name"]
    assert [str(int(x)) for x in rng] == exp["rng_out"], case["name"]


@pytest.mark.parametrize("case", GOLDEN, ids=[c["name"] for c in GOLDEN])
def test_restatement_matches_reference_fixtures(case):
    logits, hist, prm, seeds = case_inputs(case)
    res, rng = O.pick_rows(logits, prm, seeds, hist=hist, backend="oracle")
    _check(case, res, rng)


@pytest.mark.parametrize("case", GOLDEN[:4], ids=[c["name"] for c in GOLDEN[:4]])
def test_reference_build_reproduces_fixtures(case):
    if not O.available("ref"):
        pytest.skip("reference build absent")
    logits, hist, prm, seeds = case_inputs(case)
    res, rng = O.pick_rows(logits, prm, seeds, hist=hist, backend="ref")
    _check(case, res, rng)


def test_fixture_coverage():
    names = {c["name"] for c in GOLDEN}
    for want in ("config1_single_row", "config2_greedy", "config2_topk1", "config3_rows",
                 "config5_zipf"):
        assert want in names
    assert os.path.getsize(OUT) < 200_000
