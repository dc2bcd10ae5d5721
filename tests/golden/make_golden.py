"""Generate tests/golden/sampler_golden.json from the REFERENCE sampler.

Runs franzvill/quasar sample.c, compiled unmodified into oracle/_ref by
oracle/Makefile (one quasar_sampler object per row, configured through its own
quasar_sampler_config, history injected, quasar_sampler_pick), on seeded
synthetic inputs whose recipe (oracle/synth.c, mirrored bit for bit on the
device by quasar_b200/csrc/synth.cu) is stored with each case. The reference
ships no sampler tests or vectors, so these fixtures are the pinned known
answers: the CPU suite checks the C restatement against them and the GPU suite
checks the CUDA sampler against them.

    python tests/golden/make_golden.py     (needs the reference tree; CPU only)
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_golden.json")
V = 151936

# name, synth kind, logits seed, row0, rows, vocab, scale, history ids, history seed,
# params (scalars, or "temperature": ["uniform", seed, lo, hi]), PRNG seed base
CASES = [
    ("config1_single_row", O.SYNTH_NORMAL, 42, 0, 1, V, 3.0, 64, 42,
     dict(temperature=0.7, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.1), 42),
    ("config2_greedy", O.SYNTH_GUMBEL_PEAK, 2, 0, 24, V, 1.0, 0, 0,
     dict(temperature=0.0), 1000),
    ("config2_greedy_penalty", O.SYNTH_GUMBEL_PEAK, 2, 24, 24, V, 1.0, 64, 3,
     dict(temperature=0.0, repeat_penalty=1.1), 1000),
    ("config2_topk1", O.SYNTH_GUMBEL_PEAK, 2, 0, 24, V, 1.0, 0, 0,
     dict(temperature=1.0, top_k=1), 1000),
    ("config3_rows", O.SYNTH_NORMAL, 3, 0, 48, V, 3.0, 256, 33,
     dict(temperature=["uniform", 3, 0.2, 1.5], top_p=0.95, min_p=0.05, repeat_penalty=1.1), 5000),
    ("config4_params_full_rows", O.SYNTH_NORMAL, 4, 0, 16, V, 3.0, 0, 0,
     dict(temperature=0.8, top_k=40, top_p=0.9), 7000),
    ("config5_zipf", O.SYNTH_ZIPF, 5, 0, 24, V, 1.1, 2048, 55,
     dict(temperature=1.0, top_p=1.0, min_p=0.1, repeat_penalty=1.3), 9000),
    ("multinomial_full_vocab", O.SYNTH_NORMAL, 6, 0, 8, V, 3.0, 0, 0,
     dict(temperature=1.0), 11000),
    ("nucleus_only", O.SYNTH_NORMAL, 7, 0, 8, V, 3.0, 64, 7,
     dict(temperature=0.7, top_p=0.95, repeat_penalty=1.1), 12000),
]
for v_small in (1, 2, 31, 33, 4095):
    for j, prm in enumerate((dict(temperature=0.0, repeat_penalty=1.5),
                             dict(temperature=0.9, min_p=0.05, repeat_penalty=1.2),
                             dict(temperature=1.3, top_p=0.7, top_k=5),
                             dict(temperature=2.0))):
        CASES.append((f"small_v{v_small}_p{j}", O.SYNTH_NORMAL, 100 + v_small, 0, 8, v_small, 2.0,
                      min(8, v_small), v_small, prm, 300 + j))


def case_inputs(case: dict):
    """Regenerate a case's inputs (logits, hist, params, seeds) with the C recipe."""
    B, Vc = case["rows"], case["vocab"]
    logits = O.synth_logits(case["kind"], case["seed"], case["row0"], B, Vc, case["scale"],
                            backend="oracle")
    hist = None
    if case["history"]:
        hist = O.synth_hist(case["hist_seed"], case["row0"], B, case["history"], Vc, backend="oracle")
    kw = dict(case["params"])
    if isinstance(kw.get("temperature"), list):
        _, s, lo, hi = kw["temperature"]
        kw["temperature"] = O.synth_uniform(s, case["row0"], B, lo, hi, backend="oracle")
        prm = O.make_params(B, **kw)
    else:
        prm = O.make_params(1, **kw)
    seeds = np.arange(case["row0"], case["row0"] + B, dtype=np.uint64) + np.uint64(case["rng_base"])
    return logits, hist, prm, seeds


def main():
    if not O.available("ref"):
        O.build()
    assert O.available("ref"), "the reference build (oracle/_ref) is required"
    out = {"generator": "tests/golden/make_golden.py",
           "oracle": "reference sample.c via oracle/_ref/libsample_ref.so",
           "cases": []}
    for (name, kind, seed, row0, rows, vocab, scale, H, hseed, params, rbase) in CASES:
        case = dict(name=name, kind=kind, seed=seed, row0=row0, rows=rows, vocab=vocab, scale=scale,
                    history=H, hist_seed=hseed, params=params, rng_base=rbase)
        logits, hist, prm, seeds = case_inputs(case)
        res, rng = O.pick_rows(logits, prm, seeds, hist=hist, backend="ref")
        case["expected"] = {
            "id": res["id"].tolist(),
            "n_window": res["n_window"].tolist(),
            "n_kept": res["n_kept"].tolist(),
            "greedy": res["greedy"].tolist(),
            "p_chosen_bits": res["p_chosen"].view(np.uint32).tolist(),
            "inv_sum_bits": res["inv_sum"].view(np.uint32).tolist(),
            "margin": [float(m) if np.isfinite(m) else None for m in res["margin"]],
            "rng_out": [str(int(x)) for x in rng],
        }
        out["cases"].append(case)
        print(f"{name}: ids {res['id'][:6].tolist()} kept {res['n_kept'][:6].tolist()}")
    with open(OUT, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
