"""The oracle's restatement of build_functional_lora (src/lora.h:372-622): its low-rank fold of a
chain of lora / dora-rows adapters equals the chain applied to the materialized weight, adapter
after adapter (the weight dit_lin's term path stands for).  CPU only."""
import numpy as np
import pytest

import oracle


def _terms(rng, inn, out, spec):
    terms = []
    for kind, r, strength in spec:
        A = rng.normal(0, 1 / np.sqrt(inn), (r, inn))
        B = rng.normal(0, 0.05, (out, r))
        m = rng.uniform(0.5, 1.5, out) if kind == "dora" else None
        terms.append((A, B, m, 8.0 / r * strength))
    return terms


@pytest.mark.parametrize("spec", [
    [("lora", 4, 1.0)],
    [("dora", 4, 1.0)],
    [("lora", 4, 0.75), ("dora", 8, 1.0)],
    [("dora", 4, 1.0), ("lora", 4, 0.5), ("dora", 4, 1.0)],
    [("dora", 16, 1.0), ("dora", 16, 1.0), ("lora", 8, 1.0)],
])
def test_fold_equals_sequential_chain(spec):
    rng = np.random.default_rng(len(spec))
    inn, out = 96, 40
    W = rng.normal(0, 0.05, (out, inn))
    terms = _terms(rng, inn, out, spec)
    x = rng.standard_normal((7, inn))
    y_fold = oracle.functional_chain_forward(x, W, terms)
    y_def = x @ oracle.chain_weight(W, terms).T
    assert np.abs(y_fold - y_def).max() < 1e-9 * np.abs(y_def).max()
