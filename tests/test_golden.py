"""The oracle against the committed golden fixtures (tests/golden/).

The fixtures were written by tests/golden/make_golden.py from the oracle while
it was pinned by the reference's own known-answer tests; here the oracle must
reproduce every one of them bit for bit, on any machine, so a change to the
oracle (or to the seeded input generators) cannot pass silently where the
reference checkout is absent.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import make_golden as golden  # noqa: E402
from conftest import load_oracle  # noqa: E402


def fixture(name):
    return np.load(os.path.join(HERE, "golden", f"{name}.npz"))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture(autouse=True)
def single_thread():
    load_oracle().oracle_set_threads(1)


@pytest.mark.parametrize("rows,cols", golden.GEMV_SHAPES)
def test_oracle_matvec_reproduces_golden(rows, cols):
    g = fixture("gemv")
    key = f"{rows}x{cols}"
    w, x = golden.gemv_inputs(rows, cols)
    assert golden.sha256(w) == str(g[f"w_sha256_{key}"]), "weight generator drifted"
    assert golden.sha256(x) == str(g[f"x_sha256_{key}"]), "input generator drifted"
    assert np.array_equal(bits(golden.oracle_matvec(w, x)), bits(g[f"y_{key}"]))


def test_oracle_small_model_reproduces_golden():
    g = fixture("model_small")
    hm = golden.small_host_model()
    assert golden.sha256(hm.tensor("model.embed_tokens.weight")) == str(g["embed_sha256"])
    ids = golden.small_prompt()
    assert np.array_equal(ids, g["ids"])
    golden.oracle_prefill(hm, ids)
    assert np.array_equal(bits(hm.logits_array()), bits(g["prefill_logits"]))
    assert np.array_equal(bits(hm.state_array()), bits(g["prefill_state"]))
    tokens, margins = golden.oracle_greedy(hm, golden.SMALL_TOKENS)
    assert np.array_equal(tokens, g["tokens"])
    assert np.array_equal(bits(margins), bits(g["margins"]))


def test_oracle_decode_fixture_reproduces_golden():
    g = fixture("decode_fixture")
    hm = golden.fixture_model()
    o = load_oracle()
    golden.oracle_prefill(hm, g["ids"])
    got_states, got_logits = [hm.state_array().copy()], [hm.logits_array().copy()]
    for t in g["steps"]:
        assert o.plamo_forward(hm.ptr, int(t)) == 1
        got_states.append(hm.state_array().copy())
        got_logits.append(hm.logits_array().copy())
    assert np.array_equal(bits(np.stack(got_states)), bits(g["states"]))
    assert np.array_equal(bits(np.stack(got_logits)), bits(g["logits"]))
