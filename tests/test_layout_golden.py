"""The package's model description against the reference's own generators.

tests/golden/layout.json holds what the reference's Python tools produce for
the 0.8B, 2B, 8B and 31B profiles (tests/golden/make_layout_golden.py runs
tools/weight_schema.py, tools/model_layout.py and tools/rope_constants.py).
The package restates them to build the descriptor trees the CUDA path
reads; here every profile parameter, schema row, per-layer window / capacity /
table / concentration and both FP32 frequency tables must match exactly.
"""
import json
import os

import numpy as np
import pytest

from conftest import ROOT, load_package

with open(os.path.join(ROOT, "tests", "golden", "layout.json")) as f:
    GOLDEN = json.load(f)


@pytest.mark.parametrize("name", sorted(GOLDEN))
def test_profile_matches_reference_config(name):
    p = load_package().PROFILES[name]
    c = GOLDEN[name]["config"]
    assert (p.hidden, p.layers, p.qh, p.kh, p.dim, p.inter, p.vocab) == (
        c["hidden_size"], c["num_hidden_layers"], c["num_attention_heads"], c["num_key_value_heads"],
        c["head_dim"], c["intermediate_size"], c["vocab_size"])
    assert (p.window, p.pattern, p.tied, p.max_position) == (
        c["window_size"], c["sliding_window_pattern"], c["tie_word_embeddings"], c["max_position_embeddings"])


@pytest.mark.parametrize("name", sorted(GOLDEN))
def test_weight_schema_matches_reference(name):
    pkg = load_package()
    got = [[n, list(s)] for n, s in pkg.schema(pkg.PROFILES[name])]
    assert got == GOLDEN[name]["schema"]


@pytest.mark.parametrize("name", sorted(GOLDEN))
def test_layer_specs_match_reference_descriptors(name):
    pkg = load_package()
    g = GOLDEN[name]
    local = np.array(g["rope_local"], dtype=np.float32)
    glob = np.array(g["rope_global"], dtype=np.float32)
    specs = pkg.default_layer_specs(pkg.PROFILES[name])
    assert len(specs) == len(g["layers"])
    for i, (s, want) in enumerate(zip(specs, g["layers"])):
        assert s.sliding == want["sliding"], i
        assert s.capacity == want["capacity"], i
        assert np.float32(s.scale) == np.float32(want["scale"]), i
        table = glob if want["table"] == "global" else local
        assert np.array_equal(np.asarray(s.freq, dtype=np.float32).view(np.uint32), table.view(np.uint32)), i
    assert np.float32(pkg.concentration(pkg.PROFILES[name].yarn_factor)) == np.float32(g["global_concentration"])
