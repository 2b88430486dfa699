"""Whole-model greedy decode parity (configs 3 and 4) against the oracle.

Token identity is the bar (identical greedy tokens for
the first 64 tokens); logits and states are also held to the reference's GPU
acceptance rule after prefill. The top-2 logit margin of every oracle step
is reported so that a flip could be told apart from a near tie.
"""
import ctypes
import os

import numpy as np
import pytest

import synthetic
from conftest import load_oracle, load_package, rel_l2
from fixtures import oracle_forward, oracle_prefill

pytestmark = pytest.mark.gpu


def oracle_generate(hm, ids, max_tokens):
    o = load_oracle()
    ok, _ = oracle_prefill(hm, ids)
    assert ok == 1
    out, margins = [], []
    for _ in range(max_tokens):
        logits = hm.logits_array()
        top = np.partition(logits, -2)[-2:]
        margins.append(float(top[1] - top[0]))
        t = int(o.plamo_argmax(hm.model.logits, hm.profile.vocab))
        if t in (1, 16):
            break
        out.append(t)
        if len(out) == max_tokens:
            break
        assert oracle_forward(hm, t) == 1
    return out, margins


def gpu_generate(backend, hm, ids, max_tokens):
    pkg = load_package()
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    out = np.zeros(max_tokens, dtype=np.uint32)
    timing = pkg._abi.CudaTiming()
    n = backend.lib.plamo_cuda_generate(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), max_tokens,
                                        out.ctypes.data, pkg._abi.TOKEN_CALLBACK(), None,
                                        ctypes.byref(timing))
    assert n >= 0, backend.info().note
    return [int(t) for t in out[:n]]


def synthetic_pair(backend, profile, seed, full_capacity=None, specs=None):
    pkg = load_package()
    a = pkg.HostModel(profile, specs, weights="synthetic", full_capacity=full_capacity)
    backend.preload_synthetic(a, seed)
    blob = np.empty(a.blob_bytes // 2, dtype=np.uint16)
    b = pkg.HostModel(profile, specs, weights=blob, full_capacity=full_capacity)
    for (ka, count, _), (kb, _, _) in zip(a.tensor_ranges(), b.tensor_ranges()):
        assert backend.lib.plamo_cuda_read_weights(backend.ctx, ka, kb, 2 * count) == 1
    backend.prepare(a)
    return a, b


def test_small_model_with_window_eviction(backend):
    """4 layers (2 sliding with a 16-row window, 2 full), prompt 20, 48 tokens:
    sliding eviction during prefill and during decode."""
    pkg = load_package()
    prof = pkg.Profile("small", 256, 4, 4, 2, 64, 512, vocab=1000, window=16, pattern=2,
                       max_position=512)
    a, b = synthetic_pair(backend, prof, seed=11)
    b_blob_check = synthetic.bf16(11 * 1000003 + 0, 16, 0.0, 0.02)
    assert np.array_equal(b.tensor("model.embed_tokens.weight").reshape(-1)[:16], b_blob_check)
    ids = np.random.default_rng(1).integers(3, 1000, size=20).astype(np.uint32)
    want, margins = oracle_generate(b, ids, 48)
    got = gpu_generate(backend, a, ids, 48)
    assert got == want, f"margins {margins}"


@pytest.mark.parametrize("name,prompt,tokens", [("2b", 81, 64)])
def test_profile_greedy_tokens_match_oracle(backend, name, prompt, tokens):
    """Config 3: 2B profile, 81-id prompt from default_rng(1) over [3, 100000),
    64 greedy tokens identical to the oracle's."""
    pkg = load_package()
    load_oracle().oracle_set_threads(os.cpu_count() or 1)
    a, b = synthetic_pair(backend, pkg.PROFILES[name], seed=3, full_capacity=8208)
    ids = np.random.default_rng(1).integers(3, 100000, size=prompt).astype(np.uint32)
    want, margins = oracle_generate(b, ids, tokens)
    got = gpu_generate(backend, a, ids, tokens)
    print(f"{name}: min top-2 margin {min(margins):.4g}")
    assert got == want, f"margins {margins}"


def test_8b_prefix_greedy_tokens_and_logits(backend):
    """Config 4 on a token prefix: 8B profile, 12-id prompt, 6 greedy tokens,
    prefill logits and state within the reference's whole-model rule (the
    oracle streams 16 GB per token on the host)."""
    pkg = load_package()
    load_oracle().oracle_set_threads(os.cpu_count() or 1)
    a, b = synthetic_pair(backend, pkg.PROFILES["8b"], seed=4, full_capacity=8208)
    ids = np.random.default_rng(1).integers(3, 100000, size=12).astype(np.uint32)
    assert backend.lib.plamo_cuda_prefill(backend.ctx, a.ptr, ids.ctypes.data, len(ids), 0) == 1
    ok, _ = oracle_prefill(b, ids)
    assert ok == 1
    # Whole-model rule of reference tools/compare_backends.py:16-33: finite
    # values and relative L2 <= 1e-4 (the per-layer max-abs bound of
    # tests/metal_decode.c does not apply across 32 layers).
    for name, x, y in (("logits", a.logits_array(), b.logits_array()),
                       ("state", a.state_array(), b.state_array())):
        assert np.all(np.isfinite(x)) and np.all(np.isfinite(y)), name
        assert rel_l2(x, y) <= 1e-4, f"8b prefill {name}: {rel_l2(x, y):.3g}"
    a.reset()
    b.reset()
    want, margins = oracle_generate(b, ids, 6)
    got = gpu_generate(backend, a, ids, 6)
    assert got == want, f"margins {margins}"


def test_08b_draft_profile_greedy_tokens_match_oracle(backend):
    """The 0.8B draft profile of config 5 (16 query heads over one KV head, so
    every grouped-query path runs with G = 16): 30-id prompt, 32 greedy tokens
    identical to the oracle's."""
    pkg = load_package()
    load_oracle().oracle_set_threads(os.cpu_count() or 1)
    a, b = synthetic_pair(backend, pkg.PROFILES["0.8b"], seed=6, full_capacity=8208)
    ids = np.random.default_rng(2).integers(3, 100000, size=30).astype(np.uint32)
    want, margins = oracle_generate(b, ids, 32)
    got = gpu_generate(backend, a, ids, 32)
    assert got == want, f"margins {margins}"


def test_31b_shaped_layers_match_oracle(backend):
    """Layers of the 31B profile's exact shape (hidden 5120: rows end inside a
    chunk of 3 rows of ten 512-column slots; 64 query and 8 KV heads; the
    tied head) - two of them, one sliding and one full - against the oracle:
    prefill logits under the whole-model rule, then 6 greedy tokens."""
    from dataclasses import replace
    pkg = load_package()
    load_oracle().oracle_set_threads(os.cpu_count() or 1)
    prof = replace(pkg.PROFILES["31b"], name="31b-2layers", layers=2, pattern=2)
    a, b = synthetic_pair(backend, prof, seed=8, full_capacity=1024)
    ids = np.random.default_rng(1).integers(3, 100000, size=20).astype(np.uint32)
    assert backend.lib.plamo_cuda_prefill(backend.ctx, a.ptr, ids.ctypes.data, len(ids), 0) == 1
    ok, _ = oracle_prefill(b, ids)
    assert ok == 1
    for name, x, y in (("logits", a.logits_array(), b.logits_array()),
                       ("state", a.state_array(), b.state_array())):
        assert np.all(np.isfinite(x)) and np.all(np.isfinite(y)), name
        assert rel_l2(x, y) <= 1e-4, f"31b-shaped prefill {name}: {rel_l2(x, y):.3g}"
    a.reset()
    b.reset()
    want, margins = oracle_generate(b, ids, 6)
    got = gpu_generate(backend, a, ids, 6)
    assert got == want, f"margins {margins}"
