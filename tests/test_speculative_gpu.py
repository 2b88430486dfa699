"""Speculative decoding (reference runtime/engine.c:523-586, draft proposer
runtime/worker.c:198-318, rollback runtime/draft.c:258-297).

The speculative loop must emit exactly the target's greedy tokens whatever the
draft proposes: with a draft identical to the target (every proposal accepted,
long horizons, many commits) and with an unrelated draft (almost every
proposal rejected, rollbacks). The small profile has a 16-row sliding window,
so commits and draft rollbacks cross window evictions.
"""
import ctypes

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu


def small_profile(pkg):
    return pkg.Profile("small", 256, 4, 4, 2, 64, 512, vocab=1000, window=16, pattern=2, max_position=512)


def plain(backend, hm, ids, n):
    pkg = load_package()
    out = np.zeros(n, dtype=np.uint32)
    t = pkg._abi.CudaTiming()
    k = backend.lib.plamo_cuda_generate(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), n, out.ctypes.data,
                                        pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(t))
    assert k >= 0, backend.info().note
    return [int(x) for x in out[:k]]


def speculative(backend, target, draft, ids, n, block):
    pkg = load_package()
    out = np.zeros(n, dtype=np.uint32)
    st = pkg._abi.CudaSpeculation()
    k = backend.lib.plamo_cuda_generate_speculative(backend.ctx, target.ptr, draft.ptr, ids.ctypes.data, len(ids),
                                                    n, block, out.ctypes.data, pkg._abi.TOKEN_CALLBACK(), None,
                                                    ctypes.byref(st))
    assert k >= 0, backend.info().note
    return [int(x) for x in out[:k]], st


@pytest.mark.parametrize("block", [2, 4, 16])
def test_identical_draft_accepts_and_matches_greedy(backend, block):
    pkg = load_package()
    prof = small_profile(pkg)
    target = pkg.HostModel(prof, weights="synthetic")
    backend.preload_synthetic(target, seed=21)
    draft = pkg.HostModel(prof, weights="synthetic")
    backend.preload_synthetic(draft, seed=21)
    backend.prepare(target)
    backend.prepare(draft)
    ids = np.random.default_rng(5).integers(3, 1000, size=20).astype(np.uint32)
    want = plain(backend, target, ids, 60)
    got, st = speculative(backend, target, draft, ids, 60, block)
    assert got == want
    assert st.verify_batches > 0
    assert st.accepted_tokens >= (len(got) - 1) // 2  # identical models agree on (nearly) everything


@pytest.mark.parametrize("block", [4, 16])
def test_unrelated_draft_rolls_back_and_matches_greedy(backend, block):
    pkg = load_package()
    prof = small_profile(pkg)
    target = pkg.HostModel(prof, weights="synthetic")
    backend.preload_synthetic(target, seed=21)
    draft = pkg.HostModel(prof, weights="synthetic")
    backend.preload_synthetic(draft, seed=99)
    backend.prepare(target)
    backend.prepare(draft)
    ids = np.random.default_rng(6).integers(3, 1000, size=25).astype(np.uint32)
    want = plain(backend, target, ids, 50)
    got, st = speculative(backend, target, draft, ids, 50, block)
    assert got == want
    assert st.verify_batches > 0


def test_greedy_margin_is_the_top2_logit_gap(backend):
    """The draft's confidence (reference runtime/worker.c:268-286): best logit
    minus the largest logit at any other index, for the step just decoded."""
    pkg = load_package()
    prof = small_profile(pkg)
    a = pkg.HostModel(prof, weights="synthetic")
    backend.preload_synthetic(a, seed=33)
    b = pkg.HostModel(prof, weights_of=a)
    backend.prepare(a)
    backend.prepare(b)
    lib = backend.lib
    ids = np.random.default_rng(4).integers(3, prof.vocab, size=9).astype(np.uint32)
    nxt = ctypes.c_uint32()
    for hm in (a, b):
        assert lib.plamo_cuda_prefill_greedy(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), ctypes.byref(nxt)) == 1
    token = nxt.value
    for _ in range(5):
        assert lib.plamo_cuda_forward(backend.ctx, a.ptr, token) == 1
        margin = ctypes.c_float()
        assert lib.plamo_cuda_forward_greedy_margin(backend.ctx, b.ptr, token, ctypes.byref(nxt),
                                                    ctypes.byref(margin)) == 1
        logits = a.logits_array()
        best = int(np.argmax(logits))
        assert nxt.value == best
        rest = np.delete(logits, best)
        assert margin.value == np.float32(logits[best] - rest.max())
        token = nxt.value
    lib.plamo_cuda_release_model(backend.ctx, b.ptr)
    lib.plamo_cuda_release_model(backend.ctx, a.ptr)


def test_config5_form_matches_the_oracle_greedy_tokens(backend):
    """The speculative loop of BASELINE config 5 on one GPU: a 0.8B-shaped
    draft proposing 4 tokens per verification for a larger target (the 2B
    profile here, whose oracle run fits the host), 64 tokens after an 81-id
    prompt - identical to the oracle's greedy tokens, not only to the GPU's
    own greedy path."""
    import os
    from conftest import load_oracle
    from test_model_gpu import oracle_generate, synthetic_pair
    pkg = load_package()
    load_oracle().oracle_set_threads(os.cpu_count() or 1)
    target, host = synthetic_pair(backend, pkg.PROFILES["2b"], seed=3, full_capacity=8208)
    draft = pkg.HostModel(pkg.PROFILES["0.8b"], weights="synthetic", full_capacity=8208)
    backend.preload_synthetic(draft, seed=6)
    backend.prepare(draft)
    ids = np.random.default_rng(1).integers(3, 100000, size=81).astype(np.uint32)
    want, margins = oracle_generate(host, ids, 64)
    got, st = speculative(backend, target, draft, ids, 64, 4)
    assert got == want, f"margins {margins}"
    assert st.verify_batches > 0
