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
