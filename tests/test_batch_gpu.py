"""Multi-request decode: several requests, each with its own KV cache, advance
one token per step over one shared pass of the weights.

Each request's greedy tokens must equal the oracle's for that request alone
(prefill of its own prompt, then one plamo_forward per token), across sliding
window eviction and prompts of different lengths. A token outside the
vocabulary declines the whole step and changes nothing.
"""
import ctypes

import numpy as np
import pytest

from conftest import expect, load_oracle, load_package
from fixtures import oracle_forward, oracle_prefill

pytestmark = pytest.mark.gpu


def profile(pkg):
    return pkg.Profile("batch", 512, 4, 8, 2, 128, 1024, vocab=1000, window=16, pattern=2, max_position=512)


def shared_requests(backend, prof, count, seed):
    """`count` device requests over one synthetic weight set, and host copies of
    those weights for the oracle."""
    pkg = load_package()
    first = pkg.HostModel(prof, weights="synthetic")
    backend.preload_synthetic(first, seed)
    reqs = [first] + [pkg.HostModel(prof, weights_of=first) for _ in range(count - 1)]
    for r in reqs:
        backend.prepare(r)
    blob = np.empty(first.blob_bytes // 2, dtype=np.uint16)
    host = pkg.HostModel(prof, weights=blob)
    for (ka, n, _), (kb, _, _) in zip(first.tensor_ranges(), host.tensor_ranges()):
        assert backend.lib.plamo_cuda_read_weights(backend.ctx, ka, kb, 2 * n) == 1
    return reqs, blob


def oracle_tokens(prof, blob, ids, steps):
    pkg = load_package()
    o = load_oracle()
    hm = pkg.HostModel(prof, weights=blob)
    ok, _ = oracle_prefill(hm, ids)
    assert ok == 1
    out = [int(o.plamo_argmax(hm.model.logits, prof.vocab))]
    for _ in range(steps):
        assert oracle_forward(hm, out[-1]) == 1
        out.append(int(o.plamo_argmax(hm.model.logits, prof.vocab)))
    return out


@pytest.mark.parametrize("count", [1, 4, 8])
def test_batch_decode_matches_oracle_per_request(backend, count):
    pkg = load_package()
    prof = profile(pkg)
    reqs, blob = shared_requests(backend, prof, count, seed=17)
    lib = backend.lib
    prompts = [np.random.default_rng(100 + i).integers(3, prof.vocab, size=9 + 3 * i).astype(np.uint32)
               for i in range(count)]
    tokens = np.zeros(count, dtype=np.uint32)
    nxt = ctypes.c_uint32()
    for i, (r, ids) in enumerate(zip(reqs, prompts)):
        expect(backend, lib.plamo_cuda_prefill_greedy(backend.ctx, r.ptr, ids.ctypes.data, len(ids),
                                                      ctypes.byref(nxt)))
        tokens[i] = nxt.value
    arr = (ctypes.c_void_p * count)(*[ctypes.addressof(r.model) for r in reqs])
    batch = lib.plamo_cuda_batch_open(backend.ctx, arr, count)
    assert batch, backend.info().note
    try:
        steps = 20
        got = [[int(t)] for t in tokens]
        for _ in range(steps):
            out = np.zeros(count, dtype=np.uint32)
            expect(backend, lib.plamo_cuda_batch_step(batch, tokens.ctypes.data, out.ctypes.data))
            for i in range(count):
                got[i].append(int(out[i]))
            tokens = out
        for i in range(count):
            assert reqs[i].caches[0].count == min(len(prompts[i]) + steps, 17)  # sliding window (16 + 1)
            assert reqs[i].caches[1].count == len(prompts[i]) + steps
            assert got[i] == oracle_tokens(prof, blob, prompts[i], steps), f"request {i}"
        # A token outside the vocabulary declines the step; nothing moves.
        bad = tokens.copy()
        bad[-1] = prof.vocab
        counts = [r.caches[1].count for r in reqs]
        out = np.zeros(count, dtype=np.uint32)
        assert lib.plamo_cuda_batch_step(batch, bad.ctypes.data, out.ctypes.data) == 0
        assert [r.caches[1].count for r in reqs] == counts
    finally:
        lib.plamo_cuda_batch_close(batch)
        for r in reqs:
            lib.plamo_cuda_release_model(backend.ctx, r.ptr)


def test_batch_rejects_mismatched_requests(backend):
    pkg = load_package()
    prof = profile(pkg)
    a = pkg.HostModel(prof, weights="synthetic")
    b = pkg.HostModel(prof, weights="synthetic")  # other weights
    backend.preload_synthetic(a, 1)
    backend.preload_synthetic(b, 2)
    backend.prepare(a)
    backend.prepare(b)
    lib = backend.lib
    two = (ctypes.c_void_p * 2)(ctypes.addressof(a.model), ctypes.addressof(b.model))
    assert not lib.plamo_cuda_batch_open(backend.ctx, two, 2)
    same = (ctypes.c_void_p * 2)(ctypes.addressof(a.model), ctypes.addressof(a.model))
    assert not lib.plamo_cuda_batch_open(backend.ctx, same, 2)  # one cache per request
    one = (ctypes.c_void_p * 1)(ctypes.addressof(a.model))
    batch = lib.plamo_cuda_batch_open(backend.ctx, one, 1)
    assert batch
    lib.plamo_cuda_batch_close(batch)
