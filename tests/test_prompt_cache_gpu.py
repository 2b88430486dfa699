"""Device prompt (template prefix) cache.

The first test is reference tests/prompt_cache.c:13-87 run against the device
snapshots: the same two-layer shape class, ids, misuse cases and checks
(bitwise KV after restore, exact ids, immutable independent snapshots, misses
that change nothing, repeated restoration). The host K/V arrays are kept
current by the backend (copy_kv_to_host), so the restored rows are read back
through them. The second test runs the engine's request flow (reference
runtime/engine.c:358-381 capture after a fresh prefill of the template,
engine.c:474-479 restore then prefill of the suffix) and requires the same
greedy tokens, logits and KV as a full prefill of the whole prompt.
"""
import ctypes

import numpy as np
import pytest

from conftest import expect, load_package
from fixtures import decode_fixture_pair

pytestmark = pytest.mark.gpu


@pytest.fixture
def host_backend(pkg):
    b = pkg.Backend(device=0, max_context=4200, max_prefill=4096, copy_kv_to_host=True)
    yield b
    b.close()


def u32(values):
    return np.ascontiguousarray(values, dtype=np.uint32)


def capture(backend, hm, ids, tokens):
    return backend.lib.plamo_cuda_prompt_cache_capture(backend.ctx, hm.ptr, ids.ctypes.data, tokens)


def restore(backend, snap, hm, ids, tokens):
    return backend.lib.plamo_cuda_prompt_cache_restore(backend.ctx, snap, hm.ptr, ids.ctypes.data, tokens)


def prefill(backend, hm, ids):
    nxt = ctypes.c_uint32()
    expect(backend, backend.lib.plamo_cuda_prefill_greedy(backend.ctx, hm.ptr, ids.ctypes.data, len(ids),
                                                          ctypes.byref(nxt)))
    return int(nxt.value)


def test_snapshot_semantics_mirror_reference(host_backend):
    b, lib = host_backend, host_backend.lib
    L, N = 2, 3
    hm, _ = decode_fixture_pair(64, 96, 16, 19, vocab=32)
    b.preload_model(hm)
    b.prepare(hm)
    ids, wrong = u32([1, 19, 7, 5, 9, 11]), u32([1, 18, 7, 5, 9, 11])
    prefill(b, hm, ids[:N])
    original = [hm.kv_arrays(i) for i in range(L)]
    scales = [hm.rotation(i).scale_bits for i in range(L)]
    kvw = hm.profile.kh * hm.profile.dim

    a = capture(b, hm, ids, N)
    assert a, b.info().note
    assert lib.plamo_cuda_prompt_cache_tokens(a) == N
    assert lib.plamo_cuda_prompt_cache_bytes(a) >= L * 2 * N * kvw * 4
    assert not capture(b, hm, ids, 0)
    long_ids = u32(np.arange(70))
    assert not capture(b, hm, long_ids, load_package()._abi.PREFIX_LIMIT + 1)
    hm.caches[1].count = N + 1  # the host grew one layer: counts disagree
    assert not capture(b, hm, ids, N)
    hm.caches[1].count = N
    hm.caches[1].width = 2**64 - 1
    assert not capture(b, hm, ids, N)
    hm.caches[1].width = kvw
    # The host rewrites its rows (to zeros): the backend uploads them, so a
    # snapshot taken now holds zeros.
    for i in range(L):
        for arr in (hm.caches[i].k, hm.caches[i].v, hm.rotation(i).out):
            hm.view(arr, hm.caches[i].capacity * kvw)[:] = 0
    zero = capture(b, hm, wrong, N)
    assert zero, b.info().note

    for i in range(L):
        hm.caches[i].count = 0
        hm.rotation(i).processed_count = 0
    assert restore(b, a, hm, wrong, 6) == 0
    assert restore(b, a, hm, ids, N - 1) == 0
    assert restore(b, a, hm, ids, N) == 0
    hm.caches[1].capacity = N - 1
    assert restore(b, a, hm, ids, 6) == 0
    # A failed last destination cannot modify the first.
    assert hm.caches[0].count == 0 and hm.view(hm.caches[0].k, kvw)[0] == 0
    hm.caches[1].capacity = 19
    for _ in range(3):
        assert restore(b, a, hm, ids, 6) == N
        for i in range(L):
            assert hm.caches[i].count == N and hm.rotation(i).processed_count == N
            assert hm.rotation(i).scale_bits == scales[i]
            for got, want in zip(hm.kv_arrays(i), original[i]):
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert restore(b, zero, hm, wrong, 6) == N
        for i in range(L):
            for got in hm.kv_arrays(i):
                assert not np.any(got)
    assert restore(b, None, hm, ids, 6) == 0
    assert lib.plamo_cuda_prompt_cache_tokens(None) == 0 and lib.plamo_cuda_prompt_cache_bytes(None) == 0
    lib.plamo_cuda_prompt_cache_free(a)
    lib.plamo_cuda_prompt_cache_free(zero)
    lib.plamo_cuda_prompt_cache_free(None)
    b.release(hm)


def greedy_tail(backend, hm, first, steps):
    out, t = [first], ctypes.c_uint32()
    for _ in range(steps):
        expect(backend, backend.lib.plamo_cuda_forward_greedy(backend.ctx, hm.ptr, out[-1], ctypes.byref(t)))
        out.append(int(t.value))
    return out


@pytest.mark.parametrize("copy_kv", [False, True])
def test_restore_then_suffix_prefill_equals_full_prefill(pkg, copy_kv):
    """A 5-id template is declined (layer 0 is a 3-row sliding window, so its
    count is not 5); a 3-id template is cached and prompts of 12 ids share it.
    Restoring and prefilling the 9 suffix ids gives the same logits, KV and
    greedy tokens as prefilling all 12, also after an unrelated request
    dirtied the caches, with sliding-window eviction during the suffix."""
    b = pkg.Backend(device=0, max_context=4200, max_prefill=4096, copy_kv_to_host=copy_kv)
    try:
        hm, _ = decode_fixture_pair(128, 257, 128, 40, vocab=97)
        b.preload_model(hm)
        b.prepare(hm)
        lib = b.lib
        rng = np.random.default_rng(7)
        template = u32(rng.integers(2, 97, size=5))
        prompt = u32(np.concatenate([template, rng.integers(2, 97, size=7)]))
        other = u32(rng.integers(2, 97, size=9))
        # Capture after a fresh prefill of exactly the template.
        lib.plamo_cuda_reset_request(b.ctx, hm.ptr)
        prefill(b, hm, template)
        snap = capture(b, hm, template, len(template))
        assert not snap
        template = template[:3]
        prompt = u32(np.concatenate([template, prompt[3:]]))
        lib.plamo_cuda_reset_request(b.ctx, hm.ptr)
        prefill(b, hm, template)
        snap = capture(b, hm, template, len(template))
        assert snap, b.info().note

        lib.plamo_cuda_reset_request(b.ctx, hm.ptr)
        first = prefill(b, hm, prompt)
        want_logits = hm.logits_array()
        want_tokens = greedy_tail(b, hm, first, 6)
        expect(b, lib.plamo_cuda_sync_host(b.ctx, hm.ptr))
        want_kv = [hm.kv_arrays(i) for i in range(2)]

        for dirty in (False, True):
            lib.plamo_cuda_reset_request(b.ctx, hm.ptr)
            if dirty:
                prefill(b, hm, other)
                greedy_tail(b, hm, 3, 2)
            assert restore(b, snap, hm, prompt, len(prompt)) == len(template)
            first = prefill(b, hm, prompt[len(template):])
            got_logits = hm.logits_array()
            assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)), \
                f"max |d| {np.max(np.abs(got_logits - want_logits))}"
            assert greedy_tail(b, hm, first, 6) == want_tokens
            expect(b, lib.plamo_cuda_sync_host(b.ctx, hm.ptr))
            for i in range(2):
                for got, want in zip(hm.kv_arrays(i), want_kv[i]):
                    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"layer {i}"
        lib.plamo_cuda_prompt_cache_free(snap)
        b.release(hm)
    finally:
        b.close()
