"""Decode / prefill / verification parity on the two-layer fixture of
reference tests/metal_decode.c (run(), prefills(), verification()).

The CUDA model `a` and the oracle model `b` share one weight blob. The
backend keeps the host K/V arrays current (copy_kv_to_host), so every
comparison covers state, logits, unrotated K, V, rotated K, counts and
rotation bookkeeping with the reference's acceptance rule.
"""
import numpy as np
import pytest

from conftest import assert_close, expect, load_oracle, load_package
from fixtures import compare_models, decode_fixture_pair, oracle_forward, oracle_prefill

pytestmark = pytest.mark.gpu

PREFILL_COUNTS = [1, 2, 3, 4, 7, 8, 9, 17, 31, 32, 33, 116, 128, 129, 255, 256, 257, 443, 511,
                  512, 513, 4096]
SHAPES = [(7, 11, 6, 4100), (128, 257, 128, 19), (16, 16384, 6, 264), (128, 256, 128, 520)]


@pytest.fixture(scope="module")
def kv_backend():
    pkg = load_package()
    b = pkg.Backend(device=0, max_context=4200, max_prefill=4096, copy_kv_to_host=True)
    yield b
    b.close()


def reset(*models):
    for m in models:
        m.reset()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "h%d-n%d-d%d-c%d" % s)
def test_fixture_decode_prefill_verify(kv_backend, shape):
    h, n, dim, capacity = shape
    a, b = decode_fixture_pair(h, n, dim, capacity)
    try:
        run_fixture(kv_backend, a, b, h, capacity)
    finally:
        kv_backend.release(a)


def run_fixture(kv_backend, a, b, h, capacity):
    lib, ctx = kv_backend.lib, kv_backend.ctx
    # Not prepared yet: declined without touching anything.
    expect(kv_backend, lib.plamo_cuda_forward(ctx, a.ptr, 2), 0)
    ids = np.array([2, 5, 9], dtype=np.uint32)
    untouched = np.zeros((3, h), dtype=np.float32)
    expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, ids.ctypes.data, 3, untouched.ctypes.data), 0)
    compare_models(a, b)
    kv_backend.preload_model(a)
    kv_backend.prepare(a)
    # An id outside the vocabulary fails (-1) before any state changes.
    bad = np.array([2, 5, 17], dtype=np.uint32)
    expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, bad.ctypes.data, 3, untouched.ctypes.data), -1)
    compare_models(a, b)
    assert np.all(untouched == 0)

    # --- prefills (reference tests/metal_decode.c:232-296) ---------------
    for prefix in (0, 2, 6):
        for count in PREFILL_COUNTS:
            for final_only in (0, 1):
                if count + prefix >= capacity:
                    continue
                if count == 4096 and prefix != 2:
                    continue
                if h * count > 600000 and final_only:  # keep the oracle's share of runtime bounded
                    continue
                reset(a, b)
                for j in range(prefix):
                    assert oracle_forward(a, j % 17) == 1  # CPU rows the GPU must pick up
                    assert oracle_forward(b, j % 17) == 1
                ids = np.array([(j * 7 + 3) % 17 for j in range(count)], dtype=np.uint32)
                actual = np.zeros((count, h), dtype=np.float32)
                ptr = 0 if final_only else actual.ctypes.data
                expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, ids.ctypes.data, count, ptr), 1)
                ok, expected = oracle_prefill(b, ids)
                assert ok == 1
                if not final_only:
                    assert_close(actual, expected[:count], "all prompt states")
                compare_models(a, b)
                expect(kv_backend, lib.plamo_cuda_forward(ctx, a.ptr, 7), 1)
                assert oracle_forward(b, 7) == 1
                compare_models(a, b)

    # --- verification (reference tests/metal_decode.c:298-364) ------------
    prefix = np.array([2, 5], dtype=np.uint32)
    cand = np.array([(i * 7 + 3) % 17 for i in range(16)], dtype=np.uint32)
    for count in (1, 2, 3, 4, 6, 8, 12, 16):
        reset(a, b)
        assert oracle_prefill(b, prefix)[0] == 1
        gold_states, gold_logits, gold_next = [], [], []
        for i in range(count):
            assert oracle_forward(b, int(cand[i])) == 1
            gold_states.append(b.state_array())
            gold_logits.append(b.logits_array())
            gold_next.append(int(load_oracle().plamo_argmax(b.model.logits, b.profile.vocab)))
        expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, prefix.ctypes.data, 2, 0), 1)
        before = (a.state_array(), a.logits_array(), [c.count for c in a.caches])
        nxt = np.zeros(16, dtype=np.uint32)
        expect(kv_backend, lib.plamo_cuda_verify(ctx, a.ptr, cand.ctypes.data, count, nxt.ctypes.data), 1)
        assert np.array_equal(a.state_array(), before[0])
        assert [c.count for c in a.caches] == before[2]
        assert lib.plamo_cuda_commit(ctx, a.ptr, 1) == 0  # out of order
        for i in range(count):
            assert nxt[i] == gold_next[i]
            expect(kv_backend, lib.plamo_cuda_commit(ctx, a.ptr, i), 1)
            assert_close(a.state_array(), gold_states[i], "verified state")
            assert_close(a.logits_array(), gold_logits[i], "verified logits")
        compare_models(a, b)
        expect(kv_backend, lib.plamo_cuda_commit(ctx, a.ptr, count), 0)
        if count >= 4:  # rejected suffix, then ordinary decode recovers
            reset(a, b)
            assert oracle_prefill(b, prefix)[0] == 1
            for i in range(3):
                assert oracle_forward(b, int(cand[i])) == 1
            assert oracle_forward(b, 12) == 1
            expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, prefix.ctypes.data, 2, 0), 1)
            expect(kv_backend, lib.plamo_cuda_verify(ctx, a.ptr, cand.ctypes.data, count, nxt.ctypes.data), 1)
            for i in range(3):
                expect(kv_backend, lib.plamo_cuda_commit(ctx, a.ptr, i), 1)
            expect(kv_backend, lib.plamo_cuda_forward(ctx, a.ptr, 12), 1)
            expect(kv_backend, lib.plamo_cuda_commit(ctx, a.ptr, 3), 0)
            compare_models(a, b)

    # --- decode steps (reference tests/metal_decode.c:450-495) -------------
    reset(a, b)
    for step in range(min(capacity, 140)):
        if step == 9:
            # A prompt in the middle of decoding, then a fresh request.
            ids = np.array([2, 5, 9], dtype=np.uint32)
            got = np.zeros((3, h), dtype=np.float32)
            expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, ids.ctypes.data, 3, got.ctypes.data), 1)
            ok, want = oracle_prefill(b, ids)
            assert ok == 1
            assert_close(got, want[:3], "prefill")
            compare_models(a, b)
            for m in (a, b):
                for i, c in enumerate(m.caches):
                    c.count = 0
                    m.rotation(i).processed_count = 0
        if step == 17:
            for m in (a, b):
                for i in range(2):
                    m.rotation(i).processed_count = 0
        token = (step * 7 + 2) % 17
        assert oracle_forward(b, token) == 1
        expect(kv_backend, lib.plamo_cuda_forward(ctx, a.ptr, token), 1)
        compare_models(a, b)
    count = a.caches[1].count
    assert lib.plamo_cuda_forward(ctx, a.ptr, 17) == 0 and a.caches[1].count == count
    compare_models(a, b)
    launches = kv_backend.info().graph_launches
    a.caches[1].count = b.caches[1].count = capacity
    assert lib.plamo_cuda_forward(ctx, a.ptr, 2) == 0  # full global cache: declined
    assert a.caches[1].count == capacity
    assert kv_backend.info().graph_launches == launches


def test_empty_and_oversized_requests_are_declined(kv_backend):
    """An empty prompt is declined (reference src/prefill.s:9: count 0 returns 0), as are
    verification blocks of 0 or more than PLAMO_CUDA_VERIFY_MAX rows and prompts longer
    than the configured maximum: 0, with the model's state and caches unchanged."""
    a, _ = decode_fixture_pair(128, 257, 128, 40)
    try:
        kv_backend.preload_model(a)
        kv_backend.prepare(a)
        lib, ctx = kv_backend.lib, kv_backend.ctx
        ids = np.array([(j * 7 + 3) % 17 for j in range(4097)], dtype=np.uint32)
        expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, ids.ctypes.data, 0, 0), 0)
        assert [c.count for c in a.caches] == [0, 0]
        expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, ids.ctypes.data, 3, 0), 1)
        state, logits = a.state_array().copy(), a.logits_array().copy()
        counts = [c.count for c in a.caches]
        limit = load_package()._abi.VERIFY_MAX
        nxt = np.zeros(limit + 1, dtype=np.uint32)
        for n in (0, limit + 1):
            expect(kv_backend, lib.plamo_cuda_verify(ctx, a.ptr, ids.ctypes.data, n, nxt.ctypes.data), 0)
        expect(kv_backend, lib.plamo_cuda_prefill(ctx, a.ptr, ids.ctypes.data, 4097, 0), 0)
        assert np.array_equal(a.state_array(), state)
        assert np.array_equal(a.logits_array(), logits)
        assert [c.count for c in a.caches] == counts
    finally:
        kv_backend.release(a)
