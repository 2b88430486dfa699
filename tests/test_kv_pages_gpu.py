"""Paged KV cache: every layer's K/V rows live in pages of 64 rows taken from a
page pool that the backend context shares between requests (KvPool in
csrc/backend.cu; kv_key / kv_value in csrc/attention.cuh address a row through
the layer's page table). A sliding ring maps its pages when the model is
prepared; a full-attention layer maps a page when its rows reach it, so a
request holds pages for the rows it has, not for its capacity, and a reset or
release returns them to the pool for the next request.

The model is the two-layer fixture of reference tests/metal_decode.c (a
sliding layer of capacity 3 and a full-attention layer), with the full layer's
capacity far above the rows used. Prefill and decode cross page boundaries and
are compared with the oracle (state, logits, K, V, rotated K).
"""
import numpy as np
import pytest

from conftest import expect, load_package
from fixtures import compare_models, decode_fixture_pair, oracle_forward, oracle_prefill

pytestmark = pytest.mark.gpu

H, N, DIM, CAPACITY = 128, 256, 128, 4096
KVW = 2 * DIM            # two KV heads


@pytest.fixture
def backend():
    pkg = load_package()
    b = pkg.Backend(device=0, max_context=CAPACITY + 16, max_prefill=512, copy_kv_to_host=True)
    yield b
    b.close()


def prepared_pair(backend):
    a, b = decode_fixture_pair(H, N, DIM, CAPACITY)
    backend.preload_model(a)
    backend.prepare(a)
    return a, b


def prefill_both(backend, a, b, ids):
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    expect(backend, backend.lib.plamo_cuda_prefill(backend.ctx, a.ptr, ids.ctypes.data, len(ids), None))
    ok, _ = oracle_prefill(b, ids)
    assert ok == 1


def test_full_layer_maps_pages_as_rows_arrive(backend):
    a, b = prepared_pair(backend)
    try:
        info = backend.info()
        # The sliding ring (3 + 16 + 1 slots) holds one page; the full layer none yet.
        assert info.kv_pages_used == 1
        # Far below what a contiguous ring of the full layer's capacity would take.
        assert info.kv_bytes < 2 * CAPACITY * KVW * 4
        rng = np.random.default_rng(11)
        prefill_both(backend, a, b, rng.integers(0, 17, size=100))
        compare_models(a, b)
        assert backend.info().kv_pages_used == 1 + 2          # rows 0..99: two pages
        for step in range(40):                                # rows 100..139: a third page at row 128
            token = int(rng.integers(0, 17))
            expect(backend, backend.lib.plamo_cuda_forward(backend.ctx, a.ptr, token))
            assert oracle_forward(b, token) == 1
            if step % 9 == 0 or step == 39:
                compare_models(a, b)
        assert backend.info().kv_pages_used == 1 + 3
    finally:
        backend.release(a)
    assert backend.info().kv_pages_used == 0


def test_reset_and_release_return_pages_for_reuse(backend):
    a, b = prepared_pair(backend)
    try:
        rng = np.random.default_rng(12)
        prefill_both(backend, a, b, rng.integers(0, 17, size=200))   # 4 pages in the full layer
        assert backend.info().kv_pages_used == 1 + 4
        allocated = backend.info().kv_pages_allocated
        backend.lib.plamo_cuda_reset_request(backend.ctx, a.ptr)
        b.reset()
        assert backend.info().kv_pages_used == 1
        # A second request of the same length reuses the returned pages.
        prefill_both(backend, a, b, rng.integers(0, 17, size=200))
        compare_models(a, b)
        assert backend.info().kv_pages_used == 1 + 4
        assert backend.info().kv_pages_allocated == allocated
        # Another request prepared beside it takes pages from the same pool.
        c, d = prepared_pair(backend)
        try:
            prefill_both(backend, c, d, rng.integers(0, 17, size=64))    # 1 page
            compare_models(c, d)
            assert backend.info().kv_pages_used == (1 + 4) + (1 + 1)
        finally:
            # The request's model only (releasing its weights drops every prepared model).
            assert backend.lib.plamo_cuda_release_model(backend.ctx, c.ptr) == 1
        assert backend.info().kv_pages_used == 1 + 4
    finally:
        backend.release(a)
    assert backend.info().kv_pages_used == 0
    # With no page mapped, maintenance gives the pool's chunks back.
    assert backend.info().kv_pages_allocated > 0
    backend.lib.plamo_cuda_maintain(backend.ctx)
    assert backend.info().kv_pages_allocated == 0
