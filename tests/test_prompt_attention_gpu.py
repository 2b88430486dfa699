"""Blocked prompt attention against the per-token prompt attention kernel.

From 16 prompt tokens on, the backend sends queries whose window starts at row
0 to a kernel that serves 64 query rows per CTA from each staged key tile; the
others (a sliding layer whose window has filled) stay on the per-token kernel.
Both must give the same bits, at 64 and at 32 query rows per CTA: the blocked
kernel performs the same operations in the same order, so a prefill with it
disabled (PLAMO_CUDA_PROMPT_ATTN=0) must reproduce every prompt state and
every KV row exactly. The cases cover
the grouped-query ratios of the profiles (G = 2, 6, 8, 16), a prompt longer
than a sliding window (split between the kernels inside one launch pair), and
a second prompt chunk that continues from cached rows.
"""
import ctypes

import numpy as np
import pytest

from conftest import expect

pytestmark = pytest.mark.gpu


def run(pkg, monkeypatch, prof, chunks, blocked, rows=None):
    if blocked:
        monkeypatch.delenv("PLAMO_CUDA_PROMPT_ATTN", raising=False)
    else:
        monkeypatch.setenv("PLAMO_CUDA_PROMPT_ATTN", "0")
    if rows:
        monkeypatch.setenv("PLAMO_CUDA_PROMPT_ROWS", str(rows))
    else:
        monkeypatch.delenv("PLAMO_CUDA_PROMPT_ROWS", raising=False)
    b = pkg.Backend(device=0, max_context=1024, max_prefill=512)
    try:
        hm = pkg.HostModel(prof, weights="synthetic")
        b.preload_synthetic(hm, 21)
        b.prepare(hm)
        rng = np.random.default_rng(5)
        states = []
        for n in chunks:
            ids = np.ascontiguousarray(rng.integers(2, prof.vocab, size=n), dtype=np.uint32)
            out = np.zeros((n, prof.hidden), dtype=np.float32)
            expect(b, b.lib.plamo_cuda_prefill(b.ctx, hm.ptr, ids.ctypes.data, n, out.ctypes.data))
            states.append(out)
        expect(b, b.lib.plamo_cuda_sync_host(b.ctx, hm.ptr))
        kv = [hm.kv_arrays(i) for i in range(prof.layers)]
        logits = hm.logits_array()
        b.release(hm)
        return states, kv, logits
    finally:
        b.close()


@pytest.mark.parametrize("qh,kh,window,chunks", [
    (8, 1, 40, (100,)),       # G 8 (8B ratio): sliding layer split 40 blocked / 60 per token
    (24, 4, 2048, (81,)),     # G 6 (2B ratio), 81 tokens: 60 rows per CTA, ragged last block
    (16, 1, 64, (30, 50)),    # G 16: second chunk continues at row 30, window fills at 64
    (4, 2, 16, (20, 17)),     # G 2: the second chunk's sliding queries all per token
])
@pytest.mark.parametrize("rows,bufs", [(64, 2), (32, 1), (32, 2)])
def test_blocked_prompt_attention_matches_per_token_kernel(pkg, monkeypatch, qh, kh, window, chunks, rows, bufs):
    """Both block heights (64 query rows per CTA, and 32 for short prompts),
    the 32-row kernel with one and with two key/value tile buffers."""
    monkeypatch.setenv("PLAMO_CUDA_PROMPT_BUFS", str(bufs))
    prof = pkg.Profile("attn", 512, 2, qh, kh, 128, 256, vocab=500, window=window, pattern=2,
                       max_position=1024)
    want = run(pkg, monkeypatch, prof, chunks, blocked=False)
    got = run(pkg, monkeypatch, prof, chunks, blocked=True, rows=rows)
    for c, (a, b) in enumerate(zip(got[0], want[0])):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), \
            f"chunk {c} states: max |d| {np.max(np.abs(a - b))}"
    for layer, (ka, kb) in enumerate(zip(got[1], want[1])):
        for name, a, b in zip(("K", "V", "rotated K"), ka, kb):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"layer {layer} {name}"
    assert np.array_equal(got[2].view(np.uint32), want[2].view(np.uint32))
