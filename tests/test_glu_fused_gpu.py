"""The prompt MLP's gate/up projection fused with SwiGLU.

With 192-row token-major tcgen05 tiles the backend pairs 96 gate rows with
the same 96 up rows in one tile (two tensor maps over the halves of the
[2I][H] weight) and its epilogue writes the BF16 terms of SwiGLU(gate, up)
for the down projection (csrc/gemm_tc.cuh, projection_glu in
csrc/backend.cu): no [T][2I] buffer, no SwiGLU launch. It computes the same
values in the same order as the unfused path (projection, swiglu_rows, the
split into terms), so prefills with and without it (PLAMO_CUDA_TC_GLU=0)
must agree bit for bit: prompt states, every KV row, the logits. The cases
force the 192-row tiles on small models and cover an intermediate size that
is not a multiple of 96 (a partial last pair), ragged token tiles, a hidden
size with a K tail, and a second prompt chunk.
"""
import numpy as np
import pytest

from conftest import expect

pytestmark = pytest.mark.gpu


def run(pkg, monkeypatch, prof, chunks, fused):
    monkeypatch.setenv("PLAMO_CUDA_TC_TOKM", "1")
    monkeypatch.setenv("PLAMO_CUDA_TC_TOKN", "192")
    monkeypatch.setenv("PLAMO_CUDA_TC_GLU", "1" if fused else "0")
    b = pkg.Backend(device=0, max_context=1024, max_prefill=512)
    try:
        hm = pkg.HostModel(prof, weights="synthetic")
        b.preload_synthetic(hm, 33)
        b.prepare(hm)
        rng = np.random.default_rng(9)
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


@pytest.mark.parametrize("hidden,inter,chunks", [
    (512, 1000, (150, 100)),   # 11 pairs, the last with 40 rows; 2 token tiles, then a continuation
    (520, 2048, (300,)),       # hidden with a K tail (8 full K blocks + 8 columns); 22 pairs, the last 32 rows
    (256, 96, (65,)),          # a single pair; the smallest prompt that takes token-major tiles
])
def test_fused_gate_up_swiglu_matches_unfused(pkg, monkeypatch, hidden, inter, chunks):
    prof = pkg.Profile("glu", hidden, 2, 4, 2, 128, inter, vocab=500, window=64, pattern=2, max_position=1024)
    want = run(pkg, monkeypatch, prof, chunks, fused=False)
    got = run(pkg, monkeypatch, prof, chunks, fused=True)
    for c, (a, b) in enumerate(zip(got[0], want[0])):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), \
            f"chunk {c} states: max |d| {np.max(np.abs(a - b))}"
    for layer, (ka, kb) in enumerate(zip(got[1], want[1])):
        for name, a, b in zip(("K", "V", "rotated K"), ka, kb):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"layer {layer} {name}"
    assert np.array_equal(got[2].view(np.uint32), want[2].view(np.uint32))
