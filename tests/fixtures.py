"""Model fixtures shared by the GPU parity tests.

`decode_fixture` is the two-layer model of reference tests/metal_decode.c:95-175
(layer 0 sliding with capacity 3, layer 1 global with `capacity`, frequencies
powf(1e-4, j / (dim/2)), concentrations 1 and 1.5545177, vocab 17, 4 query and
2 KV heads, LCG fixture weights) built twice over one weight blob: one copy is
driven through the CUDA backend, the other through the C oracle.
"""
import numpy as np

import synthetic
from conftest import assert_close, load_oracle, load_package


def decode_fixture_pair(h, n, dim, capacity, vocab=17, qh=4, kh=2, seed=93):
    pkg = load_package()
    prof = pkg.Profile("fixture", h, 2, qh, kh, dim, n, vocab=vocab, window=2, pattern=2,
                       max_position=capacity)
    half = dim // 2
    freq = np.array([np.float32(1e-4) ** (np.float32(j) / np.float32(half)) for j in range(half)],
                    dtype=np.float32)
    specs = [pkg.LayerSpec(True, 3, freq, 1.0),
             pkg.LayerSpec(False, capacity, freq, float(np.float32(1.5545177)))]
    a = pkg.HostModel(prof, specs)
    synthetic.lcg_fixture_weights(a, seed)
    b = pkg.HostModel(prof, specs, weights=a.blob)
    return a, b


def compare_models(a, b, kv=True):
    """reference tests/metal_decode.c:217-230: state, logits, and per layer
    count, unrotated K, V and rotated K, processed count and scale bits."""
    assert_close(a.state_array(), b.state_array(), "state")
    assert_close(a.logits_array(), b.logits_array(), "logits")
    if not kv:
        return
    for i in range(a.profile.layers):
        assert a.caches[i].count == b.caches[i].count, f"layer {i} count"
        ka, va, ra = a.kv_arrays(i)
        kb, vb, rb = b.kv_arrays(i)
        assert_close(ka, kb, f"layer {i} unrotated K")
        assert_close(va, vb, f"layer {i} V")
        assert_close(ra, rb, f"layer {i} rotated K")
        assert a.rotation(i).processed_count == b.rotation(i).processed_count
        assert a.rotation(i).scale_bits == b.rotation(i).scale_bits


def oracle_forward(hm, token):
    return load_oracle().plamo_forward(hm.ptr, token)


def oracle_prefill(hm, ids, states=None):
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    if states is None:
        states = np.zeros((max(len(ids), 1), hm.profile.hidden), dtype=np.float32)
    ok = load_oracle().plamo_prefill(hm.ptr, ids.ctypes.data, len(ids), states.ctypes.data)
    return ok, states
