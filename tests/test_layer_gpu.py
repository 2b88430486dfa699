"""Config 2: one decoder layer, one decode step, hidden 2048.

RMSNorm eps 1e-6 with weights 1 + N(0, 0.02); Q 16 x 128, K/V 4 x 128; RoPE
theta 1e4 (concentration 1); full attention over 511 cached rows of FP32
N(0, 1) keys and values; SwiGLU intermediate 8192; BF16 projections from
N(0, 0.02); input hidden vector FP32 N(0, 1). The CUDA layer
(plamo_cuda_layer) is compared with the oracle's plamo_layer (reference
src/layer.s:8-48) under the reference's GPU acceptance rule.
"""
import ctypes

import numpy as np
import pytest

import synthetic
from conftest import assert_close, load_oracle, load_package

pytestmark = pytest.mark.gpu


def config2_pair(pkg, cached=511, seed=0):
    prof = pkg.Profile("config2", 2048, 1, 16, 4, 128, 8192, vocab=16, window=2048, pattern=1,
                       max_position=1024)
    freq = pkg.rope_frequencies(1e4, 64)
    specs = [pkg.LayerSpec(False, 1024, freq, 1.0)]
    a = pkg.HostModel(prof, specs)
    for k, (_, count, name) in enumerate(a.tensor_ranges()):
        off = a.offsets[name] // 2
        mean, std = (1.0, 0.02) if name.endswith("norm.weight") else (0.0, 0.02)
        a.blob[off:off + count] = synthetic.bf16(seed * 7919 + k, count, mean, std)
    b = pkg.HostModel(prof, specs, weights=a.blob)
    rng = np.random.default_rng(seed)
    kvw = 4 * 128
    keys = rng.normal(0, 1, size=cached * kvw).astype(np.float32)
    values = rng.normal(0, 1, size=cached * kvw).astype(np.float32)
    for m in (a, b):
        c = m.caches[0]
        m.view(c.k, cached * kvw)[:] = keys
        m.view(c.v, cached * kvw)[:] = values
        c.count = cached
    state = rng.normal(0, 1, size=2048).astype(np.float32)
    return a, b, state


def oracle_layer(hm, state):
    o = load_oracle()
    o.plamo_layer.restype = ctypes.c_int
    o.plamo_layer.argtypes = [ctypes.c_void_p, ctypes.c_float]
    st = hm.view(hm.model.state, hm.profile.hidden)
    st[:] = state
    layer = hm.layers[0]
    layer.state = hm.model.state
    assert o.plamo_layer(ctypes.addressof(layer), hm.scales[0]) == 1
    return st.copy()


def test_config2_single_layer_decode_step(backend):
    pkg = load_package()
    a, b, state = config2_pair(pkg)
    backend.preload_model(a)
    backend.prepare(a)
    got = state.copy()
    assert backend.lib.plamo_cuda_layer(backend.ctx, a.ptr, 0, got.ctypes.data) == 1
    want = oracle_layer(b, state)
    assert_close(got, want, "layer output")
    assert a.caches[0].count == b.caches[0].count == 512
    assert backend.lib.plamo_cuda_sync_host(backend.ctx, a.ptr) == 1
    ka, va, ra = a.kv_arrays(0)
    kb, vb, rb = b.kv_arrays(0)
    assert_close(ka, kb, "K")
    assert_close(va, vb, "V")
    assert_close(ra, rb, "rotated K")
    # the cached rows came back bit-exact (only row 511 is new)
    assert np.array_equal(ka[:511 * 512], kb[:511 * 512])


def test_config2_repeated_steps_replay_the_recorded_layer(backend):
    """plamo_cuda_layer records each layer's launches once and replays them:
    the cache position and the KV page of every later step are read on the
    device, so consecutive steps (rows 511..515, new input states) must each
    match the oracle, which appends the same rows."""
    pkg = load_package()
    a, b, _ = config2_pair(pkg, seed=1)
    backend.preload_model(a)
    backend.prepare(a)
    rng = np.random.default_rng(77)
    for step in range(5):
        state = rng.normal(0, 1, size=2048).astype(np.float32)
        got = state.copy()
        assert backend.lib.plamo_cuda_layer(backend.ctx, a.ptr, 0, got.ctypes.data) == 1
        want = oracle_layer(b, state)
        assert_close(got, want, f"layer output, step {step}")
        assert a.caches[0].count == b.caches[0].count == 512 + step
    assert backend.info().graph_launches >= 5
    assert backend.lib.plamo_cuda_sync_host(backend.ctx, a.ptr) == 1
    ka, va, _ = a.kv_arrays(0)
    kb, vb, _ = b.kv_arrays(0)
    assert_close(ka, kb, "K")
    assert_close(va, vb, "V")
