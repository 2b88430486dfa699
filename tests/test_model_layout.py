"""The C model descriptor builder (include/plamo_layout.h), host only.

Checked against what the reference's own generators produce
(tests/golden/layout.json, written from tools/weight_schema.py,
tools/model_layout.py and tools/rope_constants.py): the weight schema, each
layer's cache capacity, window flag, frequency table and concentration, and
the record wiring of tools/model_layout.py. Then a checkpoint bound through
the builder's schema must drive the oracle to the same bits as the Python
descriptor tree over the same weights.
"""
import ctypes
import json
import os

import numpy as np
import pytest

from conftest import ROOT, load_oracle, load_package

with open(os.path.join(ROOT, "tests", "golden", "layout.json")) as f:
    GOLDEN = json.load(f)


class Layout:
    def __init__(self, cfg, full_capacity):
        pkg = load_package()
        self.lib = pkg.load()
        err = ctypes.create_string_buffer(256)
        self.handle = self.lib.plamo_model_layout_create(ctypes.byref(cfg), full_capacity, err, 256)
        assert self.handle, err.value
        self.model = self.lib.plamo_model_layout_model(self.handle).contents

    def schema(self):
        out, s = [], self.lib.plamo_model_layout_schema(self.handle)
        i = 0
        while s[i].name:
            out.append((s[i].name.decode(), [s[i].shape[d] for d in range(s[i].rank)], s[i].slot))
            i += 1
        return out

    def layer(self, i):
        return self.model.layers[i].contents

    def close(self):
        self.lib.plamo_model_layout_destroy(self.handle)


def profile_config(name):
    pkg = load_package()
    cfg = pkg._abi.ModelConfig()
    assert pkg.load().plamo_model_config_profile(name.encode(), ctypes.byref(cfg)) == 1
    return cfg


def f32_array(address, n):
    return np.ctypeslib.as_array(ctypes.cast(address, ctypes.POINTER(ctypes.c_float)), shape=(n,)).copy()


@pytest.mark.parametrize("name", sorted(GOLDEN))
def test_profile_config_matches_reference(name):
    cfg, c = profile_config(name), GOLDEN[name]["config"]
    assert (cfg.hidden, cfg.layers, cfg.query_heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab,
            cfg.window, cfg.pattern, cfg.max_position, bool(cfg.tied)) == (
        c["hidden_size"], c["num_hidden_layers"], c["num_attention_heads"], c["num_key_value_heads"],
        c["head_dim"], c["intermediate_size"], c["vocab_size"], c["window_size"], c["sliding_window_pattern"],
        c["max_position_embeddings"], c["tie_word_embeddings"])


@pytest.mark.parametrize("name", sorted(GOLDEN))
def test_layout_matches_reference_generators(name):
    g = GOLDEN[name]
    cfg = profile_config(name)
    lay = Layout(cfg, 1024)
    try:
        assert [[n, s] for n, s, _ in lay.schema()] == g["schema"]
        m = lay.model
        assert (m.vocab, m.hidden, m.count) == (cfg.vocab, cfg.hidden, cfg.layers)
        local = np.array(g["rope_local"], dtype=np.float32)
        glob = np.array(g["rope_global"], dtype=np.float32)
        half = cfg.head_dim // 2
        scales = f32_array(m.scales, cfg.layers)
        kvw = cfg.kv_heads * cfg.head_dim
        for i, want in enumerate(g["layers"]):
            L = lay.layer(i)
            mix = L.mixer.contents
            kc, rot, q, a = mix.cache.contents, mix.rotation.contents, mix.qkv.contents, mix.gqa.contents
            assert bool(kc.sliding) == want["sliding"], i
            assert kc.capacity == (want["capacity"] if want["sliding"] else 1024), i
            assert (kc.count, kc.width) == (0, kvw)
            table = glob if want["table"] == "global" else local
            assert np.array_equal(f32_array(rot.freq, half).view(np.uint32), table.view(np.uint32)), i
            assert scales[i] == np.float32(want["scale"]), i
            # wiring of reference tools/model_layout.py:71-138
            assert L.state == m.state and L.mlp.contents.state == m.state
            assert L.normalized == m.normalized == q.input == L.mlp.contents.normalized
            assert L.branch == mix.out == L.mlp.contents.branch
            assert a.q == q.out and a.k == rot.out and a.v == kc.v
            assert (q.hidden, q.qh, q.kh, q.dim) == (cfg.hidden, cfg.query_heads, cfg.kv_heads, cfg.head_dim)
            assert (rot.heads, rot.dim, rot.processed_count, rot.scale_bits) == (cfg.kv_heads, cfg.head_dim, 0, 0)
            assert L.mlp.contents.intermediate == cfg.intermediate
    finally:
        lay.close()


def test_full_capacity_defaults_to_max_position():
    cfg = profile_config("0.8b")
    lay = Layout(cfg, 0)
    try:
        caps = {bool(lay.layer(i).mixer.contents.cache.contents.sliding):
                lay.layer(i).mixer.contents.cache.contents.capacity for i in range(cfg.layers)}
        assert caps == {True: cfg.window + 1, False: cfg.max_position}
    finally:
        lay.close()


def test_invalid_configurations_are_refused():
    pkg = load_package()
    lib = pkg.load()
    err = ctypes.create_string_buffer(256)
    for field, value in (("hidden", 0), ("kv_heads", 5), ("head_dim", 127), ("beta_slow", 32.0),
                         ("global_theta", 1.0)):
        cfg = profile_config("2b")
        setattr(cfg, field, value)
        assert not lib.plamo_model_layout_create(ctypes.byref(cfg), 64, err, 256), field
        assert err.value, field
    assert lib.plamo_model_config_profile(b"7b", ctypes.byref(pkg._abi.ModelConfig())) == 0


def test_bound_checkpoint_drives_the_oracle_like_the_python_tree(tmp_path):
    """A small model: weights written to a safetensors file, mapped and bound
    through the C schema; prefill + 3 forward steps on the oracle give the same
    logits and state bits as the Python descriptor tree over the same values."""
    pkg = load_package()
    lib = pkg.load()
    prof = pkg.Profile("lay", 64, 4, 4, 2, 16, 96, vocab=50, window=8, pattern=2, max_position=64)
    cfg = pkg._abi.ModelConfig(hidden=64, layers=4, query_heads=4, kv_heads=2, head_dim=16, intermediate=96,
                               vocab=50, window=8, pattern=2, max_position=64, tied=0, local_theta=10000.0,
                               global_theta=1000000.0, yarn_factor=256.0, yarn_original=4096.0, beta_fast=32.0,
                               beta_slow=1.0)
    rng = np.random.default_rng(12)
    tensors = {}
    for name, shape in pkg.schema(prof):
        x = rng.normal(0.0, 0.05, size=shape).astype(np.float32)
        if "norm" in name:
            x = (x + 1.0).astype(np.float32)
        tensors[name] = (x.view(np.uint32) >> 16).astype(np.uint16)
    path = tmp_path / "w.safetensors"
    pkg.write_safetensors(path, tensors)

    mapping = pkg._abi.Mapping()
    assert lib.plamo_map_file(str(path).encode(), ctypes.byref(mapping)) == 1
    lay = Layout(cfg, 64)
    try:
        assert lay.lib.plamo_model_layout_finish(lay.handle) == 0  # nothing bound yet
        assert lib.plamo_bind_weights(ctypes.byref(mapping), 1, lib.plamo_model_layout_schema(lay.handle)) == 1
        assert lay.lib.plamo_model_layout_finish(lay.handle) == 1
        blob = np.empty(pkg.HostModel(prof).blob_bytes // 2, dtype=np.uint16)
        hm = pkg.HostModel(prof, weights=blob)
        for name, t in tensors.items():
            off = hm.offsets[name] // 2
            blob[off:off + t.size] = t.reshape(-1)
        o = load_oracle()
        ids = np.array([3, 14, 15, 9, 2, 6, 5, 35, 8, 9, 7, 9], dtype=np.uint32)
        c_model = ctypes.addressof(lay.model)
        results = []
        for ptr, state_of, logits_of in ((c_model, lambda: f32_array(lay.model.state, 64),
                                          lambda: f32_array(lay.model.logits, 50)),
                                         (ctypes.addressof(hm.model), hm.state_array, hm.logits_array)):
            states = np.zeros((len(ids), 64), dtype=np.float32)
            assert o.plamo_prefill(ptr, ids.ctypes.data, len(ids), states.ctypes.data) == 1
            run = [states.copy(), logits_of()]
            for t in (4, 11, 2):
                assert o.plamo_forward(ptr, t) == 1
                run += [state_of(), logits_of()]
            results.append(run)
        for a, b in zip(*results):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert np.all(np.isfinite(results[0][-1]))
    finally:
        lay.close()
        lib.plamo_unmap_file(ctypes.byref(mapping))


@pytest.mark.gpu
def test_c_built_model_decodes_like_the_python_tree_on_the_gpu(tmp_path, backend):
    """The CUDA backend takes a C-built descriptor tree bound to a mapped
    checkpoint: the same greedy tokens as the Python tree over the same bytes."""
    import synthetic
    pkg = load_package()
    lib = backend.lib
    prof = pkg.Profile("lay-gpu", 256, 2, 4, 2, 64, 512, vocab=500, window=8, pattern=2, max_position=256)
    cfg = pkg._abi.ModelConfig(hidden=256, layers=2, query_heads=4, kv_heads=2, head_dim=64, intermediate=512,
                               vocab=500, window=8, pattern=2, max_position=256, tied=0, local_theta=10000.0,
                               global_theta=1000000.0, yarn_factor=256.0, yarn_original=4096.0, beta_fast=32.0,
                               beta_slow=1.0)
    blob_model = pkg.HostModel(prof)
    synthetic.fill_model(blob_model, 5)
    path = tmp_path / "model.safetensors"
    pkg.write_safetensors(path, {name: blob_model.tensor(name) for name, _ in pkg.schema(prof)})
    mapping = pkg._abi.Mapping()
    assert lib.plamo_map_file(str(path).encode(), ctypes.byref(mapping)) == 1
    lay = Layout(cfg, 256)
    ids = np.arange(3, 15, dtype=np.uint32)
    outs = []
    try:
        assert lib.plamo_bind_weights(ctypes.byref(mapping), 1, lib.plamo_model_layout_schema(lay.handle)) == 1
        assert lib.plamo_model_layout_finish(lay.handle) == 1
        assert lib.plamo_cuda_preload(backend.ctx, mapping.base, mapping.bytes) == 1
        c_ptr = ctypes.pointer(lay.model)
        for ptr, release in ((c_ptr, lambda: lib.plamo_cuda_release_weights(backend.ctx, mapping.base,
                                                                             mapping.bytes)),
                             (blob_model.ptr, lambda: backend.release(blob_model))):
            if ptr is blob_model.ptr:
                backend.preload_model(blob_model)
            assert lib.plamo_cuda_prepare_model(backend.ctx, ptr) == 1, backend.info().note
            out = np.zeros(16, dtype=np.uint32)
            timing = pkg._abi.CudaTiming()
            n = lib.plamo_cuda_generate(backend.ctx, ptr, ids.ctypes.data, len(ids), 16, out.ctypes.data,
                                        pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
            assert n > 0, backend.info().note
            outs.append(list(out[:n]))
            lib.plamo_cuda_release_model(backend.ctx, ptr)
            release()
    finally:
        lay.close()
        lib.plamo_unmap_file(ctypes.byref(mapping))
    assert outs[0] == outs[1]
