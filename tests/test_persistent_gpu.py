"""The one-launch decode step (csrc/persist.cuh) against the graph of
per-projection kernels and against the oracle.

Both paths implement the same step (reference src/forward.s:9-84); the
projections form their dot products identically, attention splits its keys
differently (all CTAs of the persistent grid vs 8-CTA clusters), so logits
agree within the reference's GPU acceptance rule and greedy tokens are
identical. The shapes are chosen so the persistent path applies (head dim
128, columns in whole 512-column slots): a sliding layer with a 16-row window
(evictions during decode) and a full-attention layer.
"""
import ctypes
import os

import numpy as np
import pytest

from conftest import assert_close, expect, load_oracle, load_package
from fixtures import oracle_forward, oracle_prefill

pytestmark = pytest.mark.gpu


def mini_profile(pkg):
    return pkg.Profile("mini", 1024, 4, 8, 2, 128, 1536, vocab=3000, window=16, pattern=2, max_position=512)


def backend_with(persistent):
    pkg = load_package()
    old = os.environ.get("PLAMO_CUDA_PERSISTENT")
    os.environ["PLAMO_CUDA_PERSISTENT"] = "1" if persistent else "0"
    try:
        return pkg.Backend(device=0, max_context=1024, max_prefill=256)
    finally:
        if old is None:
            del os.environ["PLAMO_CUDA_PERSISTENT"]
        else:
            os.environ["PLAMO_CUDA_PERSISTENT"] = old


def decode(be, hm, ids, steps):
    """Prefill, then `steps` forwards of the greedy token; logits of each."""
    lib = be.lib
    expect(be, lib.plamo_cuda_prefill(be.ctx, hm.ptr, ids.ctypes.data, len(ids), None))
    token = int(np.argmax(hm.logits_array()))
    out, logits = [], []
    for _ in range(steps):
        launches = lib.plamo_cuda_kernel_launches(be.ctx)
        expect(be, lib.plamo_cuda_forward(be.ctx, hm.ptr, token))
        out.append(token)
        logits.append(hm.logits_array())
        token = int(np.argmax(logits[-1]))
        be.last_step_launches = lib.plamo_cuda_kernel_launches(be.ctx) - launches
    return out, logits


def test_persistent_step_matches_graph_and_oracle():
    pkg = load_package()
    prof = mini_profile(pkg)
    ids = np.random.default_rng(8).integers(3, prof.vocab, size=21).astype(np.uint32)
    results = {}
    for persistent in (True, False):
        be = backend_with(persistent)
        try:
            hm = pkg.HostModel(prof, weights="synthetic")
            be.preload_synthetic(hm, seed=17)
            be.prepare(hm)
            path = be.lib.plamo_cuda_decode_path(be.ctx, hm.ptr).decode()
            assert (path == "persistent") == persistent, path
            results[persistent] = decode(be, hm, ids, 40) + (be.last_step_launches,)
            if persistent:
                blob = np.empty(hm.blob_bytes // 2, dtype=np.uint16)
                host = pkg.HostModel(prof, weights=blob)
                for (ka, count, _), (kb, _, _) in zip(hm.tensor_ranges(), host.tensor_ranges()):
                    assert be.lib.plamo_cuda_read_weights(be.ctx, ka, kb, 2 * count) == 1
        finally:
            be.close()
    (tok_p, log_p, launches_p), (tok_g, log_g, launches_g) = results[True], results[False]
    assert launches_p == 1, f"persistent step took {launches_p} launches"
    assert launches_g > 1
    assert tok_p == tok_g
    for i, (a, b) in enumerate(zip(log_p, log_g)):
        assert_close(a, b, f"step {i} logits")
    # The oracle's greedy continuation (no stop ids: every step is compared).
    o = load_oracle()
    ok, _ = oracle_prefill(host, ids)
    assert ok == 1
    want, margins = [], []
    for _ in range(40):
        logits = host.logits_array()
        top = np.partition(logits, -2)[-2:]
        margins.append(float(top[1] - top[0]))
        want.append(int(o.plamo_argmax(host.model.logits, prof.vocab)))
        assert oracle_forward(host, want[-1]) == 1
    assert want == tok_p, f"oracle margins {margins}"


@pytest.mark.parametrize("name", ["0.8b", "2b"])
def test_persistent_profiles_match_graph_tokens(name):
    """The 0.8B (16 query heads over one KV head) and 2B profiles: 24 tokens
    after a 30-id prompt, identical on both paths."""
    pkg = load_package()
    prof = pkg.PROFILES[name]
    ids = np.random.default_rng(3).integers(3, 100000, size=30).astype(np.uint32)
    tokens = {}
    for persistent in (True, False):
        be = backend_with(persistent)
        try:
            hm = pkg.HostModel(prof, weights="synthetic", full_capacity=1024)
            be.preload_synthetic(hm, seed=5)
            be.prepare(hm)
            out = np.zeros(24, dtype=np.uint32)
            timing = pkg._abi.CudaTiming()
            n = be.lib.plamo_cuda_generate(be.ctx, hm.ptr, ids.ctypes.data, len(ids), 24, out.ctypes.data,
                                           pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
            assert n > 0, be.info().note
            tokens[persistent] = out[:n].tolist()
        finally:
            be.close()
    assert tokens[True] == tokens[False]


def test_decode_trace_reports_every_phase():
    """plamo_cuda_decode_trace: one committed persistent step with the device
    timestamps of CTA 0 - kernel start, then every grid barrier in step order
    (non-decreasing), then the first chunk issued for every projection."""
    pkg = load_package()
    prof = mini_profile(pkg)
    be = backend_with(True)
    try:
        hm = pkg.HostModel(prof, weights="synthetic")
        be.preload_synthetic(hm, seed=17)
        be.prepare(hm)
        ids = np.random.default_rng(9).integers(3, prof.vocab, size=5).astype(np.uint32)
        expect(be, be.lib.plamo_cuda_prefill(be.ctx, hm.ptr, ids.ctypes.data, len(ids), None))
        L = prof.layers
        n = 1 + (5 * L + 1) + (4 * L + 1)
        stamps = np.zeros(n, dtype=np.uint64)
        assert be.lib.plamo_cuda_decode_trace(be.ctx, hm.ptr, 7, stamps.ctypes.data, n - 1) == -1
        assert be.lib.plamo_cuda_decode_trace(be.ctx, hm.ptr, 7, stamps.ctypes.data, n) == n
        barriers = stamps[1:1 + 5 * L + 1].astype(np.int64)
        issues = stamps[1 + 5 * L + 1:].astype(np.int64)
        assert np.all(barriers > 0) and np.all(issues > 0)
        assert np.all(np.diff(barriers) >= 0)
        assert barriers[0] >= int(stamps[0]) and np.all(issues >= int(stamps[0]))
        # The step was committed: the next forward continues from it.
        expect(be, be.lib.plamo_cuda_forward(be.ctx, hm.ptr, 11))
    finally:
        be.close()


def test_graph_decode_trace_orders_every_launch():
    """plamo_cuda_decode_trace on the graph path: a traced copy of the step's
    graph stamps every projection and attention launch. Within a launch the
    first entry precedes the last CTA past its wait, which precedes the last
    CTA done; each launch's dependency wait ends after the previous launch's
    last CTA is done (programmatic dependent launch orders them)."""
    pkg = load_package()
    prof = mini_profile(pkg)
    be = backend_with(False)
    try:
        hm = pkg.HostModel(prof, weights="synthetic")
        be.preload_synthetic(hm, seed=17)
        be.prepare(hm)
        ids = np.random.default_rng(9).integers(3, prof.vocab, size=5).astype(np.uint32)
        expect(be, be.lib.plamo_cuda_prefill(be.ctx, hm.ptr, ids.ctypes.data, len(ids), None))
        n = 6 * (5 * prof.layers + 1)
        stamps = np.zeros(n, dtype=np.uint64)
        assert be.lib.plamo_cuda_decode_trace(be.ctx, hm.ptr, 7, stamps.ctypes.data, n - 1) == -1
        assert be.lib.plamo_cuda_decode_trace(be.ctx, hm.ptr, 7, stamps.ctypes.data, n) == n
        t = stamps.reshape(-1, 6).astype(np.int64)
        assert np.all(t > 0)
        assert np.all(t[:, 0] <= t[:, 5]) and np.all(t[:, 5] <= t[:, 1]) and np.all(t[:, 4] <= t[:, 1])
        assert np.all(t[:, 1] <= t[:, 3]) and np.all(t[:, 0] <= t[:, 2]) and np.all(t[:, 2] <= t[:, 3])
        assert np.all(t[1:, 4] >= t[:-1, 3])
        assert be.lib.plamo_cuda_decode_path(be.ctx, hm.ptr).startswith(b"graph")
        expect(be, be.lib.plamo_cuda_forward(be.ctx, hm.ptr, 11))
    finally:
        be.close()
