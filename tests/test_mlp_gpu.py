"""plamo_cuda_mlp: the whole MLP block of several states (reference
runtime/metal.h:86-88, the plamo_mlp_kernel hook of runtime/compute.h:12 that
src/model.s:65-75 and src/batch.s:151-162 call) against the oracle's
plamo_mlp_branch (reference src/model.s:8-60): pre-MLP RMSNorm(+1), gate/up
projection, SwiGLU, down projection, post-MLP RMSNorm(+1/5^1.5), residual.

Shapes of BASELINE config 2 (hidden 2048, intermediate 8192), token counts of
reference tests/metal.c:134-160 and its tolerance (|delta| <= 2e-5 * (1 +
|expected|) per element).
"""
import ctypes

import numpy as np
import pytest

import synthetic
from conftest import expect, load_oracle, load_package

pytestmark = pytest.mark.gpu

H, N = 2048, 8192


def mlp_tensors(seed=5):
    rng = np.random.default_rng(seed)
    pre = synthetic.bf16_round((1 + rng.normal(0, 0.02, H)).astype(np.float32))
    post = synthetic.bf16_round((1 + rng.normal(0, 0.02, H)).astype(np.float32))
    gu = synthetic.bf16_round(rng.normal(0, 0.02, (2 * N, H)).astype(np.float32))
    down = synthetic.bf16_round(rng.normal(0, 0.02, (H, N)).astype(np.float32))
    return pre, post, gu, down


def descriptor(pkg, pre, post, gu, down, keep):
    def f32(n):
        a = np.zeros(n, dtype=np.float32)
        keep.append(a)
        return a.ctypes.data
    return pkg._abi.Mlp(state=None, pre=pre.ctypes.data, post=post.ctypes.data, gu=gu.ctypes.data,
                        down=down.ctypes.data, normalized=f32(H), branch=f32(H), scratch=f32(2 * N),
                        hidden=H, intermediate=N)


def oracle_block(pkg, desc, states, tokens):
    o = load_oracle()
    o.plamo_mlp_branch.restype, o.plamo_mlp_branch.argtypes = None, [ctypes.c_void_p]
    out = states.copy()
    for t in range(tokens):
        row = out[t]
        d = pkg._abi.Mlp(**{f: getattr(desc, f) for f, _ in pkg._abi.Mlp._fields_})
        d.state = row.ctypes.data
        o.plamo_mlp_branch(ctypes.byref(d))
    return out


@pytest.mark.parametrize("tokens", [0, 1, 3, 4, 8, 21])
def test_mlp_block_matches_oracle(backend, tokens):
    pkg = load_package()
    keep = []
    pre, post, gu, down = mlp_tensors()
    for t in (pre, post, gu, down):
        expect(backend, backend.lib.plamo_cuda_preload(backend.ctx, t.ctypes.data, t.nbytes))
    desc = descriptor(pkg, pre, post, gu, down, keep)
    rows = max(tokens, 1) + 2
    states = np.random.default_rng(100 + tokens).normal(0, 1, (rows, H)).astype(np.float32)
    want = oracle_block(pkg, desc, states, tokens)
    got = states.copy()
    expect(backend, backend.lib.plamo_cuda_mlp(backend.ctx, ctypes.byref(desc), got.ctypes.data, tokens))
    assert np.all(np.isfinite(got))
    err = np.abs(got.astype(np.float64) - want) - 2e-5 * (1 + np.abs(want.astype(np.float64)))
    assert err.max() <= 0, f"{tokens} tokens: worst excess {err.max():.3g}"
    assert np.array_equal(got[tokens:], states[tokens:]), "rows past the block changed"


def test_mlp_declines_weights_it_does_not_hold(backend):
    """Weights that were never preloaded: declined, states untouched
    (reference tests/metal.c:163-166)."""
    pkg = load_package()
    keep = []
    pre, post, gu, down = mlp_tensors(seed=6)
    desc = descriptor(pkg, pre, post, gu, down, keep)
    states = np.random.default_rng(7).normal(0, 1, (21, H)).astype(np.float32)
    got = states.copy()
    assert backend.lib.plamo_cuda_mlp(backend.ctx, ctypes.byref(desc), got.ctypes.data, 21) == 0
    assert np.array_equal(got, states)
