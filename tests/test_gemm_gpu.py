"""Prompt projections on the tensor cores (tcgen05, BF16 hi/lo split of the
FP32 activations, FP32 accumulation in TMEM) against the oracle's batched
matvec (reference src/matmul*.s is bitwise the per-token matvec,
tests/matmul.c:20-77), within the 1e-5 relative L2 bound BASELINE sets for
projections. Shapes cover ragged token and row tiles, K tails and the
prefill shapes of the 8B profile."""
import numpy as np
import pytest

import synthetic
from conftest import expect, load_oracle, rel_l2

pytestmark = pytest.mark.gpu


def oracle_rows(w, x):
    o = load_oracle()
    rows, cols = w.shape
    out = np.zeros((x.shape[0], rows), dtype=np.float32)
    for t in range(x.shape[0]):
        xt = np.ascontiguousarray(x[t])
        o.plamo_bf16_matvec(w.ctypes.data, xt.ctypes.data, out[t].ctypes.data, rows, cols)
    return out


def gpu_gemm(backend, w, x):
    lib, ctx = backend.lib, backend.ctx
    T, K = x.shape
    R = w.shape[0]
    dw = lib.plamo_cuda_device_alloc(ctx, w.nbytes)
    dx = lib.plamo_cuda_device_alloc(ctx, x.nbytes)
    dy = lib.plamo_cuda_device_alloc(ctx, T * R * 4)
    try:
        assert lib.plamo_cuda_copy_to_device(ctx, dw, w.ctypes.data, w.nbytes)
        assert lib.plamo_cuda_copy_to_device(ctx, dx, x.ctypes.data, x.nbytes)
        expect(backend, lib.plamo_cuda_gemm_device(ctx, dx, K, dw, dy, R, T, R, K), 1)
        y = np.zeros((T, R), dtype=np.float32)
        assert lib.plamo_cuda_copy_to_host(ctx, y.ctypes.data, dy, y.nbytes)
        return y
    finally:
        for p in (dw, dx, dy):
            lib.plamo_cuda_device_free(ctx, p)


@pytest.mark.parametrize("T,R,K", [(1, 128, 64), (5, 200, 128), (16, 256, 4096), (17, 130, 72), (31, 384, 512),
                                   (64, 1000, 256), (100, 5120, 4096), (129, 512, 1024), (455, 640, 4096),
                                   (455, 4096, 16384),
                                   # split K (few tokens over few row tiles): verify / batched decode shapes
                                   (8, 5120, 4096), (12, 4096, 16384), (3, 1000, 520)])
def test_tc_projection_matches_oracle(backend, T, R, K):
    rng = np.random.default_rng(T * 131 + R * 7 + K)
    w = np.ascontiguousarray(synthetic.bf16_round(rng.normal(0, 0.02, size=(R, K)).astype(np.float32)))
    x = rng.normal(0, 1, size=(T, K)).astype(np.float32)
    got = gpu_gemm(backend, w, x)
    want = oracle_rows(w, x)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, want) <= 1e-5, rel_l2(got, want)


@pytest.mark.parametrize("layout", ["0", "1:192", "1:160", "1:144"])
@pytest.mark.parametrize("T,R,K", [(65, 200, 72), (129, 385, 1024), (455, 5120, 4096), (300, 1000, 520)])
def test_tc_tile_layouts_match_oracle(monkeypatch, layout, T, R, K):
    """Every tile layout of a prompt projection (PLAMO_CUDA_TC_TOKM=0:
    128 weight rows x 128 tokens; =1: 128 tokens x 192, 160 or 144 weight
    rows (PLAMO_CUDA_TC_TOKN), stored through shared memory), with ragged
    token and row tiles and K tails."""
    from conftest import load_package
    tokm, _, tokn = layout.partition(":")
    monkeypatch.setenv("PLAMO_CUDA_TC_TOKM", tokm)
    if tokn:
        monkeypatch.setenv("PLAMO_CUDA_TC_TOKN", tokn)
    else:
        monkeypatch.delenv("PLAMO_CUDA_TC_TOKN", raising=False)
    pkg = load_package()
    b = pkg.Backend(device=0, max_context=64, max_prefill=512)
    try:
        rng = np.random.default_rng(T * 17 + R + K)
        w = np.ascontiguousarray(synthetic.bf16_round(rng.normal(0, 0.02, size=(R, K)).astype(np.float32)))
        x = rng.normal(0, 1, size=(T, K)).astype(np.float32)
        got = gpu_gemm(b, w, x)
        want = oracle_rows(w, x)
        assert np.all(np.isfinite(got))
        assert rel_l2(got, want) <= 1e-5, rel_l2(got, want)
    finally:
        b.close()
