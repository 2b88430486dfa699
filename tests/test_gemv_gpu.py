"""Config 1: the decode projection (BF16 GEMV, FP32 accumulation) against the oracle.

W 4096x4096 BF16 from N(0, 0.02) and x 4096 FP32 from N(0, 1)
(numpy default_rng(0), W drawn first), plus the 14336x4096 variant; parity
within 1e-5 relative L2 of the reference CPU matvec (oracle restatement of
reference src/math.s:86-344). Odd shapes follow reference tests/matmul.c:21-23.
"""
import ctypes

import numpy as np
import pytest

import synthetic
from conftest import load_oracle, rel_l2

pytestmark = pytest.mark.gpu


def config1_inputs(rows, cols, seed=0):
    rng = np.random.default_rng(seed)
    w = synthetic.bf16_round(rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32))
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    return np.ascontiguousarray(w), x


def oracle_matvec(w, x):
    rows, cols = w.shape
    y = np.zeros(max(rows, 1), dtype=np.float32)
    load_oracle().plamo_bf16_matvec(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols)
    return y[:rows]


def gpu_matvec(backend, w, x, offset_elements=0):
    lib, ctx = backend.lib, backend.ctx
    rows, cols = w.shape
    wbytes = (w.size + offset_elements) * 2
    dw = lib.plamo_cuda_device_alloc(ctx, wbytes)
    dx = lib.plamo_cuda_device_alloc(ctx, max(x.nbytes, 4))
    dy = lib.plamo_cuda_device_alloc(ctx, max(rows * 4, 4))
    try:
        assert lib.plamo_cuda_copy_to_device(ctx, dw + 2 * offset_elements, w.ctypes.data, w.nbytes)
        assert lib.plamo_cuda_copy_to_device(ctx, dx, x.ctypes.data, x.nbytes)
        assert lib.plamo_cuda_gemv_device(ctx, dw + 2 * offset_elements, dx, dy, rows, cols) == 1
        y = np.zeros(max(rows, 1), dtype=np.float32)
        assert lib.plamo_cuda_copy_to_host(ctx, y.ctypes.data, dy, rows * 4)
        return y[:rows]
    finally:
        for p in (dw, dx, dy):
            lib.plamo_cuda_device_free(ctx, p)


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096)])
def test_config1_gemv_matches_reference_matvec(backend, rows, cols):
    w, x = config1_inputs(rows, cols)
    y = gpu_matvec(backend, w, x)
    ref = oracle_matvec(w, x)
    assert rel_l2(y, ref) <= 1e-5
    # an FP64 shadow bounds both: the GPU is as close to exact as the CPU order
    exact = synthetic.bf16_to_f32(w).astype(np.float64) @ x.astype(np.float64)
    assert rel_l2(y, exact) <= 1e-5


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (4, 4), (3, 4), (5, 12), (8, 12), (16, 128),
                                       (12, 64), (128, 4096), (64, 16384), (7, 256), (9, 512),
                                       (33, 1536), (17, 3072), (5, 25600), (300, 2048),
                                       # rows ending inside a 512-column slot (tensor-parallel shards)
                                       (40, 3200), (33, 6400), (21, 1000), (64, 9992), (300, 5128)])
def test_gemv_odd_shapes(backend, rows, cols):
    rng = np.random.default_rng(rows * 1000 + cols)
    w = synthetic.bf16_round(rng.normal(0, 0.05, size=(rows, cols)).astype(np.float32))
    x = rng.normal(0, 1, size=cols).astype(np.float32)
    assert rel_l2(gpu_matvec(backend, w, x), oracle_matvec(w, x)) <= 1e-5


def test_gemv_unaligned_weights_use_generic_path(backend):
    w, x = config1_inputs(96, 1024, seed=3)
    y = gpu_matvec(backend, w, x, offset_elements=1)
    assert rel_l2(y, oracle_matvec(w, x)) <= 1e-5


def test_linear_entry_point_strides_and_tails(backend, pkg):
    """plamo_cuda_linear == per-token matvec with input/output strides; rows
    outside [0, rows) of each output token row stay untouched
    (reference tests/matmul.c:20-77 shapes)."""
    lib, ctx = backend.lib, backend.ctx
    alive = []  # preloaded ranges are keyed by host address: keep them mapped
    for r, c, t in [(3, 7, 5), (4, 4, 4), (5, 12, 17), (16, 128, 9), (12, 64, 17), (128, 4096, 7)]:
        rng = np.random.default_rng(r + c + t)
        w = synthetic.bf16_round(rng.normal(0, 0.05, size=(r, c)).astype(np.float32))
        xs, ys = c + 7, r + 9
        x = rng.normal(0, 1, size=t * xs + 1).astype(np.float32)
        y = np.full(t * ys + 1, -123456.0, dtype=np.float32)
        alive.append(w)
        assert lib.plamo_cuda_preload(ctx, w.ctypes.data, w.nbytes) == 1
        mm = pkg._abi.Matmul(w.ctypes.data, x.ctypes.data, y.ctypes.data, r, c, t, xs, ys)
        assert lib.plamo_cuda_linear(ctx, ctypes.byref(mm)) == 1
        for k in range(t):
            ref = oracle_matvec(w, np.ascontiguousarray(x[k * xs:k * xs + c]))
            assert rel_l2(y[k * ys:k * ys + r], ref) <= 1e-5
            assert np.all(y[k * ys + r:(k + 1) * ys] == -123456.0)
    # a weight range that was never preloaded is declined, output untouched
    w = np.ones((2, 2), dtype=np.uint16)
    x = np.ones(4, dtype=np.float32)
    y = np.zeros(4, dtype=np.float32)
    mm = pkg._abi.Matmul(w.ctypes.data, x.ctypes.data, y.ctypes.data, 2, 2, 2, 2, 2)
    assert lib.plamo_cuda_linear(ctx, ctypes.byref(mm)) == 0
    assert np.all(y == 0)


def test_device_synthetic_fill_matches_host_restatement(backend):
    lib, ctx = backend.lib, backend.ctx
    n = 1 << 20
    d = lib.plamo_cuda_device_alloc(ctx, n * 4)
    try:
        for seed, mean, std in [(0, 0.0, 0.02), (12345, 1.0, 0.02), (7, 1.0, 0.0)]:
            assert lib.plamo_cuda_fill_synthetic_bf16(ctx, d, n, seed, mean, std)
            got = np.zeros(n, dtype=np.uint16)
            assert lib.plamo_cuda_copy_to_host(ctx, got.ctypes.data, d, n * 2)
            assert np.array_equal(got, synthetic.bf16(seed, n, mean, std))
            assert lib.plamo_cuda_fill_synthetic_f32(ctx, d, n, seed, mean, std)
            gotf = np.zeros(n, dtype=np.float32)
            assert lib.plamo_cuda_copy_to_host(ctx, gotf.ctypes.data, d, n * 4)
            assert np.array_equal(gotf.view(np.uint32), synthetic.f32(seed, n, mean, std).view(np.uint32))
    finally:
        lib.plamo_cuda_device_free(ctx, d)
