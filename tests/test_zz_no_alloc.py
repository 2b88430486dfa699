"""plamo_cuda_linear_static: the projection entry point that allocates nothing.

Some callers cannot allocate device memory at the point where they need a
projection - for example the reference CPU kernels, which reach a GPU backend
through the plamo_matmul_kernel hook from inside their assembly loops, with no
way to handle an allocation failure, and where a cudaFree would synchronise
the whole device. This entry point stages the host rows in a fixed array
compiled into the library instead. It must give the same results as the
allocating plamo_cuda_linear, call after call (the array keeps the previous
call's contents), and decline requests larger than its array.

This file is collected last on purpose: it must pass in a fresh process and
after every other test.
"""
import ctypes

import numpy as np
import pytest

import synthetic
from conftest import expect, load_oracle, load_package, rel_l2

pytestmark = pytest.mark.gpu


def run_linear(backend, entry, w, x, rows, cols, tokens, xs, ys):
    pkg = load_package()
    y = np.full(tokens * ys + 1, -7.0, dtype=np.float32)
    mm = pkg._abi.Matmul(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols, tokens, xs, ys)
    expect(backend, getattr(backend.lib, entry)(backend.ctx, ctypes.byref(mm)), 1)
    return y


def test_static_linear_matches_allocating_linear_twice(backend):
    rows, cols, tokens = 300, 1024, 5
    xs, ys = cols + 3, rows + 5
    rng = np.random.default_rng(2024)
    w = synthetic.bf16_round(rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32))
    expect(backend, backend.lib.plamo_cuda_preload(backend.ctx, w.ctypes.data, w.nbytes), 1)
    for call in range(2):  # the second call must not see the first call's rows
        x = rng.normal(0, 1, size=tokens * xs + 1).astype(np.float32)
        want = run_linear(backend, "plamo_cuda_linear", w, x, rows, cols, tokens, xs, ys)
        got = run_linear(backend, "plamo_cuda_linear_static", w, x, rows, cols, tokens, xs, ys)
        for t in range(tokens):
            a, b = got[t * ys:t * ys + rows], want[t * ys:t * ys + rows]
            assert rel_l2(a, b) <= 1e-5, f"call {call} token {t}"
            assert np.all(got[t * ys + rows:(t + 1) * ys] == -7.0), "wrote outside the output rows"
            # And the reference's CPU matvec order (the oracle) on the same row.
            ref = np.zeros(rows, dtype=np.float32)
            xt = np.ascontiguousarray(x[t * xs:t * xs + cols])
            load_oracle().plamo_bf16_matvec(w.ctypes.data, xt.ctypes.data, ref.ctypes.data, rows, cols)
            assert rel_l2(a, ref) <= 1e-5, f"call {call} token {t} against the oracle"


def test_static_linear_declines_requests_beyond_its_array(backend):
    pkg = load_package()
    limit = pkg._abi.LINEAR_STATIC_FLOATS
    rows, cols = 64, 4096
    tokens = limit // (rows + cols) + 1  # one token more than the array holds
    w = np.zeros((rows, cols), dtype=np.uint16)
    expect(backend, backend.lib.plamo_cuda_preload(backend.ctx, w.ctypes.data, w.nbytes), 1)
    x = np.zeros(tokens * cols, dtype=np.float32)
    y = np.full(tokens * rows, 5.0, dtype=np.float32)
    mm = pkg._abi.Matmul(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols, tokens, cols, rows)
    assert backend.lib.plamo_cuda_linear_static(backend.ctx, ctypes.byref(mm)) == 0
    assert b"static staging" in backend.info().note
    assert np.all(y == 5.0)


def test_static_linear_declines_sizes_whose_sum_would_wrap(backend):
    """tokens x columns and tokens x rows each fit in 64 bits, but their sum
    wraps to zero: declined by the size check, before any address is used."""
    pkg = load_package()
    x = np.zeros(4, dtype=np.float32)
    y = np.full(4, 5.0, dtype=np.float32)
    w = np.zeros(4, dtype=np.uint16)
    mm = pkg._abi.Matmul(w.ctypes.data, x.ctypes.data, y.ctypes.data, 1 << 31, 1 << 31, 1 << 32, 1 << 31, 1 << 31)
    assert backend.lib.plamo_cuda_linear_static(backend.ctx, ctypes.byref(mm)) == 0
    assert b"static staging" in backend.info().note
    assert np.all(y == 5.0)
