"""The CUDA path against the committed golden fixtures (tests/golden/).

No oracle call and no reference checkout: the expected values are the
oracle's frozen outputs (tests/golden/make_golden.py), so this is the parity
check that travels with the repository.
  * GEMV: relative L2 <= 1e-5 of the reference matvec.
  * 4-layer model: prefill logits and state within relative L2 <= 1e-4 (the
    whole-model rule of reference tools/compare_backends.py:16-33), then the
    48 greedy tokens identical.
  * two-layer fixture of reference tests/metal_decode.c: state and logits
    after the prefill and after every forward step within that test's rule
    (relative L2 <= 1e-4, max |delta| <= 1e-5 * (1 + max |ref|)).
"""
import ctypes
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import make_golden as golden  # noqa: E402
from conftest import assert_close, expect, load_package, rel_l2  # noqa: E402
from fixtures import decode_fixture_pair  # noqa: E402
from test_gemv_gpu import gpu_matvec  # noqa: E402

pytestmark = pytest.mark.gpu


def fixture(name):
    return np.load(os.path.join(HERE, "golden", f"{name}.npz"))


@pytest.mark.parametrize("rows,cols", golden.GEMV_SHAPES)
def test_gemv_matches_golden(backend, rows, cols):
    g = fixture("gemv")
    key = f"{rows}x{cols}"
    w, x = golden.gemv_inputs(rows, cols)
    assert golden.sha256(w) == str(g[f"w_sha256_{key}"])
    assert rel_l2(gpu_matvec(backend, w, x), g[f"y_{key}"]) <= 1e-5


def test_small_model_matches_golden(backend):
    pkg = load_package()
    g = fixture("model_small")
    hm = pkg.HostModel(golden.small_profile(), weights="synthetic")
    backend.preload_synthetic(hm, golden.SMALL_SEED)
    backend.prepare(hm)
    try:
        ids = np.ascontiguousarray(g["ids"], dtype=np.uint32)
        expect(backend, backend.lib.plamo_cuda_prefill(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), 0))
        for name, got, want in (("logits", hm.logits_array(), g["prefill_logits"]),
                                ("state", hm.state_array(), g["prefill_state"])):
            assert np.all(np.isfinite(got)), name
            assert rel_l2(got, want) <= 1e-4, f"prefill {name}: {rel_l2(got, want):.3g}"
        hm.reset()
        out = np.zeros(golden.SMALL_TOKENS, dtype=np.uint32)
        timing = pkg._abi.CudaTiming()
        n = backend.lib.plamo_cuda_generate(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), golden.SMALL_TOKENS,
                                            out.ctypes.data, pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
        assert n >= 0, backend.info().note
        assert out[:n].tolist() == g["tokens"].tolist(), f"oracle top-2 margins {g['margins'].tolist()}"
    finally:
        backend.release(hm)


def test_decode_fixture_matches_golden(backend):
    g = fixture("decode_fixture")
    a, _ = decode_fixture_pair(128, 257, 128, 40)
    backend.preload_model(a)
    backend.prepare(a)
    try:
        lib, ctx = backend.lib, backend.ctx
        ids = np.ascontiguousarray(g["ids"], dtype=np.uint32)
        expect(backend, lib.plamo_cuda_prefill(ctx, a.ptr, ids.ctypes.data, len(ids), 0))
        assert_close(a.state_array(), g["states"][0], "prefill state")
        assert_close(a.logits_array(), g["logits"][0], "prefill logits")
        for i, t in enumerate(g["steps"], start=1):
            expect(backend, lib.plamo_cuda_forward(ctx, a.ptr, int(t)))
            assert_close(a.state_array(), g["states"][i], f"step {i} state")
            assert_close(a.logits_array(), g["logits"][i], f"step {i} logits")
    finally:
        backend.release(a)
