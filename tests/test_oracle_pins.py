"""Pins the C oracle to the reference.

The reference's CPU path (AArch64 assembly for Darwin) cannot run on this
host, so its own known-answer C tests are compiled, unchanged and where they
lie, against the oracle (oracle/Makefile `ref-tests`) and must all pass:
math, activation, token, qkv, rope, cache, cache_rope, rope_table, trig,
attention, model, mixer (closed-form layer/model), matmul (bitwise tiling),
prefill (40 bitwise prefill cases) and cache_rope_cached. The reference's
portable prompt cache (runtime/prompt_cache.c) is built from its source with
its own test, which pins the semantics the device prompt cache mirrors.
"""
import os
import subprocess

import numpy as np
import pytest

from conftest import REF, ORACLE_DIR, load_oracle, load_package


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "tests")),
                    reason="reference checkout not mounted on this machine")
def test_reference_known_answer_tests_pass_against_oracle():
    r = subprocess.run(["make", "-s", "-C", ORACLE_DIR, "ref-tests", f"REF={REF}"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    passes = [line for line in r.stdout.splitlines() if "PASS" in line]
    assert len(passes) == 17, r.stdout
    assert "template prefix snapshots: PASS" in r.stdout


def test_rope_frequencies_match_oracle_constants():
    """The package's RoPE frequency tables (used for descriptors) are the
    oracle's, bit for bit (reference tools/rope_constants.py:21-76)."""
    import ctypes
    pkg = load_package()
    o = load_oracle()
    local = np.ctypeslib.as_array((ctypes.c_float * 64).in_dll(o, "plamo_rope_local"))
    glob = np.ctypeslib.as_array((ctypes.c_float * 64).in_dll(o, "plamo_rope_global"))
    scale = ctypes.c_float.in_dll(o, "plamo_rope_global_scale").value
    p = pkg.PROFILES["8b"]
    assert np.array_equal(pkg.rope_frequencies(p.local_theta, 64), local)
    assert np.array_equal(
        pkg.rope_frequencies(p.global_theta, 64, (p.yarn_factor, p.yarn_original, p.beta_fast,
                                                  p.beta_slow)), glob)
    assert np.float32(pkg.concentration(p.yarn_factor)) == np.float32(scale)


def test_oracle_exp_is_the_reference_polynomial():
    """Spot values of the restated exp (reference src/activation.s:6-46) against
    libm within the reference's own bound (tests/activation.c: 5e-6)."""
    o = load_oracle()
    for x in np.linspace(-86, 87, 1001, dtype=np.float32):
        a, e = o.plamo_exp(float(x)), float(np.exp(np.float64(x)))
        assert abs(a / e - 1) < 5e-6
    assert o.plamo_exp(-100.0) == 0.0
    assert o.plamo_exp(100.0) == float("inf")


def test_oracle_threads_do_not_change_results():
    """Row-split threading keeps each row's accumulation order."""
    o = load_oracle()
    rng = np.random.default_rng(5)
    w = rng.integers(0, 1 << 16, size=(300, 1000), dtype=np.uint16) & np.uint16(0xBFFF)
    x = rng.normal(size=1000).astype(np.float32)
    ys = []
    for t in (1, 4):
        o.oracle_set_threads(t)
        y = np.zeros(300, dtype=np.float32)
        o.plamo_bf16_matvec(w.ctypes.data, x.ctypes.data, y.ctypes.data, 300, 1000)
        ys.append(y)
    o.oracle_set_threads(1)
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))
