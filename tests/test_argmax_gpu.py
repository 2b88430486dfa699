"""Greedy argmax edge cases on the GPU (reference src/token.s:37-63, pinned by
reference tests/token.c:19-30): ties go to the lowest index, any NaN logit
makes the choice an error (UINT32_MAX on the device, UINT64_MAX in the
reference), and a vector of -inf chooses index 0.

The logits come out of the real head projection: a small model whose head
rows are crafted, so the device argmax runs where it runs in production - the
head GEMV's per-block candidates and their merge (decode), the prompt's head
(prefill) and the per-row argmax of a verification block. Every device choice
is also compared with the oracle's plamo_argmax on the same logits.
"""
import ctypes

import numpy as np
import pytest

import synthetic
from conftest import expect, load_oracle, load_package

pytestmark = pytest.mark.gpu

ERROR = 0xFFFFFFFF
BF16_POS_INF, BF16_NEG_INF, BF16_NAN = 0x7F80, 0xFF80, 0x7FC0


def profile(pkg):
    return pkg.Profile("argmax", 256, 2, 4, 2, 64, 512, vocab=1000, window=16, pattern=2, max_position=512)


def base_model(pkg, seed=41):
    hm = pkg.HostModel(profile(pkg))
    synthetic.fill_model(hm, seed)
    return hm


def crafted(pkg, base, edit):
    """Copy of `base` whose head rows `edit(head)` rewrites in place."""
    hm = pkg.HostModel(base.profile, weights=base.blob.copy())
    edit(hm.tensor("lm_head.weight"))
    return hm


def prompt_ids():
    return np.random.default_rng(12).integers(3, 1000, size=7).astype(np.uint32)


def final_normalized(backend, base):
    """The final-norm output after the prompt (independent of the head)."""
    backend.preload_model(base)
    backend.prepare(base)
    ids = prompt_ids()
    expect(backend, backend.lib.plamo_cuda_prefill(backend.ctx, base.ptr, ids.ctypes.data, len(ids), None))
    n = base.normalized_array()
    backend.release(base)
    return n


def prefill_choice(backend, hm):
    """(device greedy choice after the prompt, host logits of the same prompt)."""
    lib = backend.lib
    ids = prompt_ids()
    nxt = ctypes.c_uint32(12345)
    hm.reset()
    lib.plamo_cuda_reset_request(backend.ctx, hm.ptr)
    expect(backend, lib.plamo_cuda_prefill_greedy(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), ctypes.byref(nxt)))
    hm.reset()
    lib.plamo_cuda_reset_request(backend.ctx, hm.ptr)
    expect(backend, lib.plamo_cuda_prefill(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), None))
    return nxt.value, hm.logits_array()


def oracle_choice(logits):
    x = np.ascontiguousarray(logits, dtype=np.float32)
    r = int(load_oracle().plamo_argmax(x.ctypes.data, len(x)))
    return ERROR if r == 2**64 - 1 else r


def load(backend, hm):
    backend.preload_model(hm)
    backend.prepare(hm)


def test_tie_across_the_whole_vocabulary_chooses_index_0(backend):
    """Every head row identical: all logits equal at every step; the prefill
    head, each decode step (per-block candidates + merge) and every row of a
    verification block choose 0."""
    pkg = load_package()
    base = base_model(pkg)
    hm = crafted(pkg, base, lambda head: head.__setitem__(slice(None), head[0]))
    load(backend, hm)
    lib = backend.lib
    nxt, logits = prefill_choice(backend, hm)
    assert np.all(logits == logits[0]) and np.isfinite(logits[0])
    assert nxt == 0 == oracle_choice(logits)
    for token in (5, 17, 999):
        expect(backend, lib.plamo_cuda_forward(backend.ctx, hm.ptr, token))
        logits = hm.logits_array()
        assert np.all(logits == logits[0])
        out = ctypes.c_uint32(12345)
        expect(backend, lib.plamo_cuda_forward_greedy(backend.ctx, hm.ptr, token, ctypes.byref(out)))
        assert out.value == 0 == oracle_choice(logits)
    block = np.array([3, 9, 400, 77], dtype=np.uint32)
    got = np.full(len(block), 12345, dtype=np.uint32)
    expect(backend, lib.plamo_cuda_verify(backend.ctx, hm.ptr, block.ctypes.data, len(block), got.ctypes.data))
    assert np.all(got == 0)
    backend.release(hm)


@pytest.mark.parametrize("rows", [(3, 700), (701, 702), (998, 999), (0, 513)])
def test_tie_at_the_maximum_chooses_the_lower_index(backend, rows):
    """Two identical head rows aligned with the final normalised vector (so
    their logit is far above every other): the lower index wins, whether the
    two rows fall in one block of the head projection or in two."""
    pkg = load_package()
    base = base_model(pkg)
    n = final_normalized(backend, base)
    row = synthetic.bf16_round(np.where(n >= 0, 0.05, -0.05).astype(np.float32))

    def edit(head):
        for r in rows:
            head[r] = row

    hm = crafted(pkg, base, edit)
    load(backend, hm)
    nxt, logits = prefill_choice(backend, hm)
    a, b = rows
    assert logits[a] == logits[b] and logits[a] == logits.max()
    assert np.count_nonzero(logits == logits.max()) == 2
    assert nxt == min(rows) == oracle_choice(logits)
    backend.release(hm)


@pytest.mark.parametrize("row", [0, 517, 999])
def test_nan_logit_is_an_error(backend, row):
    """One NaN head weight makes its logit NaN: the greedy choice is the
    error value on the prefill and decode paths, and the request loop fails."""
    pkg = load_package()
    base = base_model(pkg)
    hm = crafted(pkg, base, lambda head: head.__setitem__((row, 7), BF16_NAN))
    load(backend, hm)
    lib = backend.lib
    nxt, logits = prefill_choice(backend, hm)
    assert np.isnan(logits[row]) and np.count_nonzero(np.isnan(logits)) == 1
    assert nxt == ERROR == oracle_choice(logits)
    out = ctypes.c_uint32(12345)
    expect(backend, lib.plamo_cuda_forward_greedy(backend.ctx, hm.ptr, 11, ctypes.byref(out)))
    assert out.value == ERROR
    ids = prompt_ids()
    tokens = np.zeros(4, dtype=np.uint32)
    timing = pkg._abi.CudaTiming()
    assert lib.plamo_cuda_generate(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), 4, tokens.ctypes.data,
                                   pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing)) == -1
    backend.release(hm)


def test_all_negative_infinity_chooses_index_0(backend):
    """Every head row holds -inf times the sign of one normalised element and
    zeros elsewhere, so every logit is exactly -inf: the choice is 0."""
    pkg = load_package()
    base = base_model(pkg)
    n = final_normalized(backend, base)
    c = int(np.argmax(np.abs(n)))

    def edit(head):
        head[:] = 0
        head[:, c] = BF16_NEG_INF if n[c] > 0 else BF16_POS_INF

    hm = crafted(pkg, base, edit)
    load(backend, hm)
    nxt, logits = prefill_choice(backend, hm)
    assert np.all(logits == -np.inf)
    assert nxt == 0 == oracle_choice(logits)
    backend.release(hm)
