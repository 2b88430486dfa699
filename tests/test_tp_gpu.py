"""Tensor-parallel prefill and greedy decode against the oracle (2+ GPUs).

Each rank is a process with its own context on its own GPU holding its shard
(qh/size query heads, kh/size KV heads, intermediate/size MLP rows and a
slice of the head), with synthetic weights cut bit for bit from the full
model's. The ranks exchange their buffer handles over a gloo group, then run
the same calls: the prompt logits, gathered from the ranks' slices, must meet
the reference's GPU acceptance rule against the oracle's full-model prefill,
and the greedy tokens must equal the oracle's, also when a draft model
proposes them and the tensor-parallel target verifies blocks of 4.

Ranks leave only between calls (every call synchronises its stream), after a
barrier, so no rank frees its exchange buffer while a peer may still write
to it.
"""
import ctypes
import os
import socket
import time
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import synthetic
from conftest import assert_close, load_oracle, load_package
from fixtures import oracle_forward, oracle_prefill

pytestmark = pytest.mark.gpu

SEED = 29


def profile(pkg):
    return pkg.Profile("tp-small", 512, 4, 8, 4, 128, 1024, vocab=1000, window=16, pattern=2,
                       max_position=512)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, size, port, ids, max_tokens, out):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size, timeout=datetime.timedelta(seconds=120))
    b = None
    try:
        pkg = load_package()
        full = profile(pkg)
        shard = pkg.tp_shard_profile(full, size)
        b = pkg.Backend(device=rank, max_context=1024, max_prefill=256)
        hm = pkg.HostModel(shard, weights="synthetic")
        b.preload_synthetic_tp(hm, full, rank, size, SEED)
        handles = pkg.tp_all_gather_handles(b.tp_prepare(hm, rank, size))
        b.tp_connect(hm, handles)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        states = np.zeros((len(ids), full.hidden), dtype=np.float32)
        rc = b.lib.plamo_cuda_prefill(b.ctx, hm.ptr, ids.ctypes.data, len(ids), states.ctypes.data)
        first, rows = pkg.tp_vocab_slice(full.vocab, size, rank)
        logits = hm.logits_array()[first:first + rows]
        toks = np.zeros(max_tokens, dtype=np.uint32)
        timing = pkg._abi.CudaTiming()
        n = b.lib.plamo_cuda_generate(b.ctx, hm.ptr, ids.ctypes.data, len(ids), max_tokens, toks.ctypes.data,
                                      pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
        # Speculative decoding with the target tensor-parallel: a draft model
        # (the full model's heads on every rank: the shard profile's own
        # shapes, unrelated weights) proposes 4 tokens per verification.
        draft = pkg.HostModel(shard, weights="synthetic")
        b.preload_synthetic(draft, SEED + 50)
        b.prepare(draft)
        spec = np.zeros(max_tokens, dtype=np.uint32)
        stats = pkg._abi.CudaSpeculation()
        k = b.lib.plamo_cuda_generate_speculative(b.ctx, hm.ptr, draft.ptr, ids.ctypes.data, len(ids), max_tokens,
                                                  4, spec.ctypes.data, pkg._abi.TOKEN_CALLBACK(), None,
                                                  ctypes.byref(stats))
        out[rank] = dict(rc=rc, logits=logits, states=states, tokens=[int(t) for t in toks[:max(n, 0)]], n=n,
                         spec=[int(t) for t in spec[:max(k, 0)]], verify_batches=int(stats.verify_batches),
                         note=b.info().note.decode(), errors=b.info().errors)
    except Exception:
        out[rank] = dict(error=traceback.format_exc())
        # Keep the exchange buffer mapped until the peers' bounded waits
        # (2 s) have given up writing to it.
        time.sleep(5)
    finally:
        try:
            dist.barrier()
        finally:
            if b is not None:
                b.close()
            dist.destroy_process_group()


@pytest.mark.parametrize("size", [2, 4])
def test_tensor_parallel_matches_oracle(size):
    if torch.cuda.device_count() < size:
        pytest.skip(f"needs {size} GPUs")
    pkg = load_package()
    full = profile(pkg)
    ids = np.random.default_rng(3).integers(3, full.vocab, size=20).astype(np.uint32)
    max_tokens = 24
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_rank, args=(size, _free_port(), ids, max_tokens, out), nprocs=size, join=True)
        res = [dict(out[r]) for r in range(size)]
    for r in res:
        assert "error" not in r, r.get("error")
        assert r["rc"] == 1 and r["n"] >= 0, r["note"]
        assert r["errors"] == 0, r["note"]
    # Oracle on the full model (host copy of the same synthetic weights).
    ref = pkg.HostModel(full)
    synthetic.fill_model(ref, SEED)
    ok, want_states = oracle_prefill(ref, ids)
    assert ok == 1
    want_logits = ref.logits_array()
    got_logits = np.concatenate([r["logits"] for r in res])
    assert_close(got_logits, want_logits, "tensor-parallel prompt logits")
    for r in res:
        assert_close(r["states"], want_states, "prompt states")
    o = load_oracle()
    want_tokens = []
    for _ in range(max_tokens):
        t = int(o.plamo_argmax(ref.model.logits, full.vocab))
        if t in (1, 16):
            break
        want_tokens.append(t)
        if len(want_tokens) == max_tokens:
            break
        assert oracle_forward(ref, t) == 1
    for rank, r in enumerate(res):
        assert r["tokens"] == want_tokens, f"rank {rank}"
        assert r["spec"] == want_tokens, f"rank {rank} speculative"
        assert r["verify_batches"] > 0


def _absent_peer(rank, size, port, out):
    """Rank 1 prepares and connects, then never runs the step: rank 0's step
    must fail within its bounded waits (about 2 s per wait, then the rest of
    the operation skips its waits) and report the missing peer."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size, timeout=datetime.timedelta(seconds=120))
    b = None
    try:
        pkg = load_package()
        full = profile(pkg)
        shard = pkg.tp_shard_profile(full, size)
        b = pkg.Backend(device=rank, max_context=1024, max_prefill=256)
        hm = pkg.HostModel(shard, weights="synthetic")
        b.preload_synthetic_tp(hm, full, rank, size, SEED)
        b.tp_connect(hm, pkg.tp_all_gather_handles(b.tp_prepare(hm, rank, size)))
        if rank == 0:
            ids = np.arange(3, 23, dtype=np.uint32)
            t0 = time.perf_counter()
            rc = b.lib.plamo_cuda_prefill(b.ctx, hm.ptr, ids.ctypes.data, len(ids), None)
            out[rank] = dict(rc=rc, seconds=time.perf_counter() - t0, note=b.info().note.decode(),
                             errors=b.info().errors)
        else:
            out[rank] = dict(rc=None)
    except Exception:
        out[rank] = dict(error=traceback.format_exc())
        time.sleep(5)
    finally:
        try:
            dist.barrier()  # rank 1 stays mapped until rank 0's call has returned
        finally:
            if b is not None:
                b.close()
            dist.destroy_process_group()


def test_missing_peer_fails_the_call_instead_of_hanging():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_absent_peer, args=(2, _free_port(), out), nprocs=2, join=True)
        res = [dict(out[r]) for r in range(2)]
    for r in res:
        assert "error" not in r, r.get("error")
    r0 = res[0]
    assert r0["rc"] == -1
    assert "did not arrive" in r0["note"]
    assert r0["seconds"] < 60
