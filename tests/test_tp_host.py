"""Host logic of tensor parallelism (no GPU).

The shard cuts must partition every split tensor of the full model exactly
(each weight on exactly one rank, in the order the shard's kernels expect),
the head slices must partition the vocabulary, a shard's synthetic weights
must be the full tensor's elements at the cut positions, and the exchange of
the ranks' buffer handles must hand every rank all handles in rank order
(run as two gloo ranks on the CPU).
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import synthetic
from conftest import load_package



def small(pkg, qh=8, kh=4, inter=96):
    return pkg.Profile("tp", 64, 2, qh, kh, 16, inter, vocab=1003, window=8, pattern=2, max_position=64)


@pytest.mark.parametrize("size", [2, 4])
def test_shards_partition_every_split_tensor(size):
    pkg = load_package()
    full = small(pkg)
    shard = pkg.tp_shard_profile(full, size)
    shapes, shard_shapes = dict(pkg.schema(full)), dict(pkg.schema(shard))
    for name, shape in shapes.items():
        owners = np.zeros(shape if len(shape) == 2 else (shape[0], 1), dtype=np.int32)
        for rank in range(size):
            cut = pkg.tp_segments(full, size, rank, name)
            if cut is None:
                assert shard_shapes[name] == shape, name
                continue
            cols, full_cols, col0, segs = cut
            assert full_cols == shape[1]
            assert sum(n for _, n in segs) == shard_shapes[name][0] and cols == shard_shapes[name][1], name
            for start, n in segs:
                owners[start:start + n, col0:col0 + cols] += 1
        if pkg.tp_segments(full, size, 0, name) is not None:
            assert np.all(owners == 1), name


def test_vocab_slices_partition_vocabulary():
    pkg = load_package()
    for vocab in (1000, 1003, 107520):
        for size in (2, 4, 8):
            rows = [pkg.tp_vocab_slice(vocab, size, r) for r in range(size)]
            assert rows[0][0] == 0
            for (a, n), (b, _) in zip(rows, rows[1:]):
                assert a + n == b
            assert rows[-1][0] + rows[-1][1] == vocab


def test_shard_values_are_the_full_tensor_at_the_cut():
    """The index rule of plamo_cuda_preload_synthetic_rows: element (r, c) of
    segment (row0, n) is element (row0 + r) * full_cols + col0 + c of the
    full tensor (numpy restatement of the device generator)."""
    pkg = load_package()
    full = small(pkg)
    seed = 7
    for name, shape in pkg.schema(full):
        cut = pkg.tp_segments(full, 2, 1, name)
        if cut is None:
            continue
        whole = synthetic.bf16(seed, int(np.prod(shape)), 0.0, 0.02).reshape(shape)
        cols, full_cols, col0, segs = cut
        parts = []
        for start, n in segs:
            idx = (start + np.arange(n))[:, None] * full_cols + col0 + np.arange(cols)[None, :]
            z = synthetic.z(seed, int(idx.max()) + 1)[idx.reshape(-1)].reshape(idx.shape)
            parts.append(synthetic.bf16_round(np.float32(0.02) * z))
        got = np.concatenate(parts)
        want = np.concatenate([whole[s:s + n, col0:col0 + cols] for s, n in segs])
        assert np.array_equal(got, want), name


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange(rank, size, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        pkg = load_package()
        mine = bytes([rank + 1]) * 64
        got = pkg.tp_all_gather_handles(mine)
        out[rank] = b"".join(got)
    finally:
        dist.destroy_process_group()


def test_handle_exchange_two_gloo_ranks():
    size = 2
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_exchange, args=(size, _free_port(), out), nprocs=size, join=True)
        for rank in range(size):
            assert out[rank] == b"".join(bytes([r + 1]) * 64 for r in range(size))
