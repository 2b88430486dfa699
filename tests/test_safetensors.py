"""BF16 safetensors loader (include/plamo_safetensors.h), host only.

Pinned by the reference's own loader tests (tests/find.c, tests/load.c),
compiled unchanged where they lie and linked against the product library;
then checkpoints written here are mapped and bound to a profile's schema:
every slot must point at its tensor's bytes, shards may split the tensors,
and any dtype, shape, name or bounds problem must fail the whole binding.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from conftest import REF, load_package


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "tests")),
                    reason="reference checkout not mounted on this machine")
@pytest.mark.parametrize("name", ["find", "load"])
def test_reference_loader_tests_pass_against_library(tmp_path, name):
    pkg = load_package()
    libdir = os.path.dirname(pkg.LIB_PATH)
    exe = tmp_path / f"test-{name}"
    subprocess.run(["gcc", "-O2", "-w", os.path.join(REF, "tests", f"{name}.c"), "-L", libdir, "-lplamo_cuda",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True, capture_output=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout


def small(pkg):
    return pkg.Profile("st", 64, 2, 4, 2, 16, 96, vocab=50, window=8, pattern=2, max_position=64)


def tensors_of(pkg, prof, seed=3):
    rng = np.random.default_rng(seed)
    return {name: rng.integers(0, 65535, size=shape, dtype=np.uint16) for name, shape in pkg.schema(prof)}


def test_checkpoint_binds_every_schema_tensor_across_shards(tmp_path):
    pkg = load_package()
    prof = small(pkg)
    t = tensors_of(pkg, prof)
    names = list(t)
    half = len(names) // 2
    a, b = tmp_path / "a.safetensors", tmp_path / "b.safetensors"
    pkg.write_safetensors(a, {n: t[n] for n in names[half:]}, metadata={"format": "pt"})
    pkg.write_safetensors(b, {n: t[n] for n in names[:half]})
    ck = pkg.Checkpoint([str(a), str(b)], prof)
    try:
        hm = ck.model
        for addr, count, name in hm.tensor_ranges():
            got = np.ctypeslib.as_array(ctypes.cast(addr, ctypes.POINTER(ctypes.c_uint16)), shape=(count,))
            assert np.array_equal(got, t[name].reshape(-1)), name
        assert hm.model.embedding == hm.addresses["model.embed_tokens.weight"]
    finally:
        ck.close()


@pytest.mark.parametrize("problem", ["shape", "missing", "dtype", "bounds"])
def test_checkpoint_mismatch_fails_the_whole_binding(tmp_path, problem):
    pkg = load_package()
    prof = small(pkg)
    t = tensors_of(pkg, prof)
    path = tmp_path / "m.safetensors"
    victim = "model.layers.layers.1.mlp.down_proj.weight"
    if problem == "shape":
        t[victim] = t[victim].reshape(-1)
    elif problem == "missing":
        del t[victim]
    pkg.write_safetensors(path, t)
    if problem in ("dtype", "bounds"):
        raw = bytearray(path.read_bytes())
        n = int.from_bytes(raw[:8], "little")
        header = raw[8:8 + n].decode()
        if problem == "dtype":
            header = header.replace('"BF16"', '"BF17"', 1)
        else:
            raw = raw[:len(raw) - 2]  # the last tensor's data runs past the end
        raw[8:8 + n] = header.encode()
        path.write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        pkg.Checkpoint([str(path)], prof)


def test_find_tensor_rejects_malformed_headers():
    pkg = load_package()
    lib = pkg.load()

    def file_with(header, data=b"\0" * 8):
        text = header.encode()
        return len(text).to_bytes(8, "little") + text + data

    def find(buf, name):
        t = pkg._abi.Tensor()
        ok = lib.plamo_find_tensor(buf, len(buf), name.encode(), ctypes.byref(t))
        return ok, t

    good = '{"x":{"dtype":"BF16","shape":[2,2],"data_offsets":[0,8]}}'
    ok, t = find(file_with(good), "x")
    assert ok == 1 and t.bytes == 8 and t.rank == 2 and list(t.dims[:2]) == [2, 2]
    for bad in ['{"x":{"dtype":"BF16","shape":[2,2],"data_offsets":[0,6]}}',     # bytes != shape
                '{"x":{"dtype":"BF16","shape":[2,2],"data_offsets":[0,16]}}',    # past the data
                '{"x":{"dtype":"BF16","shape":[2,2],"data_offsets":[08,16]}}',   # leading zero
                '{"x":{"dtype":"BF16","shape":[1,1,1,1,8],"data_offsets":[0,16]}}',  # rank 5
                '{"x":{"dtype":"BF16","dtype":"BF16","shape":[4],"data_offsets":[0,8]}}',  # repeated key
                '{"x":{"dtype":"BF16","shape":[4]}}',                             # missing offsets
                '{"x":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}}',          # not BF16
                '{}']:
        ok, t = find(file_with(bad), "x")
        assert ok == 0 and not t.data, bad
    ok, _ = find(file_with(good), "y")
    assert ok == 0


@pytest.mark.gpu
def test_mapped_checkpoint_decodes_like_the_same_weights_in_memory(tmp_path, backend):
    """A checkpoint written from synthetic weights, mapped and uploaded by host
    address, gives the same greedy tokens as the same bytes held in a blob."""
    pkg = load_package()
    prof = pkg.Profile("st-gpu", 256, 2, 4, 2, 64, 512, vocab=500, window=8, pattern=2, max_position=256)
    blob_model = pkg.HostModel(prof)
    import synthetic
    synthetic.fill_model(blob_model, 5)
    tensors = {name: blob_model.tensor(name) for name, _ in pkg.schema(prof)}
    path = tmp_path / "model.safetensors"
    pkg.write_safetensors(path, tensors)
    ck = pkg.Checkpoint([str(path)], prof)
    lib = backend.lib
    ids = np.arange(3, 15, dtype=np.uint32)
    outs = []
    try:
        for hm in (ck.model, blob_model):
            backend.preload_model(hm)
            backend.prepare(hm)
            out = np.zeros(16, dtype=np.uint32)
            timing = pkg._abi.CudaTiming()
            n = lib.plamo_cuda_generate(backend.ctx, hm.ptr, ids.ctypes.data, len(ids), 16, out.ctypes.data,
                                        pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
            assert n > 0, backend.info().note
            outs.append(list(out[:n]))
            backend.release(hm)
    finally:
        ck.close()
    assert outs[0] == outs[1]
