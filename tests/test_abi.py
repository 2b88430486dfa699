"""The C-ABI library loads and exports every entry point include/plamo_cuda.h declares."""
import ctypes
import os
import re
import subprocess

from conftest import ROOT, load_package


def declared_entry_points():
    text = open(os.path.join(ROOT, "include", "plamo_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(plamo_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    pkg = load_package()
    lib = pkg.load()
    names = declared_entry_points()
    assert len(names) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(plamo_cuda_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        getattr(lib, n)
    # ctypes bindings cover exactly the declared ABI
    assert sorted(pkg._abi.SIGNATURES) == names


def test_library_exports_the_checkpoint_loader():
    pkg = load_package()
    pkg.load()
    text = open(os.path.join(ROOT, "include", "plamo_safetensors.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(plamo_\w+)\s*\(", text)))
    assert sorted(pkg._abi.LOADER_SIGNATURES) == names
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(plamo_\w+)", out))
    assert not [n for n in names if n not in exported]


def test_record_layouts_match_reference_abi():
    pkg = load_package()
    a = pkg._abi
    sizes = {a.Qkv: 72, a.Cache: 48, a.Rotation: 72, a.Gqa: 72, a.Mixer: 56, a.Mlp: 80,
             a.Layer: 64, a.Model: 88, a.Matmul: 64, a.Mapping: 16, a.WeightSpec: 32, a.Tensor: 64}
    for s, n in sizes.items():
        assert ctypes.sizeof(s) == n
    assert a.Layer.mixer.offset == 40
    assert a.Cache.count.offset == 24
    assert a.Rotation.processed_count.offset == 56


def test_open_reports_missing_device_without_gpu():
    pkg = load_package()
    lib = pkg.load()
    cfg = pkg._abi.CudaConfig(device=0)
    err = ctypes.create_string_buffer(256)
    ctx = lib.plamo_cuda_open(ctypes.byref(cfg), err, 256)
    if ctx:  # a GPU is present: nothing to check here
        lib.plamo_cuda_close(ctx)
        return
    assert err.value, "open must explain a failure"


def test_missing_library_fails_loudly(tmp_path):
    """No CPU fallback: without the CUDA library the package refuses to load."""
    import pytest
    pkg = load_package()
    with pytest.raises(OSError, match="no non-CUDA implementation"):
        pkg._abi.load(str(tmp_path / "libplamo_cuda.so"))


def test_python_constants_match_the_header():
    """The ctypes layer's copies of the header's limits."""
    text = open(os.path.join(ROOT, "include", "plamo_cuda.h")).read()
    a = load_package()._abi
    for name, value in (("PLAMO_CUDA_VERIFY_MAX", a.VERIFY_MAX), ("PLAMO_CUDA_PREFIX_LIMIT", a.PREFIX_LIMIT),
                        ("PLAMO_CUDA_TP_MAX", a.TP_MAX)):
        m = re.search(name + r"\s*=\s*(\d+)", text) or re.search(r"#define\s+" + name + r"\s+(\d+)", text)
        assert m, name
        assert int(m.group(1)) == value, name


def test_library_exports_the_model_layout_builder():
    pkg = load_package()
    pkg.load()
    text = open(os.path.join(ROOT, "include", "plamo_layout.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(plamo_\w+)\s*\(", text)))
    assert sorted(pkg._abi.LAYOUT_SIGNATURES) == names
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(plamo_\w+)", out))
    assert not [n for n in names if n not in exported]
    assert ctypes.sizeof(pkg._abi.ModelConfig) == 136


def test_library_exports_the_tokenizer():
    pkg = load_package()
    pkg.load()
    text = open(os.path.join(ROOT, "include", "plamo_tokenizer.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(plamo_\w+)\s*\(", text)))
    assert len(names) == 23
    assert set(pkg._abi.TOKENIZER_SIGNATURES) <= set(names)
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(plamo_\w+)", out))
    assert not [n for n in names if n not in exported]
