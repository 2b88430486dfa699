"""The reference-side adapter (plamo-3-translate.c_b200/integration/metal_cuda.c)
compiled against the reference's own headers: runtime/metal.h, compute.h,
model.h, parallel.h and weight_cache.h, together with include/plamo_cuda.h.

The object must define every plamo_metal_* entry point the reference
declares, and every plamo_cuda_* symbol it calls must be exported by the
library. Skips where the reference checkout is absent (GPU hosts)."""
import os
import re
import subprocess

import pytest

from conftest import REF, ROOT, load_package

ADAPTER = os.path.join(ROOT, "plamo-3-translate.c_b200", "integration", "metal_cuda.c")
RUNTIME = os.path.join(REF, "runtime")


def nm(path, *flags):
    return subprocess.run(["nm", *flags, path], capture_output=True, text=True, check=True).stdout


@pytest.mark.skipif(not os.path.isfile(os.path.join(RUNTIME, "metal.h")), reason="reference checkout absent")
def test_adapter_compiles_against_the_reference_headers(tmp_path):
    obj = tmp_path / "metal_cuda.o"
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-c", ADAPTER, "-I", RUNTIME, "-I",
                        os.path.join(ROOT, "include"), "-o", str(obj)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    header = open(os.path.join(RUNTIME, "metal.h")).read()
    declared = set(re.findall(r"\b(plamo_metal_\w+)\s*\(", re.sub(r"/\*.*?\*/", "", header, flags=re.S)))
    symbols = nm(str(obj))
    defined = set(re.findall(r"\sT\s(plamo_metal_\w+)", symbols))
    assert declared and declared <= defined, sorted(declared - defined)
    needed = set(re.findall(r"\sU\s(plamo_cuda_\w+)", symbols))
    pkg = load_package()
    pkg.load()
    exported = set(re.findall(r"\sT\s(plamo_cuda_\w+)", nm(pkg.LIB_PATH, "-D", "--defined-only")))
    assert needed and needed <= exported, sorted(needed - exported)
    # The compute hooks and the CPU fallback come from the reference's own objects.
    assert {"plamo_compute_context", "plamo_forward_kernel", "plamo_bf16_matmul_core"} <= \
        set(re.findall(r"\sU\s(\w+)", symbols))
