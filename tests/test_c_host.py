"""A C host program over include/*.h alone, compiled with the C compiler.

The drop-in boundary is C: an engine on Linux links the library and includes
its headers, with no Python anywhere. This program follows the integration
path: the tokenizer wraps a request in the translation prompt, a checkpoint
is mapped and bound into descriptors built at run time, then the CUDA
backend preloads, prepares and generates. Without a GPU plamo_cuda_open
declines with a message and the program stops there, so the host half runs
on any machine.
"""
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, load_package

PROGRAM = r"""
#include "plamo_cuda.h"
#include "plamo_layout.h"
#include "plamo_safetensors.h"
#include "plamo_tokenizer.h"

#include <stdio.h>
#include <string.h>

static int keep_going(uint32_t id, void *context) {
    (void)id;
    ++*(unsigned *)context;
    return 1;
}

int main(int argc, char **argv) {
    char err[256];
    if (argc != 3) return 90;
    struct plamo_tokenizer *tok = plamo_tokenizer_open(argv[1], err, sizeof err);
    if (!tok) { fprintf(stderr, "tokenizer: %s\n", err); return 1; }
    const uint32_t *ids;
    uint64_t n = plamo_tokenizer_encode(tok, "Hello.", 1, &ids, err, sizeof err);
    if (n == UINT64_MAX || n == 0) { fprintf(stderr, "encode: %s\n", err); return 2; }

    struct plamo_model_config cfg = {64, 2, 4, 2, 16, 96, 50, 8, 2, 128, 0,
                                     10000.0, 1000000.0, 256.0, 4096.0, 32.0, 1.0};
    struct plamo_model_layout *lay = plamo_model_layout_create(&cfg, 128, err, sizeof err);
    if (!lay) { fprintf(stderr, "layout: %s\n", err); return 3; }
    struct plamo_mapping map;
    if (!plamo_map_file(argv[2], &map)) return 4;
    if (!plamo_bind_weights(&map, 1, plamo_model_layout_schema(lay)) || !plamo_model_layout_finish(lay)) return 5;
    struct model *model = plamo_model_layout_model(lay);
    printf("prompt %llu ids, model of %llu layers bound\n", (unsigned long long)n,
           (unsigned long long)model->count);

    struct plamo_cuda_config cc;
    memset(&cc, 0, sizeof cc);
    struct plamo_cuda *cuda = plamo_cuda_open(&cc, err, sizeof err);
    if (!cuda) {
        printf("no CUDA device: %s\n", err[0] ? "declined with a reason" : "declined");
    } else {
        /* This small model's vocabulary is 50 rows: fold the prompt ids into it. */
        uint32_t prompt[64], out[8];
        uint64_t k = n < 64 ? n : 64;
        for (uint64_t i = 0; i < k; ++i) prompt[i] = ids[i] % 50;
        unsigned seen = 0;
        struct plamo_cuda_timing timing;
        if (!plamo_cuda_preload(cuda, map.base, map.bytes) || plamo_cuda_prepare_model(cuda, model) != 1) return 6;
        int64_t made = plamo_cuda_generate(cuda, model, prompt, k, 8, out, keep_going, &seen, &timing);
        if (made < 0) return 7;
        for (int64_t i = 0; i < made; ++i) {
            const char *bytes;
            if (plamo_tokenizer_decode(tok, out[i], &bytes) == UINT64_MAX) return 8;
        }
        printf("generated %lld tokens\n", (long long)made);
        plamo_cuda_release_model(cuda, model);
        plamo_cuda_close(cuda);
    }
    plamo_unmap_file(&map);
    plamo_model_layout_destroy(lay);
    plamo_tokenizer_close(tok);
    return 0;
}
"""


def build_host_program(tmp_path):
    """(executable, vocabulary file, checkpoint) of the C host program."""
    pkg = load_package()
    pkg.load()
    libdir = os.path.dirname(pkg.LIB_PATH)
    src = tmp_path / "host.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "host"
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(src), "-L", libdir, "-lplamo_cuda", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr

    vocab = tmp_path / "tokenizer.jsonl"
    rows = ['["unused", 0, "NORMAL"]'] + [f'["<0x{b:02X}>", 0, "BYTE"]' for b in range(256)]
    rows += ['["Hello", -1.0, "NORMAL"]', '["<|plamo:bos|>", 0, "CONTROL"]']
    rows += ['["x", -1, "NORMAL"]'] * (107520 - len(rows))
    vocab.write_text("\n".join(rows) + "\n", encoding="utf-8")

    prof = pkg.Profile("c-host", 64, 2, 4, 2, 16, 96, vocab=50, window=8, pattern=2, max_position=128)
    rng = np.random.default_rng(3)
    tensors = {}
    for name, shape in pkg.schema(prof):
        x = rng.normal(0.0, 0.05, size=shape).astype(np.float32) + (1.0 if "norm" in name else 0.0)
        tensors[name] = (x.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    ckpt = tmp_path / "model.safetensors"
    pkg.write_safetensors(ckpt, tensors)
    return exe, vocab, ckpt


def test_c_host_program_builds_and_runs_the_host_path(tmp_path):
    exe, vocab, ckpt = build_host_program(tmp_path)
    r = subprocess.run([str(exe), str(vocab), str(ckpt)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "model of 2 layers bound" in r.stdout
    assert "no CUDA device: declined with a reason" in r.stdout or "generated" in r.stdout


@pytest.mark.gpu
def test_c_host_program_generates_on_the_gpu(tmp_path):
    """The same program on a GPU host: the backend opens, preloads the mapped
    checkpoint, prepares the run-time descriptors and generates up to 8
    tokens (fewer when a stop id comes first)."""
    exe, vocab, ckpt = build_host_program(tmp_path)
    r = subprocess.run([str(exe), str(vocab), str(ckpt)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert re.search(r"generated [0-8] tokens", r.stdout), r.stdout
