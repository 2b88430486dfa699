"""The Linux engine (include/plamo_engine.h; reference runtime/engine.h:48-62)
driven by a C program over the public headers alone: open from a checkpoint
and a vocabulary, prepare (template prefixes snapshotted on the device),
tokenize, translate with streamed token callbacks.

On any host: the tokenizer-only engine encodes the translation prompt and
refuses generation; a full open without a GPU fails with a message. On a GPU
host: "Hello." English -> Japanese on a synthetic checkpoint and vocabulary
emits, token for token, the ids plamo_cuda_generate produces for the same
prompt ids, both with and without the device prefix snapshot, and the
snapshot covers the template's head.
"""
import ctypes
import json
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, load_package

PROGRAM = r"""
#define _POSIX_C_SOURCE 200809L
#include "plamo_engine.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static int on_token(uint32_t id, const char *bytes, size_t count, void *context) {
    (void)bytes;
    (void)count;
    unsigned *seen = context;
    printf("token %u\n", id);
    return ++*seen < 1000;
}

static void on_prefill(uint64_t tokens, void *context) {
    (void)context;
    printf("prefill %llu\n", (unsigned long long)tokens);
}

int main(int argc, char **argv) {
    if (argc != 4) return 90;
    const int tokenizer_only = !strcmp(argv[3], "tokenizer");
    const char *weights[1] = {argv[2]};
    struct plamo_model_config cfg = {128, 2, 4, 2, 32, 192, 107520, 64, 2, 512, 0,
                                     10000.0, 1000000.0, 256.0, 4096.0, 32.0, 1.0};
    struct plamo_engine_files files = {argv[1], weights, 1, NULL, &cfg, 512, 0};
    struct plamo_engine_info info;
    char err[512];
    struct plamo_engine *e = plamo_engine_open_files(&files, PLAMO_MEMORY_RESIDENT, tokenizer_only, 4,
                                                     PLAMO_BACKEND_AUTO, &info, err, sizeof err);
    if (!e) {
        printf("open failed: %s\n", err);
        return 0;
    }
    printf("backend %s memory %s\n", info.backend, info.memory_mode);
    const uint32_t *ids;
    uint64_t n = plamo_engine_tokenize(e, "Hello.", 1, &ids, err, sizeof err);
    if (n == UINT64_MAX) return 2;
    printf("prompt");
    for (uint64_t i = 0; i < n; ++i) printf(" %u", ids[i]);
    printf("\n");
    if (!strcmp(argv[3], "noprefix")) setenv("PLAMO_PREFIX_CACHE", "0", 1);
    if (!plamo_engine_prepare(e, err, sizeof err)) {
        printf("prepare failed: %s\n", err);
        return 3;
    }
    plamo_engine_get_info(e, &info);
    printf("prefix %llu %llu\n", (unsigned long long)info.prefix_tokens[0], (unsigned long long)info.prefix_tokens[1]);
    unsigned seen = 0;
    struct plamo_callbacks cb = {on_prefill, on_token, &seen};
    struct plamo_result r;
    if (!plamo_engine_translate(e, "Hello.", 1, 12, &cb, &r, err, sizeof err)) {
        printf("translate refused: %s\n", err);
    } else {
        printf("finish %s completion %llu cached %llu steps %llu\n", r.finish_reason,
               (unsigned long long)r.completion_tokens, (unsigned long long)r.cached_prompt_tokens,
               (unsigned long long)r.decode_steps);
        size_t need = plamo_engine_report_json(e, &r, NULL, 0);
        char *json = malloc(need + 1);
        if (!json || plamo_engine_report_json(e, &r, json, need + 1) != need) return 4;
        printf("report %s\n", json);
        free(json);
    }
    char compute[4096];
    if (plamo_engine_report_json(e, NULL, compute, sizeof compute) >= sizeof compute) return 5;
    printf("compute %s\n", compute);
    plamo_engine_close(e);
    return 0;
}
"""


def write_vocab(path):
    rows = ['["unused", 0, "NORMAL"]'] + [f'["<0x{b:02X}>", 0, "BYTE"]' for b in range(256)]
    # The template's special and word pieces, as the real vocabulary has them,
    # so the fixed prefix is a dozen ids (the device snapshot holds at most 64).
    rows += ['["Hello", -1.0, "NORMAL"]']
    rows += [f'["<|plamo:{t}|>", 0, "CONTROL"]' for t in ("bos", "tag", "msg", "key", "val", "op")]
    rows += [f'["{w}", -2.0, "NORMAL"]' for w in ("dataset", "translation", "input", "output", "lang", "en", "ja")]
    rows += [f'["w{i}", -3, "NORMAL"]' for i in range(107520 - len(rows))]
    path.write_text("\n".join(rows) + "\n", encoding="utf-8")


def engine_profile(pkg):
    # The sliding window holds the whole template prefix (the reference's
    # snapshot rule: every layer keeps exactly the prefix's rows).
    return pkg.Profile("engine", 128, 2, 4, 2, 32, 192, vocab=107520, window=64, pattern=2, max_position=512)


def write_checkpoint(pkg, path):
    rng = np.random.default_rng(7)
    tensors = {}
    for name, shape in pkg.schema(engine_profile(pkg)):
        x = rng.normal(0.0, 0.05, size=shape).astype(np.float32) + (1.0 if "norm" in name else 0.0)
        tensors[name] = (x.view(np.uint32) >> 16).astype(np.uint16)
    pkg.write_safetensors(path, tensors)


@pytest.fixture
def engine_files(tmp_path):
    pkg = load_package()
    pkg.load()
    libdir = os.path.dirname(pkg.LIB_PATH)
    src = tmp_path / "engine.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "engine"
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(src), "-L", libdir, "-lplamo_cuda", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    vocab = tmp_path / "tokenizer.jsonl"
    write_vocab(vocab)
    ckpt = tmp_path / "model.safetensors"
    write_checkpoint(pkg, ckpt)
    return exe, vocab, ckpt


def run(exe, vocab, ckpt, mode):
    r = subprocess.run([str(exe), str(vocab), str(ckpt), mode], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_tokenizer_only_engine_encodes_and_refuses_generation(engine_files):
    out = run(*engine_files, "tokenizer")
    assert "backend none memory tokenizer" in out
    prompt = [int(x) for x in re.search(r"prompt ((?:\d+ ?)+)", out).group(1).split()]
    pkg = load_package()
    with pkg.Tokenizer(str(engine_files[1])) as tok:
        assert prompt == tok.encode("Hello.", 1).tolist()
    assert "translate refused: engine: translation needs a loaded model" in out
    compute = json.loads(re.search(r"^compute (.*)$", out, re.M).group(1))
    assert compute["backend"] == "none" and compute["gpu_dispatches"] == 0


def cuda_device_present():
    pkg = load_package()
    lib = pkg.load()
    cfg = pkg._abi.CudaConfig(device=0)
    err = ctypes.create_string_buffer(256)
    ctx = lib.plamo_cuda_open(ctypes.byref(cfg), err, 256)
    if ctx:
        lib.plamo_cuda_close(ctx)
    return bool(ctx)


def test_full_open_without_device_fails_with_a_message(engine_files):
    if cuda_device_present():
        pytest.skip("a CUDA device is present")
    out = run(*engine_files, "full")
    assert "open failed: " in out and "CUDA" in out


def test_open_from_environment_needs_the_model_directory(monkeypatch):
    pkg = load_package()
    lib = pkg.load()
    monkeypatch.delenv("PLAMO_MODEL_DIR", raising=False)
    err = ctypes.create_string_buffer(256)
    info = ctypes.create_string_buffer(4096)
    lib.plamo_engine_open.restype = ctypes.c_void_p
    assert not lib.plamo_engine_open(0, 1, 1, 0, info, err, ctypes.c_size_t(256))
    assert b"PLAMO_MODEL_DIR" in err.value


def generate_reference(pkg, ckpt, ids, n):
    """plamo_cuda_generate over the same checkpoint and prompt ids."""
    cp = pkg.Checkpoint([str(ckpt)], engine_profile(pkg), full_capacity=512)
    be = pkg.Backend(device=0, max_context=512, max_prefill=4096)
    try:
        be.preload_model(cp.model)
        be.prepare(cp.model)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros(n, dtype=np.uint32)
        timing = pkg._abi.CudaTiming()
        k = be.lib.plamo_cuda_generate(be.ctx, cp.model.ptr, ids.ctypes.data, len(ids), n, out.ctypes.data,
                                       pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
        assert k >= 0, be.info().note
        return out[:k].tolist()
    finally:
        be.close()
        cp.close()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["full", "noprefix"])
def test_translate_streams_the_greedy_ids_of_the_device_loop(engine_files, mode):
    exe, vocab, ckpt = engine_files
    out = run(exe, vocab, ckpt, mode)
    assert "backend cuda memory resident" in out, out
    prompt = [int(x) for x in re.search(r"prompt ((?:\d+ ?)+)", out).group(1).split()]
    assert f"prefill {len(prompt)}" in out
    emitted = [int(x) for x in re.findall(r"^token (\d+)$", out, re.M)]
    done = re.search(r"finish (\w+) completion (\d+) cached (\d+) steps (\d+)", out)
    assert done, out
    assert int(done.group(2)) == len(emitted)
    prefix = [int(x) for x in re.search(r"prefix (\d+) (\d+)", out).groups()]
    if mode == "full":
        assert prefix[0] > 0 and int(done.group(3)) == prefix[0]
    else:
        assert prefix == [0, 0] and int(done.group(3)) == 0
    want = generate_reference(load_package(), ckpt, prompt, 12)
    assert emitted == want
    # The worker's telemetry for this request (reference runtime/worker.c:84-184 keys).
    report = json.loads(re.search(r"^report (.*)$", out, re.M).group(1))
    assert report["event"] == "done" and report["finish_reason"] == done.group(1)
    assert report["usage"]["prompt_tokens"] == len(prompt)
    assert report["usage"]["completion_tokens"] == len(emitted)
    assert report["usage"]["cached_prompt_tokens"] == int(done.group(3))
    assert report["timings"]["decode_steps"] == int(done.group(4))
    assert report["timings"]["prefill_gpu_seconds"] > 0
    compute = report["compute"]
    assert compute["backend"] == "cuda" and compute["gpu_dispatches"] > 0 and compute["errors"] == 0
    assert compute["fused_prefills"] >= 1 and compute["gpu_seconds"] > 0
    assert compute["decode_path"].startswith(("graph", "persistent"))
    assert compute["kv_pages_used"] > 0 and compute["kv_pages_allocated"] >= compute["kv_pages_used"]
    assert re.fullmatch(r"[0-9a-f]{16}", report["verification"]["logits_hash"])
