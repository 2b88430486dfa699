"""Writes the golden fixtures of tests/golden/ from the C oracle.

The oracle (oracle/) restates the reference's CPU token loop and is pinned by
the reference's own known-answer tests (tests/test_oracle_pins.py compiles
them against it). These fixtures freeze its outputs on seeded inputs so that
the pin travels without the reference checkout:

  gemv.npz        BF16 matvec (reference src/math.s:5-344) on the GEMV
                  benchmark's inputs (numpy default_rng(0): W ~ N(0, 0.02)
                  rounded to BF16, then x ~ N(0, 1)) at 4096x4096 and
                  14336x4096, plus two odd shapes; sha256 of every input.
  model_small.npz a 4-layer PLaMo-3 model (hidden 256, 4 query / 2 KV heads
                  of 64, sliding window 16 on every other layer, vocab 1000)
                  with the seeded synthetic weights of include/plamo_synthetic.h
                  (seed 11): prefill of 20 ids (default_rng(1) over [3, 1000)),
                  its logits and state, then 48 greedy tokens and their top-2
                  margins (reference src/prefill.s, src/forward.s,
                  src/token.s:37-63; stop ids 1 and 16 as runtime/engine.c).
  decode_fixture.npz
                  the two-layer model of reference tests/metal_decode.c:95-175
                  (LCG weights, seed 93; hidden 128, intermediate 257, dim 128,
                  global capacity 40, vocab 17): prefill of 6 ids, then 4
                  forward steps; state and logits after each call.

  model_8b.npz    (--large) BASELINE config 4 at its full size: profile 8b
                  with the seeded synthetic weights of seed 4 (the benchmark's
                  model), a 455-id prompt (default_rng(1) over [3, 100000)),
                  the state and logits after the prefill, then 64 greedy
                  tokens with the top-2 logit margin of every step.
  tp_31b_cut.npz  (--large) a two-layer cut of profile 31b (one sliding and
                  one full layer, tied head, seed 8): prefill of 20 ids
                  (default_rng(1) over [3, 100000)), then 32 greedy tokens and
                  their margins - the token check of the tensor-parallel
                  benchmark at every rank count.

Usage: python tests/golden/make_golden.py [--large]
(rewrites the three small .npz files; --large writes the two whole-model
fixtures instead, which streams 16 GB of weights per oracle token on the host
and takes several minutes with every host core).
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import synthetic  # noqa: E402
from conftest import load_oracle, load_package, rel_l2  # noqa: E402

GEMV_SHAPES = [(4096, 4096), (14336, 4096), (3, 7), (33, 1000)]
SMALL_SEED = 11
SMALL_PROMPT = 20
SMALL_TOKENS = 48
FIXTURE_IDS = [3, 7, 1, 12, 5, 9]
FIXTURE_STEPS = [4, 11, 2, 8]


def sha256(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def gemv_inputs(rows, cols, seed=0):
    rng = np.random.default_rng(seed)
    w = synthetic.bf16_round(rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32))
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    return np.ascontiguousarray(w), x


def oracle_matvec(w, x):
    rows, cols = w.shape
    y = np.zeros(max(rows, 1), dtype=np.float32)
    load_oracle().plamo_bf16_matvec(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols)
    return y[:rows]


def small_profile():
    pkg = load_package()
    return pkg.Profile("golden-small", 256, 4, 4, 2, 64, 512, vocab=1000, window=16, pattern=2,
                       max_position=512)


def small_host_model():
    """Host copy of the synthetic weights (the device generator makes the same bits)."""
    pkg = load_package()
    prof = small_profile()
    probe = pkg.HostModel(prof, weights="synthetic")
    blob = np.empty(probe.blob_bytes // 2, dtype=np.uint16)
    hm = pkg.HostModel(prof, weights=blob)
    synthetic.fill_model(hm, SMALL_SEED)
    return hm


def small_prompt():
    return np.random.default_rng(1).integers(3, 1000, size=SMALL_PROMPT).astype(np.uint32)


def oracle_prefill(hm, ids):
    states = np.zeros((len(ids), hm.profile.hidden), dtype=np.float32)
    ok = load_oracle().plamo_prefill(hm.ptr, ids.ctypes.data, len(ids), states.ctypes.data)
    assert ok == 1
    return states


def oracle_greedy(hm, max_tokens):
    """Greedy continuation after a prefill: the reference engine's loop."""
    o = load_oracle()
    out, margins = [], []
    while len(out) < max_tokens:
        logits = hm.logits_array()
        top = np.partition(logits, -2)[-2:]
        margins.append(float(top[1] - top[0]))
        t = int(o.plamo_argmax(hm.model.logits, hm.profile.vocab))
        if t in (1, 16):
            break
        out.append(t)
        if len(out) < max_tokens:
            assert o.plamo_forward(hm.ptr, t) == 1
    return np.array(out, dtype=np.uint32), np.array(margins, dtype=np.float32)


def make_gemv():
    fields = {}
    for rows, cols in GEMV_SHAPES:
        w, x = gemv_inputs(rows, cols)
        key = f"{rows}x{cols}"
        fields[f"y_{key}"] = oracle_matvec(w, x)
        fields[f"w_sha256_{key}"] = np.array(sha256(w))
        fields[f"x_sha256_{key}"] = np.array(sha256(x))
    return fields


def make_small():
    hm = small_host_model()
    ids = small_prompt()
    oracle_prefill(hm, ids)
    fields = {"ids": ids, "prefill_logits": hm.logits_array().copy(), "prefill_state": hm.state_array().copy(),
              "embed_sha256": np.array(sha256(hm.tensor("model.embed_tokens.weight")))}
    tokens, margins = oracle_greedy(hm, SMALL_TOKENS)
    fields["tokens"] = tokens
    fields["margins"] = margins
    return fields


def fixture_model():
    from fixtures import decode_fixture_pair
    _, b = decode_fixture_pair(128, 257, 128, 40)
    return b


def make_decode_fixture():
    hm = fixture_model()
    o = load_oracle()
    ids = np.array(FIXTURE_IDS, dtype=np.uint32)
    oracle_prefill(hm, ids)
    states, logits = [hm.state_array().copy()], [hm.logits_array().copy()]
    for t in FIXTURE_STEPS:
        assert o.plamo_forward(hm.ptr, t) == 1
        states.append(hm.state_array().copy())
        logits.append(hm.logits_array().copy())
    return {"ids": ids, "steps": np.array(FIXTURE_STEPS, dtype=np.uint32), "states": np.stack(states),
            "logits": np.stack(logits)}


LARGE_8B = dict(profile="8b", seed=4, prompt=455, tokens=64, prompt_seed=1, full_capacity=8208)
LARGE_31B_CUT = dict(profile="31b", seed=8, prompt=20, tokens=32, prompt_seed=1, full_capacity=1024, layers=2,
                     pattern=2)


def large_host_model(spec):
    """Host model of a profile with the device generator's synthetic weights
    (seed * 1000003 + tensor slot, the restatement in the oracle)."""
    from dataclasses import replace
    pkg = load_package()
    prof = pkg.PROFILES[spec["profile"]]
    if "layers" in spec:
        prof = replace(prof, name=f"{prof.name}-{spec['layers']}layers", layers=spec["layers"],
                       pattern=spec["pattern"])
    o = load_oracle()
    hm = pkg.HostModel(prof, weights=np.empty(pkg.HostModel(prof, weights="synthetic").blob_bytes // 2,
                                              dtype=np.uint16), full_capacity=spec["full_capacity"])
    threads = os.cpu_count() or 1
    for k, (addr, count, name) in enumerate(hm.tensor_ranges()):
        mean, std = pkg.synthetic_parameters(name)
        o.oracle_synthetic_bf16(addr, count, spec["seed"] * 1000003 + k, mean, std, threads)
    return hm


def make_large(spec):
    """The fixture, plus `order_spread_logits` / `order_spread_state`: the
    relative L2 distance between the reference-order prefill and the same
    prefill with an equally valid FP32 summation order (8 matvec lanes
    instead of 4). Across many layers and long prompts the model amplifies
    rounding differences; any implementation that does not replicate the
    reference's order bit for bit lands at about this distance, so the GPU
    tests hold whole-model prefill outputs to a multiple of it."""
    o = load_oracle()
    o.oracle_set_threads(os.cpu_count() or 1)
    hm = large_host_model(spec)
    ids = np.random.default_rng(spec["prompt_seed"]).integers(3, 100000, size=spec["prompt"]).astype(np.uint32)
    o.oracle_set_matvec_lanes(8)
    try:
        oracle_prefill(hm, ids)
        other_logits, other_state = hm.logits_array().copy(), hm.state_array().copy()
    finally:
        o.oracle_set_matvec_lanes(4)
    hm.reset()
    oracle_prefill(hm, ids)
    fields = {"ids": ids, "prefill_logits": hm.logits_array().copy(), "prefill_state": hm.state_array().copy(),
              "profile": np.array(hm.profile.name), "seed": np.array(spec["seed"]),
              "embed_sha256": np.array(sha256(hm.tensor("model.embed_tokens.weight")))}
    fields["order_spread_logits"] = np.array(rel_l2(other_logits, fields["prefill_logits"]))
    fields["order_spread_state"] = np.array(rel_l2(other_state, fields["prefill_state"]))
    tokens, margins = oracle_greedy(hm, spec["tokens"])
    fields["tokens"] = tokens
    fields["margins"] = margins
    return fields


def main():
    if "--large" in sys.argv[1:]:
        for name, spec in (("tp_31b_cut", LARGE_31B_CUT), ("model_8b", LARGE_8B)):
            path = os.path.join(HERE, f"{name}.npz")
            np.savez_compressed(path, **make_large(spec))
            print(f"wrote {path} ({os.path.getsize(path)} bytes)", flush=True)
        return
    load_oracle().oracle_set_threads(1)
    for name, make in (("gemv", make_gemv), ("model_small", make_small), ("decode_fixture", make_decode_fixture)):
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **make())
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
