#!/usr/bin/env python3
"""Benchmark of the PLaMo-3 token loop on B200.

Metric: batch-1 greedy decode tok/s of the 8B-shaped model
(profile 8b: hidden 4096, 32 layers, 32/4 heads x 128, intermediate 16384,
vocab 107520) after a 455-token prompt, with the fraction of the HBM roofline;
prefill tok/s; and aggregate tok/s of data-parallel replicas at N GPUs.

One step = one decode token through every layer (one CUDA-graph launch).
Weights are seeded synthetic BF16 (N(0, 0.02) stand-in, norms 1.0) generated
in HBM; every step streams 16.2 GB of weights, far above the 126 MB L2, so no
L2 flush is needed between steps. At N > 1 every rank runs an independent
replica (own prompt) with no collective on the data path; rank 0 prints the
aggregate (N x steps / max-over-ranks device time).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload 8b-decode|31b-tp]

At N > 1 the line also carries "tp": BASELINE config 5 at that rank count
(the 31B-shaped tensor-parallel decode and its speculative form), the
oracle token check of a 31B-shaped two-layer cut sharded the same way, and
the latency of an NCCL all-reduce of one exchange's vector for comparison
(--no-tp skips it).

--workload 31b-tp: the 31B-shaped model (profile 31b,
tied head) tensor-parallel over the N ranks of the launch (N = 1: one GPU, no
tensor parallelism): a 128-token prompt, then batch-1 greedy decode of one
token stream (strong scaling: the work per token is fixed, N GPUs share it);
also the same request through the speculative loop with a 0.8B-shaped draft
proposing 4 tokens per verification.
"""
import argparse
import ctypes
import datetime
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "plamo-3-translate.c_b200")
ORACLE = os.path.join(ROOT, "oracle", "liboracle.so")
PROMPT = 455
METRIC = "bs1 decode tok/s (8B-shaped)"
BATCH = 8  # independent requests per GPU in the multi-request measurement
TP_PROMPT = 128
TP_METRIC = "bs1 decode tok/s (31B-shaped, tensor-parallel)"


def load_package():
    spec = importlib.util.spec_from_file_location(
        "plamo_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["plamo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_traffic():
    """ncu-measured DRAM traffic (profiles/traffic.json; commands in
    profiles/dram_traffic_decode.md), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f)


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    return 6650.0, "fallback (6.65 TB/s, earlier measurement on this pool)"


def tensor_peak():
    """Dense BF16 peak for a kernel timed inside a long step (the sustained
    cuBLAS loop under the power cap), else the pool's earlier measurement."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        if "bf16_tflops_sustained" in p:
            return float(p["bf16_tflops_sustained"]), "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
    return 1400.0, "fallback (1.4 PFLOP/s sustained, earlier measurement on this pool)"


def prefill_flops(profile, tokens):
    """Algorithmic FLOP of a layer-major prefill of `tokens` prompt ids: every
    projection for every token, causal attention (QK^T and PV over the keys a
    query sees, all query heads) and the head for the last token only."""
    h = profile.hidden
    per_token = profile.qkv_rows * h + h * profile.attention_width + 3 * profile.inter * h
    flops = 2.0 * tokens * profile.layers * per_token + 2.0 * profile.vocab * h
    for layer in range(profile.layers):
        span = tokens if profile.full(layer) else profile.window
        keys = sum(min(t + 1, span) for t in range(tokens))
        flops += 4.0 * profile.qh * profile.dim * keys
    return flops


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.first = threading.Event()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        # A short timed region must not end before the first sample: wait for it
        # (bounded) so every measurement carries at least one clock reading.
        self.first.wait(timeout=10)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)
            self.first.set()
        self.first.set()

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.reader.join(timeout=5)
        return self.summarise(self.lines, self.gpu)

    @staticmethod
    def summarise(lines, gpu):
        """Median SM clock, max clock and the throttle reasons seen Active in
        `nvidia-smi --format=csv,noheader,nounits` lines of FIELDS for one GPU."""
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) != gpu:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sms)) if sms else None,
                "sm_max_mhz": max(maxes) if maxes else None, "samples": len(sms),
                "reasons": sorted(reasons)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local, dist


def reduce_max(dist, value):
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


def oracle_lib():
    if not os.path.exists(ORACLE):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True,
                       capture_output=True)
    lib = ctypes.CDLL(ORACLE)
    P, U64 = ctypes.c_void_p, ctypes.c_uint64
    lib.plamo_forward.restype, lib.plamo_forward.argtypes = ctypes.c_int, [P, U64]
    lib.plamo_prefill.restype, lib.plamo_prefill.argtypes = ctypes.c_int, [P, P, U64, P]
    lib.plamo_argmax.restype, lib.plamo_argmax.argtypes = U64, [P, U64]
    lib.oracle_set_threads.argtypes = [ctypes.c_int]
    lib.oracle_synthetic_bf16.argtypes = [P, U64, U64, ctypes.c_float, ctypes.c_float, ctypes.c_int]
    return lib


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def gemv_cpu_baseline(rows=4096, cols=4096, threads=(1, 8), seconds=0.5):
    """GEMV benchmark case 1 on the host cores: the oracle's matvec (the
    reference CPU accumulation order, rows split across threads) on W ~ N(0,
    0.02) rounded to BF16 and x ~ N(0, 1) from default_rng(0); GB/s of
    algorithmic bytes (2*rows*cols + 4*cols + 4*rows) per thread count."""
    lib = oracle_lib()
    P, U64 = ctypes.c_void_p, ctypes.c_uint64
    lib.plamo_bf16_matvec.restype, lib.plamo_bf16_matvec.argtypes = None, [P, P, P, U64, U64]
    rng = np.random.default_rng(0)
    bits = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32).view(np.uint32).astype(np.uint64)
    w = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    y = np.zeros(rows, dtype=np.float32)
    algorithmic = 2 * rows * cols + 4 * cols + 4 * rows
    out = {}
    for t in threads:
        lib.oracle_set_threads(int(t))
        lib.plamo_bf16_matvec(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols)
        calls, t0 = 0, time.perf_counter()
        while True:
            lib.plamo_bf16_matvec(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols)
            calls += 1
            elapsed = time.perf_counter() - t0
            if elapsed >= seconds:
                break
        out[f"threads_{t}"] = algorithmic * calls / elapsed / 1e9
    lib.oracle_set_threads(1)
    return {"unit": "GB/s", "shape": f"{rows}x{cols}", "kind": "port", **out}


def oracle_decode_rate(pkg, hm, tokens, prompt_tokens, threads):
    """C oracle (restatement of the reference CPU path) decode tok/s on `hm`."""
    lib = oracle_lib()
    lib.oracle_set_threads(threads)
    ids = np.random.default_rng(1).integers(3, 100000, size=prompt_tokens).astype(np.uint32)
    states = np.zeros((prompt_tokens, hm.profile.hidden), dtype=np.float32)
    assert lib.plamo_prefill(hm.ptr, ids.ctypes.data, prompt_tokens, states.ctypes.data) == 1
    tok = int(lib.plamo_argmax(hm.model.logits, hm.profile.vocab))
    t0 = time.perf_counter()
    for _ in range(tokens):
        assert lib.plamo_forward(hm.ptr, tok) == 1
        tok = int(lib.plamo_argmax(hm.model.logits, hm.profile.vocab))
    return tokens / (time.perf_counter() - t0)


def host_model_for_oracle(pkg, profile, seed, threads):
    """Weights generated on the host by the oracle's copy of the generator."""
    lib = oracle_lib()
    hm = pkg.HostModel(profile, full_capacity=8208)
    for k, (addr, count, name) in enumerate(hm.tensor_ranges()):
        mean, std = pkg.synthetic_parameters(name)
        lib.oracle_synthetic_bf16(addr, count, seed * 1000003 + k, mean, std, threads)
    return hm


def run_reference(args, world, rank):
    """The reference arm: the reference CPU path of this loop (its C oracle
    restatement; the AArch64/Darwin original cannot run on this host) timed on
    the host cores, same metric and workload."""
    if rank != 0:
        return
    pkg = load_package()
    threads = host_threads()
    profile = pkg.PROFILES["8b"]
    hm = host_model_for_oracle(pkg, profile, seed=4, threads=threads)
    sample_prompt = 4
    lib = oracle_lib()
    lib.oracle_set_threads(threads)
    ids = np.random.default_rng(1).integers(3, 100000, size=sample_prompt).astype(np.uint32)
    states = np.zeros((sample_prompt, profile.hidden), dtype=np.float32)
    assert lib.plamo_prefill(hm.ptr, ids.ctypes.data, sample_prompt, states.ctypes.data) == 1
    tok = int(lib.plamo_argmax(hm.model.logits, profile.vocab))
    for _ in range(args.warmup):
        assert lib.plamo_forward(hm.ptr, tok) == 1
        tok = int(lib.plamo_argmax(hm.model.logits, profile.vocab))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        assert lib.plamo_forward(hm.ptr, tok) == 1
        tok = int(lib.plamo_argmax(hm.model.logits, profile.vocab))
    seconds = time.perf_counter() - t0
    value = args.steps / seconds
    sample = (f"8B-shaped decode, {args.steps} tokens after a {sample_prompt}-token prompt "
              f"(+{args.warmup} warm-up); KV context {sample_prompt + args.warmup}.."
              f"{sample_prompt + args.warmup + args.steps} instead of 455..519 (KV is <0.5% of "
              "the bytes per token)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * seconds / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": sample_config(world, sample_prompt),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("reference CPU path = C restatement of the reference's AArch64 assembly "
                 "(oracle/); the original is Darwin/AArch64 and cannot run on this x86 host"),
    }
    print(json.dumps(line), flush=True)


def workload_config(world):
    return {"workload": "8b-decode: plamo-3 profile 8b, 455-token prompt then greedy decode, batch 1",
            "model": "plamo-3-8b-shaped (random init)", "global_batch": world, "seq_len": PROMPT,
            "parallelism": f"dp{world} (independent replicas)",
            "l2": "inputs larger than L2 (16.2 GB of weights streamed per step)"}


def sample_config(world, prompt):
    """Config of the host-core sample: the same model and decode step after a
    `prompt`-token prompt (the 455-token prefill alone would take minutes on
    the host; the KV rows read per token are < 0.5 % of its bytes)."""
    cfg = workload_config(world)
    cfg.update({"workload": f"8b-decode sample: plamo-3 profile 8b, {prompt}-token prompt then greedy decode, "
                            "batch 1", "seq_len": prompt, "parallelism": "host cores (one replica)"})
    return cfg


def run_ours(args, world, rank, local, dist):
    pkg = load_package()
    lib = pkg.load()
    profile = pkg.PROFILES["8b"]
    be = pkg.Backend(device=local, max_context=8192 + 16, max_prefill=4096)
    ctx = be.ctx
    hm = pkg.HostModel(profile, weights="synthetic", full_capacity=8208)
    be.preload_synthetic(hm, seed=4)
    be.prepare(hm)
    ids = np.random.default_rng(1 + rank).integers(3, 100000, size=PROMPT).astype(np.uint32)

    # Prefill (timed on the device; second run after a warm-up run).
    nxt = ctypes.c_uint32()
    prefill_s = None
    for _ in range(2):
        lib.plamo_cuda_reset_request(ctx, hm.ptr)
        before = be.info().gpu_seconds
        assert lib.plamo_cuda_prefill_greedy(ctx, hm.ptr, ids.ctypes.data, PROMPT,
                                             ctypes.byref(nxt)) == 1, be.info().note
        prefill_s = be.info().gpu_seconds - before
    prefill_rate = world * PROMPT / reduce_max(dist, prefill_s)

    # Decode: warm-up, then exactly K steps between barriers.
    decode_path = (lib.plamo_cuda_decode_path(ctx, hm.ptr) or b"?").decode()
    assert lib.plamo_cuda_time_decode(ctx, hm.ptr, args.warmup) > 0, be.info().note
    barrier(dist)
    lib.plamo_cuda_synchronize(ctx)
    clocks = ClockSampler(local)
    launches0 = lib.plamo_cuda_kernel_launches(ctx)
    ms = lib.plamo_cuda_time_decode(ctx, hm.ptr, args.steps)
    launches = lib.plamo_cuda_kernel_launches(ctx) - launches0
    clock_info = clocks.stop()
    assert ms > 0, be.info().note
    lib.plamo_cuda_synchronize(ctx)
    barrier(dist)
    ms_max = reduce_max(dist, ms)
    ms_per_step = ms_max / args.steps
    value = world * args.steps / (ms_max / 1000.0)

    # Algorithmic bytes of one step: weights, norms, one embedding row, and
    # the K/V rows read by attention at the mean context of the timed steps.
    ctx_mean = PROMPT + args.warmup + (args.steps + 1) / 2.0
    kv_bytes = profile.layers * ctx_mean * profile.kh * profile.dim * 4 * 2
    step_bytes = (profile.weight_bytes_per_token() + profile.norm_bytes_per_token() +
                  2 * profile.hidden + kv_bytes)
    peak, peak_src = measured_peaks()
    achieved = step_bytes / (ms_per_step / 1000.0) / 1e9

    # Standalone projection kernel at the largest layer shape (gate_up,
    # 32768 x 4096, 268 MB > L2): CUDA events around back-to-back launches.
    rows, cols = 2 * profile.inter, profile.hidden
    dw = lib.plamo_cuda_device_alloc(ctx, rows * cols * 2)
    dx = lib.plamo_cuda_device_alloc(ctx, cols * 4)
    dy = lib.plamo_cuda_device_alloc(ctx, rows * 4)
    lib.plamo_cuda_fill_synthetic_bf16(ctx, dw, rows * cols, 99, 0.0, 0.02)
    lib.plamo_cuda_fill_synthetic_f32(ctx, dx, cols, 98, 0.0, 1.0)
    lib.plamo_cuda_time_gemv(ctx, dw, dx, dy, rows, cols, 5)
    gemv_ms = lib.plamo_cuda_time_gemv(ctx, dw, dx, dy, rows, cols, 50) / 50
    gemv_bytes = rows * cols * 2 + cols * 4 + rows * 4
    for p in (dw, dx, dy):
        lib.plamo_cuda_device_free(ctx, p)

    # End to end through the public request API: host ids in, each token's
    # id back on the host (pinned H2D of the token, D2H of the next id).
    lib.plamo_cuda_reset_request(ctx, hm.ptr)
    out = np.zeros(args.steps + 1, dtype=np.uint32)
    timing = pkg._abi.CudaTiming()
    barrier(dist)
    n = lib.plamo_cuda_generate(ctx, hm.ptr, ids.ctypes.data, PROMPT, args.steps + 1,
                                out.ctypes.data, pkg._abi.TOKEN_CALLBACK(), None,
                                ctypes.byref(timing))
    assert n > 0, be.info().note
    steps_e2e = max(int(timing.decode_steps), 1)
    e2e_s = reduce_max(dist, timing.decode_seconds / steps_e2e)
    e2e_value = world / e2e_s

    batch_info = run_batch(args, pkg, lib, be, hm, profile, world, rank, dist, peak)
    config1 = gemv_configs(lib, ctx, peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        blob = np.empty(hm.blob_bytes // 2, dtype=np.uint16)
        host = pkg.HostModel(profile, weights=blob, full_capacity=8208)
        for (ka, count, _), (kb, _, _) in zip(hm.tensor_ranges(), host.tensor_ranges()):
            assert lib.plamo_cuda_read_weights(ctx, ka, kb, 2 * count) == 1
        tokens, prompt = 3, 4
        rate = oracle_decode_rate(pkg, host, tokens, prompt, threads)
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"8B-shaped decode, {tokens} tokens after a {prompt}-token prompt "
                         "(same weights; C restatement of the reference CPU path, row-split "
                         "threads)", "config": sample_config(1, prompt),
               "gemv": gemv_cpu_baseline()}
        del host, blob

    line = None
    if rank == 0:
        traffic = measured_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload_config(world),
            "prefill_tok_s": prefill_rate,
            "prefill_roofline": prefill_roofline(profile, prefill_rate / world),
            "decode_path": decode_path,
            "roofline": {"bound": "hbm",
                         "kernel": ("decode_token_kernel (one persistent launch per token)"
                                    if decode_path == "persistent" else
                                    "decode step (one CUDA graph launch per token)"),
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": (step_bytes * traffic["decode_step_ratio"]["ratio"]) if traffic else None,
                         "traffic_source": ("ncu DRAM bytes of a 2B decode step, traffic/algorithmic ratio "
                                            "applied to this step") if traffic else None,
                         "algorithmic_bytes": step_bytes, "peak_source": peak_src},
            "gemv_roofline": {"bound": "hbm", "kernel": "gemv 32768x4096 bf16 (gate_up shape)",
                              "achieved": gemv_bytes / (gemv_ms / 1000) / 1e9, "peak": peak,
                              "unit": "GB/s", "frac": gemv_bytes / (gemv_ms / 1000) / 1e9 / peak,
                              "traffic": (traffic["gemv_gate_up_8b"]["dram_read"] +
                                          traffic["gemv_gate_up_8b"]["dram_write"]) if traffic else None,
                              "ms": gemv_ms},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4, "api": "plamo_cuda_generate (per-token host round trip)"},
            "gpu_launches": int(launches),
            "clocks": clock_info,
            "cpu_baseline": cpu,
            "batch": batch_info,
            "config1_gemv": config1,
        }
    be.close()
    if rank == 0 and world == 1:
        line["config3_2b_decode"] = decode_2b(args, pkg, local, peak)
        line["config2_layer"] = layer_config2(pkg, local, peak)
    return line if rank == 0 else None


def prefill_roofline(profile, rate):
    """Per-GPU prefill of the PROMPT-id prompt against the sustained tensor peak."""
    tflops = prefill_flops(profile, PROMPT) * rate / PROMPT / 1e12
    peak, src = tensor_peak()
    return {"bound": "tensor", "kernel": "layer-major prefill (tcgen05 projections, prompt attention)",
            "achieved": tflops, "peak": peak, "unit": "TFLOP/s", "frac": tflops / peak,
            "algorithmic_flops": prefill_flops(profile, PROMPT), "peak_source": src}


def gemv_configs(lib, ctx, peak):
    """BASELINE config 1 on the GPU: the single BF16 GEMV at 4096 x 4096 and its
    8-row-block variant 14336 x 4096 (synthetic N(0, 0.02)-like weights, x
    N(0, 1)). Both matrices fit in the 126 MB L2, so consecutive launches
    rotate through enough copies (> 400 MB) that each streams its weights from
    HBM; CUDA-event time over 200 launches, algorithmic bytes."""
    out = {}
    for rows, cols in ((4096, 4096), (14336, 4096)):
        copies = -(-400_000_000 // (2 * rows * cols))
        dw = lib.plamo_cuda_device_alloc(ctx, copies * rows * cols * 2)
        dx = lib.plamo_cuda_device_alloc(ctx, cols * 4)
        dy = lib.plamo_cuda_device_alloc(ctx, rows * 4)
        lib.plamo_cuda_fill_synthetic_bf16(ctx, dw, copies * rows * cols, 7, 0.0, 0.02)
        lib.plamo_cuda_fill_synthetic_f32(ctx, dx, cols, 6, 0.0, 1.0)
        lib.plamo_cuda_time_gemv_copies(ctx, dw, copies, dx, dy, rows, cols, 2 * copies)
        ms = lib.plamo_cuda_time_gemv_copies(ctx, dw, copies, dx, dy, rows, cols, 200) / 200
        for q in (dw, dx, dy):
            lib.plamo_cuda_device_free(ctx, q)
        nbytes = 2 * rows * cols + 4 * cols + 4 * rows
        gbs = nbytes / (ms / 1000) / 1e9
        out[f"{rows}x{cols}"] = {"us": ms * 1000, "GB_s": gbs, "frac": gbs / peak, "copies_rotated": copies,
                                 "algorithmic_bytes": nbytes}
    return out


def decode_2b(args, pkg, local, peak):
    """BASELINE config 3 on the GPU: the 2B profile, 81-id prompt
    (default_rng(1)), batch-1 greedy decode; tok/s and the HBM roofline."""
    lib = pkg.load()
    profile = pkg.PROFILES["2b"]
    be = pkg.Backend(device=local, max_context=8192 + 16, max_prefill=4096)
    try:
        hm = pkg.HostModel(profile, weights="synthetic", full_capacity=8208)
        be.preload_synthetic(hm, seed=3)
        be.prepare(hm)
        ids = np.random.default_rng(1).integers(3, 100000, size=81).astype(np.uint32)
        nxt = ctypes.c_uint32()
        assert lib.plamo_cuda_prefill_greedy(be.ctx, hm.ptr, ids.ctypes.data, 81, ctypes.byref(nxt)) == 1
        assert lib.plamo_cuda_time_decode(be.ctx, hm.ptr, 3) > 0, be.info().note
        steps = 60
        ms = lib.plamo_cuda_time_decode(be.ctx, hm.ptr, steps)
        assert ms > 0, be.info().note
        ctx_mean = 81 + 3 + (steps + 1) / 2.0
        step_bytes = (profile.weight_bytes_per_token() + profile.norm_bytes_per_token() + 2 * profile.hidden +
                      profile.layers * ctx_mean * profile.kh * profile.dim * 4 * 2)
        gbs = step_bytes / (ms / steps / 1000) / 1e9
        return {"value": steps / (ms / 1000), "unit": "tok/s", "ms_per_step": ms / steps, "steps": steps,
                "roofline": {"achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                             "algorithmic_bytes": step_bytes}}
    finally:
        be.close()


def layer_config2(pkg, local, peak):
    """BASELINE config 2 on the GPU: one decoder layer at hidden 2048 (Q 16 x
    128, K/V 4 x 128, SwiGLU 8192, BF16 weights N(0, 0.02) generated in HBM,
    norm weights 1.0: the time does not depend on their values), one decode
    step over 511 cached rows of FP32 N(0, 1) keys and
    values, through plamo_cuda_layer (the reference's plamo_metal_layer
    entry). Device time per step from the entry's own events
    (plamo_cuda_info.gpu_seconds), e2e per call with the state's host copies;
    each step appends one row, so the context grows from 511 to 511 + steps."""
    lib = pkg.load()
    prof = pkg.Profile("config2", 2048, 1, 16, 4, 128, 8192, vocab=16, window=2048, pattern=1,
                       max_position=1024)
    specs = [pkg.LayerSpec(False, 1024, pkg.rope_frequencies(1e4, 64), 1.0)]
    be = pkg.Backend(device=local, max_context=1024, max_prefill=64)
    try:
        hm = pkg.HostModel(prof, specs, weights="synthetic")
        be.preload_synthetic(hm, seed=2)
        rng = np.random.default_rng(0)
        cached, kvw = 511, 4 * 128
        c = hm.caches[0]
        hm.view(c.k, cached * kvw)[:] = rng.normal(0, 1, size=cached * kvw).astype(np.float32)
        hm.view(c.v, cached * kvw)[:] = rng.normal(0, 1, size=cached * kvw).astype(np.float32)
        c.count = cached
        be.prepare(hm)
        state = rng.normal(0, 1, size=2048).astype(np.float32)
        buf = state.copy()
        for _ in range(3):
            buf[:] = state
            assert lib.plamo_cuda_layer(be.ctx, hm.ptr, 0, buf.ctypes.data) == 1, be.info().note
        steps = 200
        g0, t0 = be.info().gpu_seconds, time.perf_counter()
        for _ in range(steps):
            buf[:] = state
            assert lib.plamo_cuda_layer(be.ctx, hm.ptr, 0, buf.ctypes.data) == 1, be.info().note
        wall = (time.perf_counter() - t0) / steps
        dev = (be.info().gpu_seconds - g0) / steps
        weights = 2 * (prof.hidden * (prof.qh + 2 * prof.kh) * prof.dim + prof.hidden * prof.qh * prof.dim +
                       2 * prof.inter * prof.hidden + prof.hidden * prof.inter)
        ctx_mean = cached + 3 + (steps + 1) / 2.0
        step_bytes = weights + ctx_mean * kvw * 4 * 2
        gbs = step_bytes / dev / 1e9
        return {"workload": "config 2: one decoder layer, hidden 2048, 511 cached rows, plamo_cuda_layer",
                "us_per_step": dev * 1e6, "steps": steps,
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                             "algorithmic_bytes": step_bytes},
                "e2e": {"us_per_call": wall * 1e6, "h2d_bytes_per_step": 2048 * 4, "d2h_bytes_per_step": 2048 * 4}}
    finally:
        be.close()


def run_batch(args, pkg, lib, be, hm, profile, world, rank, dist, peak):
    """BASELINE config 4's second form: 8 independent requests per GPU (each its
    own 455-token prompt and KV cache) decoded together, one pass over the
    weights per step (plamo_cuda_batch_*). Aggregate tok/s over all ranks."""
    ctx = be.ctx
    reqs = [hm] + [pkg.HostModel(profile, weights_of=hm, full_capacity=8208) for _ in range(BATCH - 1)]
    for r in reqs[1:]:
        be.prepare(r)
    toks = np.zeros(BATCH, dtype=np.uint32)
    nxt = ctypes.c_uint32()
    for i, r in enumerate(reqs):
        lib.plamo_cuda_reset_request(ctx, r.ptr)
        ids = np.random.default_rng(1000 + rank * BATCH + i).integers(3, 100000, size=PROMPT).astype(np.uint32)
        assert lib.plamo_cuda_prefill_greedy(ctx, r.ptr, ids.ctypes.data, PROMPT, ctypes.byref(nxt)) == 1, \
            be.info().note
        toks[i] = nxt.value
    arr = (ctypes.c_void_p * BATCH)(*[ctypes.addressof(r.model) for r in reqs])
    batch = lib.plamo_cuda_batch_open(ctx, arr, BATCH)
    assert batch, be.info().note
    try:
        out = np.zeros(BATCH, dtype=np.uint32)
        assert lib.plamo_cuda_batch_step(batch, toks.ctypes.data, out.ctypes.data) == 1, be.info().note
        assert lib.plamo_cuda_time_batch(batch, args.warmup) > 0, be.info().note
        barrier(dist)
        ms = lib.plamo_cuda_time_batch(batch, args.steps)
        assert ms > 0, be.info().note
        barrier(dist)
        ms_max = reduce_max(dist, ms)
        ms_step = ms_max / args.steps
        value = world * BATCH * args.steps / (ms_max / 1000.0)
        ctx_mean = PROMPT + 1 + args.warmup + (args.steps + 1) / 2.0
        kv = BATCH * profile.layers * ctx_mean * profile.kh * profile.dim * 4 * 2
        step_bytes = (profile.weight_bytes_per_token() + profile.norm_bytes_per_token() +
                      BATCH * 2 * profile.hidden + kv)
        achieved = step_bytes / (ms_step / 1000.0) / 1e9
        # End to end through the public step call: host tokens in, host tokens out.
        tokens = out.copy()
        barrier(dist)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            assert lib.plamo_cuda_batch_step(batch, tokens.ctypes.data, out.ctypes.data) == 1, be.info().note
            tokens = out.copy()
        e2e_s = reduce_max(dist, (time.perf_counter() - t0) / args.steps)
    finally:
        lib.plamo_cuda_batch_close(batch)
    for r in reqs[1:]:
        lib.plamo_cuda_release_model(ctx, r.ptr)
    return {"requests_per_gpu": BATCH, "value": value, "unit": "tok/s", "ms_per_step": ms_step,
            "roofline": {"bound": "hbm", "kernel": "batched decode step (one CUDA graph per step)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "algorithmic_bytes": step_bytes},
            "e2e": {"value": world * BATCH / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * BATCH,
                    "d2h_bytes_per_step": 4 * BATCH, "api": "plamo_cuda_batch_step (host wall clock per step)"}}


def shard_bytes_per_token(full, shard, vocab_rows, ctx_mean):
    """Bytes one rank streams per decode token: its projections, its head
    slice, the replicated norms and embedding row, and its K/V rows."""
    h = full.hidden
    per_layer = shard.qkv_rows * h + h * shard.attention_width + 3 * shard.inter * h
    weights = 2 * (full.layers * per_layer + vocab_rows * h)
    kv = full.layers * ctx_mean * shard.kh * shard.dim * 4 * 2
    return weights + full.norm_bytes_per_token() + 2 * h + kv


def tp_cut_check(world, rank, local, dist):
    """Token check of the tensor-parallel path: the two-layer cut of the 31B
    profile sharded over the ranks of this launch, its prefill and greedy
    tokens against the oracle's (tests/golden/tp_31b_cut.npz, written by
    tests/golden/make_golden.py --large)."""
    from dataclasses import replace
    pkg = load_package()
    lib = pkg.load()
    g = np.load(os.path.join(ROOT, "tests", "golden", "tp_31b_cut.npz"))
    full = replace(pkg.PROFILES["31b"], name="31b-2layers", layers=2, pattern=2)
    shard = pkg.tp_shard_profile(full, world)
    be = pkg.Backend(device=local, max_context=1024, max_prefill=256)
    try:
        hm = pkg.HostModel(shard, weights="synthetic", full_capacity=1024)
        be.preload_synthetic_tp(hm, full, rank, world, seed=int(g["seed"]))
        be.tp_connect(hm, pkg.tp_all_gather_handles(be.tp_prepare(hm, rank, world)))
        ids = np.ascontiguousarray(g["ids"], dtype=np.uint32)
        n_want = len(g["tokens"])
        out = np.zeros(n_want, dtype=np.uint32)
        timing = pkg._abi.CudaTiming()
        barrier(dist)
        n = lib.plamo_cuda_generate(be.ctx, hm.ptr, ids.ctypes.data, len(ids), n_want, out.ctypes.data,
                                    pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
        assert n > 0, be.info().note
        got = out[:n].tolist()
        equal = got == g["tokens"].tolist()
        equal_all = reduce_max(dist, 0.0 if equal else 1.0) == 0.0
        barrier(dist)
    finally:
        be.close()
    return {"model": "31b profile, 2 layers (sliding + full), tied head", "prompt": len(ids), "tokens": n_want,
            "tokens_equal_oracle": bool(equal_all), "oracle_fixture": "tests/golden/tp_31b_cut.npz"}


def nccl_allreduce_latency(dist, hidden, iters=200):
    """Device time of one NCCL all-reduce of a [hidden] FP32 vector (the size
    of one tensor-parallel exchange), mean over `iters` back-to-back calls,
    max over ranks."""
    import torch
    x = torch.ones(hidden, dtype=torch.float32, device="cuda")
    for _ in range(20):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        dist.all_reduce(x)
    end.record()
    torch.cuda.synchronize()
    return reduce_max(dist, start.elapsed_time(end) / iters * 1000.0)


def run_tp31b(args, world, rank, local, dist):
    line = measure_tp31b(args, world, rank, local, dist)
    if rank == 0:
        print(json.dumps(line), flush=True)


def measure_tp31b(args, world, rank, local, dist):
    pkg = load_package()
    lib = pkg.load()
    full = pkg.PROFILES["31b"]
    shard = pkg.tp_shard_profile(full, world) if world > 1 else full
    cap = 1024
    be = pkg.Backend(device=local, max_context=cap, max_prefill=256)
    ctx = be.ctx
    hm = pkg.HostModel(shard, weights="synthetic", full_capacity=cap)
    if world > 1:
        be.preload_synthetic_tp(hm, full, rank, world, seed=5)
        be.tp_connect(hm, pkg.tp_all_gather_handles(be.tp_prepare(hm, rank, world)))
        vocab_rows = pkg.tp_vocab_slice(full.vocab, world, rank)[1]
    else:
        be.preload_synthetic(hm, seed=5)
        be.prepare(hm)
        vocab_rows = full.vocab
    ids = np.random.default_rng(1).integers(3, 100000, size=TP_PROMPT).astype(np.uint32)
    nxt = ctypes.c_uint32()
    prefill_s = None
    for _ in range(2):
        lib.plamo_cuda_reset_request(ctx, hm.ptr)
        before = be.info().gpu_seconds
        assert lib.plamo_cuda_prefill_greedy(ctx, hm.ptr, ids.ctypes.data, TP_PROMPT,
                                             ctypes.byref(nxt)) == 1, be.info().note
        prefill_s = be.info().gpu_seconds - before
    prefill_rate = TP_PROMPT / reduce_max(dist, prefill_s)

    assert lib.plamo_cuda_time_decode(ctx, hm.ptr, args.warmup) > 0, be.info().note
    barrier(dist)
    lib.plamo_cuda_synchronize(ctx)
    clocks = ClockSampler(local)
    launches0 = lib.plamo_cuda_kernel_launches(ctx)
    ms = lib.plamo_cuda_time_decode(ctx, hm.ptr, args.steps)
    launches = lib.plamo_cuda_kernel_launches(ctx) - launches0
    clock_info = clocks.stop()
    assert ms > 0, be.info().note
    lib.plamo_cuda_synchronize(ctx)
    barrier(dist)
    ms_max = reduce_max(dist, ms)
    ms_per_step = ms_max / args.steps
    value = args.steps / (ms_max / 1000.0)
    ctx_mean = TP_PROMPT + args.warmup + (args.steps + 1) / 2.0
    rank_bytes = shard_bytes_per_token(full, shard, vocab_rows, ctx_mean)
    peak, peak_src = measured_peaks()
    achieved = rank_bytes / (ms_per_step / 1000.0) / 1e9

    # End to end through the request API on every rank (same ids, same tokens).
    out = np.zeros(args.steps + 1, dtype=np.uint32)
    timing = pkg._abi.CudaTiming()
    barrier(dist)
    n = lib.plamo_cuda_generate(ctx, hm.ptr, ids.ctypes.data, TP_PROMPT, args.steps + 1, out.ctypes.data,
                                pkg._abi.TOKEN_CALLBACK(), None, ctypes.byref(timing))
    assert n > 0, be.info().note
    e2e_value = 1.0 / reduce_max(dist, timing.decode_seconds / max(int(timing.decode_steps), 1))

    # Speculative: 0.8B-shaped draft (replicated on every rank), 4 proposals
    # per verification of the tensor-parallel target.
    draft_profile = pkg.PROFILES["0.8b"]
    draft = pkg.HostModel(draft_profile, weights="synthetic", full_capacity=cap)
    be.preload_synthetic(draft, seed=6)
    be.prepare(draft)
    spec_out = np.zeros(args.steps + 1, dtype=np.uint32)
    stats = pkg._abi.CudaSpeculation()
    barrier(dist)
    k = lib.plamo_cuda_generate_speculative(ctx, hm.ptr, draft.ptr, ids.ctypes.data, TP_PROMPT, args.steps + 1, 4,
                                            spec_out.ctypes.data, pkg._abi.TOKEN_CALLBACK(), None,
                                            ctypes.byref(stats))
    assert k > 0, be.info().note
    spec_rate = max(int(stats.completion_tokens) - 1, 1) / reduce_max(dist, stats.decode_seconds)
    same = bool(np.array_equal(spec_out[:k], out[:k]))
    barrier(dist)

    line = None
    if rank == 0:
        line = {
            "metric": TP_METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "31b-tp: plamo-3 profile 31b (tied head), 128-token prompt then greedy "
                                   "decode, batch 1", "model": "plamo-3-31b-shaped (random init)",
                       "global_batch": 1, "seq_len": TP_PROMPT,
                       "parallelism": f"tp{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (weights streamed per step)"},
            "prefill_tok_s": prefill_rate,
            "roofline": {"bound": "hbm", "kernel": "decode step per rank (one CUDA graph launch per token)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "algorithmic_bytes": rank_bytes, "peak_source": peak_src},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "api": "plamo_cuda_generate on every rank"},
            "speculative": {"value": spec_rate, "unit": "tok/s", "draft": "0.8b profile, 4 proposals",
                            "verify_batches": int(stats.verify_batches),
                            "accepted": int(stats.accepted_tokens), "proposed": int(stats.proposed_tokens),
                            "tokens_equal_greedy": same,
                            "note": "random-init draft and target: acceptance says nothing about real models"},
            "gpu_launches": int(launches),
            "clocks": clock_info,
            "cpu_baseline": None,
        }
    be.close()
    return line


def tp_section(args, world, rank, local, dist):
    """BASELINE config 5 at this launch's rank count, for the scaling runs:
    the 31B-shaped tensor-parallel decode (tok/s, per-rank roofline, e2e,
    speculative with a 0.8B-shaped draft), its oracle token check on the
    two-layer cut, and an NCCL all-reduce of one exchange's vector beside the
    fused peer-memory exchanges (129 per token: two per layer and the head's)."""
    check = tp_cut_check(world, rank, local, dist)
    tp = measure_tp31b(args, world, rank, local, dist)
    nccl_us = nccl_allreduce_latency(dist, pkg_profile_hidden("31b"))
    if rank != 0:
        return None
    exchanges = 2 * 64 + 1
    return {"workload": tp["config"]["workload"], "parallelism": tp["config"]["parallelism"],
            "value": tp["value"], "unit": "tok/s", "ms_per_step": tp["ms_per_step"],
            "scaling": "strong", "prefill_tok_s": tp["prefill_tok_s"], "roofline": tp["roofline"],
            "e2e": tp["e2e"], "speculative": tp["speculative"], "gpu_launches": tp["gpu_launches"],
            "clocks": tp["clocks"], "oracle_check": check,
            "nccl_reference": {"allreduce_us": nccl_us, "vector": "[5120] fp32",
                               "per_token_ms_if_nccl": nccl_us * exchanges / 1000.0,
                               "exchanges_per_token": exchanges,
                               "note": "latency of the library collective for one exchange; the step "
                                       "uses fused peer-memory exchanges inside its projection kernels"}}


def pkg_profile_hidden(name):
    return load_package().PROFILES[name].hidden


def run_profile(args):
    """Small fixed workloads for ncu captures (profiles/ gives the commands).
    Each prints the launch count before the part to capture (ncu -s) and the
    number of kernels it launches (ncu -c)."""
    pkg = load_package()
    lib = pkg.load()
    be = pkg.Backend(device=0, max_context=8208, max_prefill=512)
    ctx = be.ctx
    shape = [int(x) for x in args.shape.split(",")] if args.shape else []
    if args.profile in ("gemv", "gemm"):
        if args.profile == "gemv":
            (rows, cols), tokens = shape, 1
        else:
            tokens, rows, cols = shape
        dw = lib.plamo_cuda_device_alloc(ctx, rows * cols * 2)
        dx = lib.plamo_cuda_device_alloc(ctx, tokens * cols * 4)
        dy = lib.plamo_cuda_device_alloc(ctx, tokens * rows * 4)
        lib.plamo_cuda_fill_synthetic_bf16(ctx, dw, rows * cols, 9, 0.0, 0.02)
        lib.plamo_cuda_fill_synthetic_f32(ctx, dx, tokens * cols, 8, 0.0, 1.0)
        timed = (lambda n: lib.plamo_cuda_time_gemv(ctx, dw, dx, dy, rows, cols, n)) if args.profile == "gemv" \
            else (lambda n: lib.plamo_cuda_time_gemm(ctx, dx, dw, dy, tokens, rows, cols, n))
        timed(2)
        before = lib.plamo_cuda_kernel_launches(ctx)
        ms = timed(1)
    else:
        profile = pkg.PROFILES[args.model]
        if args.layers:
            from dataclasses import replace
            profile = replace(profile, name=f"{profile.name}-{args.layers}layers", layers=args.layers)
        hm = pkg.HostModel(profile, weights="synthetic", full_capacity=8208)
        be.preload_synthetic(hm, seed=4)
        reqs = [hm] + [pkg.HostModel(profile, weights_of=hm, full_capacity=8208)
                       for _ in range((args.requests if args.profile == "batch" else 1) - 1)]
        nxt = ctypes.c_uint32()
        toks = np.zeros(len(reqs), dtype=np.uint32)
        prompt = PROMPT if args.profile in ("step", "timeline", "prefill") else 16
        for i, r in enumerate(reqs):
            be.prepare(r)
            ids = np.random.default_rng(1 + i).integers(3, 100000, size=prompt).astype(np.uint32)
            assert lib.plamo_cuda_prefill_greedy(ctx, r.ptr, ids.ctypes.data, prompt, ctypes.byref(nxt)) == 1
            toks[i] = nxt.value
        if args.profile == "timeline":
            # Device timeline of one decode step of the graph path (the launch
            # records of plamo_cuda_decode_trace), after three warm steps.
            ids = np.random.default_rng(1).integers(3, 100000, size=PROMPT).astype(np.uint32)
            lib.plamo_cuda_reset_request(ctx, hm.ptr)
            assert lib.plamo_cuda_prefill_greedy(ctx, hm.ptr, ids.ctypes.data, PROMPT, ctypes.byref(nxt)) == 1
            n = 6 * (5 * profile.layers + 1)
            st = np.zeros(n, dtype=np.uint64)
            before = lib.plamo_cuda_kernel_launches(ctx)
            for k in range(4):
                assert lib.plamo_cuda_decode_trace(ctx, hm.ptr, 5 + k, st.ctypes.data, n) == n, be.info().note
            rel = (st.reshape(-1, 6).astype(np.int64) - int(st[0])) / 1000.0
            kinds = ["qkv", "attention", "o_proj", "gate_up", "down"]
            summary = {}
            for j, kind in enumerate(kinds):
                rows = [5 * l + j for l in range(1, profile.layers)]
                summary[kind] = {
                    "span_us": float(np.mean([rel[i, 3] - rel[i, 1] for i in rows])),
                    "gap_us": float(np.mean([rel[i, 1] - rel[i - 1, 3] for i in rows])),
                    "last_entry_us": float(np.mean([rel[i, 5] - rel[i - 1, 3] for i in rows])),
                    "wait_passed_us": float(np.mean([rel[i, 4] - rel[i - 1, 3] for i in rows])),
                    "prologue_us": float(np.mean([rel[i, 1] - rel[i, 4] for i in rows]))}
            print(json.dumps({"timeline": summary, "step_us": float(rel[-1, 3]),
                              "per_layer_us": float((rel[5 * (profile.layers - 1), 1] - rel[5, 1]) /
                                                    (profile.layers - 2))}), flush=True)
            ms = float(rel[-1, 3]) / 1000
        elif args.profile == "prefill":
            ids = np.random.default_rng(1).integers(3, 100000, size=PROMPT).astype(np.uint32)
            lib.plamo_cuda_reset_request(ctx, hm.ptr)
            before = lib.plamo_cuda_kernel_launches(ctx)
            t0 = be.info().gpu_seconds
            assert lib.plamo_cuda_prefill_greedy(ctx, hm.ptr, ids.ctypes.data, PROMPT, ctypes.byref(nxt)) == 1
            ms = (be.info().gpu_seconds - t0) * 1000
        elif args.profile == "step":
            assert lib.plamo_cuda_time_decode(ctx, hm.ptr, 3) > 0
            before = lib.plamo_cuda_kernel_launches(ctx)
            ms = lib.plamo_cuda_time_decode(ctx, hm.ptr, 1)
        else:
            arr = (ctypes.c_void_p * len(reqs))(*[ctypes.addressof(r.model) for r in reqs])
            batch = lib.plamo_cuda_batch_open(ctx, arr, len(reqs))
            out = np.zeros(len(reqs), dtype=np.uint32)
            assert lib.plamo_cuda_batch_step(batch, toks.ctypes.data, out.ctypes.data) == 1
            assert lib.plamo_cuda_time_batch(batch, 3) > 0
            before = lib.plamo_cuda_kernel_launches(ctx)
            ms = lib.plamo_cuda_time_batch(batch, 1)
            lib.plamo_cuda_batch_close(batch)
    kernels = lib.plamo_cuda_kernel_launches(ctx) - before
    print(json.dumps({"profile": args.profile, "launches_before": int(before), "kernels": int(kernels),
                      "ms": ms}), flush=True)
    be.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp", action="store_true",
                    help="at N > 1, skip the 31B tensor-parallel section of the line")
    ap.add_argument("--workload", choices=["8b-decode", "31b-tp"], default="8b-decode")
    ap.add_argument("--profile", choices=["step", "timeline", "prefill", "batch", "gemv", "gemm"],
                    help="run one small fixed workload for an ncu capture instead of the benchmark")
    ap.add_argument("--model", default="8b", help="profile of --profile step/batch")
    ap.add_argument("--requests", type=int, default=8, help="requests of --profile batch")
    ap.add_argument("--layers", type=int, default=0, help="--profile step/batch: keep only this many layers")
    ap.add_argument("--shape", default="", help="rows,cols (gemv) or tokens,rows,cols (gemm)")
    args = ap.parse_args()
    if args.profile:
        run_profile(args)
        return
    if args.warmup < 1 or args.steps < 1:
        ap.error("steps and warmup must be positive")
    if args.impl == "reference":
        if args.workload != "8b-decode":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference CPU path is timed on the "
                                  "8b-decode workload only (the 31B host model alone is 63.5 GB)"}))
            return
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local, dist = dist_setup(args.gpus)
    try:
        if args.workload == "31b-tp":
            try:
                run_tp31b(args, world, rank, local, dist)
            except BaseException:
                # Keep this rank's exchange buffer mapped until the peers'
                # bounded waits (2 s) have given up writing to it.
                if world > 1:
                    time.sleep(5)
                raise
        else:
            line = run_ours(args, world, rank, local, dist)
            if world > 1 and not args.no_tp:
                try:
                    tp = tp_section(args, world, rank, local, dist)
                except BaseException:
                    time.sleep(5)  # peers' bounded waits end before this rank's buffers go
                    raise
                if rank == 0:
                    line["tp"] = tp
            if rank == 0:
                print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
