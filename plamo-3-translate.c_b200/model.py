"""Model descriptors for the B200 backend: profiles, weight schema, RoPE tables.

`HostModel` builds the reference's `struct model` descriptor tree (the records
of reference runtime/model.h) in host memory, the way the reference's
generated layout does (reference tools/model_layout.py:71-199): one layer
record per decoder layer, a KV cache of `window + 1` rows for sliding layers and
`max_position_embeddings` rows for every 8th (full-attention) layer, the
sliding/full RoPE frequency tables and per-layer concentration. Weights are
BF16 tensors in the order of reference tools/weight_schema.py:15-42, either in
a host blob (uploaded by plamo_cuda_preload) or generated directly in HBM
(plamo_cuda_preload_synthetic; the host addresses then only name the ranges).
"""
import ctypes
import math
import os
from dataclasses import dataclass, field, replace

import numpy as np

from . import _abi


@dataclass(frozen=True)
class Profile:
    name: str
    hidden: int
    layers: int
    qh: int
    kh: int
    dim: int
    inter: int
    vocab: int = 107520
    window: int = 2048
    pattern: int = 8
    max_position: int = 262144
    tied: bool = False
    local_theta: float = 10000.0
    global_theta: float = 1000000.0
    yarn_factor: float = 256.0
    yarn_original: float = 4096.0
    beta_fast: float = 32.0
    beta_slow: float = 1.0

    @property
    def qkv_rows(self):
        return (self.qh + 2 * self.kh) * self.dim

    @property
    def attention_width(self):
        return self.qh * self.dim

    def full(self, layer):
        """Layer i is full attention iff (i + 1) % pattern == 0 (tools/model_layout.py:75)."""
        return (layer + 1) % self.pattern == 0

    def weight_bytes_per_token(self):
        """Projection + head bytes streamed by one decode step (reference docs/METAL.md:233)."""
        h, per_layer = self.hidden, 0
        per_layer += self.qkv_rows * h + h * self.attention_width + 3 * self.inter * h
        return 2 * (self.layers * per_layer + self.vocab * h)

    def norm_bytes_per_token(self):
        return 2 * (self.layers * (4 * self.hidden + 2 * self.dim) + self.hidden)


# The four pinned checkpoints (reference tools/profiles/<model>/config.json).
PROFILES = {
    "0.8b": Profile("0.8b", 1536, 16, 16, 1, 128, 6144),
    "2b": Profile("2b", 2560, 24, 24, 4, 128, 10240),
    "8b": Profile("8b", 4096, 32, 32, 4, 128, 16384),
    "31b": Profile("31b", 5120, 64, 64, 8, 128, 25600, tied=True),
}


def schema(p):
    """(name, shape) of every tensor in slot order (reference tools/weight_schema.py:15-42)."""
    rows = [("model.embed_tokens.weight", (p.vocab, p.hidden)), ("model.norm.weight", (p.hidden,))]
    if not p.tied:
        rows.append(("lm_head.weight", (p.vocab, p.hidden)))
    per_layer = [
        ("mixer.qkv_proj.weight", (p.qkv_rows, p.hidden)),
        ("mixer.o_proj.weight", (p.hidden, p.attention_width)),
        ("mixer.q_norm.weight", (p.dim,)),
        ("mixer.k_norm.weight", (p.dim,)),
        ("mlp.gate_up_proj.weight", (2 * p.inter, p.hidden)),
        ("mlp.down_proj.weight", (p.hidden, p.inter)),
        ("pre_mixer_norm.weight", (p.hidden,)),
        ("post_mixer_norm.weight", (p.hidden,)),
        ("pre_mlp_norm.weight", (p.hidden,)),
        ("post_mlp_norm.weight", (p.hidden,)),
    ]
    for layer in range(p.layers):
        rows.extend((f"model.layers.layers.{layer}.{name}", shape) for name, shape in per_layer)
    return rows


def _fp(x):
    return float(np.float32(x))


def rope_frequencies(theta, half, yarn=None):
    """Inverse frequencies with FP32 rounding after every step, as
    reference tools/rope_constants.py:21-52 forms them. `yarn` is
    (factor, original, beta_fast, beta_slow) or None."""
    if yarn:
        factor, original, beta_fast, beta_slow = yarn
        low = half * math.log(original / (beta_fast * 2 * math.pi)) / math.log(theta)
        high = half * math.log(original / (beta_slow * 2 * math.pi)) / math.log(theta)
    out = []
    for index in range(half):
        frequency = _fp(theta ** (index / half))
        value = _fp(1 / frequency)
        if yarn:
            ramp = _fp(_fp(index - _fp(low)) / _fp(high - low))
            mask = _fp(1 - max(0, min(1, ramp)))
            interpolated = _fp(1 / _fp(factor * frequency))
            value = _fp(_fp(interpolated * _fp(1 - mask)) + _fp(value * mask))
        out.append(value)
    return np.array(out, dtype=np.float32)


def concentration(factor):
    return _fp(1 + 0.1 * math.log(factor))


@dataclass
class LayerSpec:
    sliding: bool
    capacity: int
    freq: np.ndarray
    scale: float


def default_layer_specs(p, full_capacity=None):
    local = rope_frequencies(p.local_theta, p.dim // 2)
    glob = rope_frequencies(p.global_theta, p.dim // 2,
                            (p.yarn_factor, p.yarn_original, p.beta_fast, p.beta_slow))
    specs = []
    for i in range(p.layers):
        if p.full(i):
            specs.append(LayerSpec(False, full_capacity or p.max_position, glob,
                                   concentration(p.yarn_factor)))
        else:
            specs.append(LayerSpec(True, p.window + 1, local, 1.0))
    return specs


def tp_shard_profile(p, size):
    """Profile of one tensor-parallel rank's shard: qh/size query heads,
    kh/size KV heads and intermediate/size MLP rows; hidden size, layers,
    vocabulary and the attention pattern are the full model's."""
    if p.qh % size or p.kh % size or p.inter % size:
        raise ValueError(f"{p.name}: heads {p.qh}/{p.kh} and intermediate {p.inter} must split {size} ways")
    return replace(p, name=f"{p.name}-tp{size}", qh=p.qh // size, kh=p.kh // size, inter=p.inter // size)


def tp_vocab_slice(vocab, size, rank):
    """(first row, rows) of rank's head slice: ceil(vocab/size) rows each, the
    last rank takes the rest."""
    per = -(-vocab // size)
    first = min(rank * per, vocab)
    return first, min(per, vocab - first)


def tp_segments(full, size, rank, name):
    """How a rank's shard of tensor `name` is cut from the full model's tensor:
    (cols, full_cols, col0, [(row_start, row_count), ...]) or None when the
    tensor is replicated. Rank r holds query heads [r*qh/size, ...), KV heads
    [r*kh/size, ...) (Q, K and V row blocks of qkv_proj), the matching o_proj
    columns, gate and up rows [r*I/size, ...) and the matching down_proj
    columns."""
    d, h = full.dim, full.hidden
    qr, kr, ir = full.qh // size, full.kh // size, full.inter // size
    if name.endswith("mixer.qkv_proj.weight"):
        return h, h, 0, [(rank * qr * d, qr * d), (full.qh * d + rank * kr * d, kr * d),
                         ((full.qh + full.kh) * d + rank * kr * d, kr * d)]
    if name.endswith("mixer.o_proj.weight"):
        return qr * d, full.qh * d, rank * qr * d, [(0, h)]
    if name.endswith("mlp.gate_up_proj.weight"):
        return h, h, 0, [(rank * ir, ir), (full.inter + rank * ir, ir)]
    if name.endswith("mlp.down_proj.weight"):
        return ir, full.inter, rank * ir, [(0, h)]
    return None


def tp_all_gather_handles(handle, group=None):
    """Every rank's exchange-buffer handle, indexed by rank, through the
    caller's torch.distributed process group (any backend: the handles are
    64-byte host records)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


def _align(n, a=256):
    return (n + a - 1) // a * a


class _Reservation:
    """Address range with no backing memory (PROT_NONE): the keys under which
    weights generated directly in HBM are registered. Never dereferenced."""

    PROT_NONE, MAP_PRIVATE, MAP_ANONYMOUS, MAP_NORESERVE = 0, 0x02, 0x20, 0x4000

    def __init__(self, size):
        self.size = max(int(size), 1)
        libc = ctypes.CDLL(None, use_errno=True)
        libc.mmap.restype = ctypes.c_void_p
        libc.mmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_long]
        libc.munmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        self._munmap = libc.munmap
        addr = libc.mmap(None, self.size, self.PROT_NONE,
                         self.MAP_PRIVATE | self.MAP_ANONYMOUS | self.MAP_NORESERVE, -1, 0)
        if addr in (None, ctypes.c_void_p(-1).value):
            raise OSError(ctypes.get_errno(), "cannot reserve weight address range")
        self.address = addr

    def __del__(self):
        if getattr(self, "address", None):
            self._munmap(self.address, self.size)
            self.address = None


class HostModel:
    """The descriptor tree of one model plus the host buffers it points to.

    weights: "synthetic" (generated in HBM by `Backend.preload_synthetic`),
    a numpy uint16 blob laid out by `self.offsets`, a dict {tensor name: host
    address} (a mapped checkpoint, see open_checkpoint), or None to allocate a
    zero blob the caller fills. weights_of: another HostModel of the same profile
    whose weights this one shares (same host keys, so the same device copies):
    a second request with its own descriptors and KV cache.
    """

    def __init__(self, profile, layer_specs=None, weights=None, full_capacity=None, weights_of=None):
        p = self.profile = profile
        self.specs = layer_specs or default_layer_specs(p, full_capacity)
        assert len(self.specs) == p.layers
        self.schema = schema(p)
        self.offsets, total = {}, 0
        for name, shape in self.schema:
            self.offsets[name] = total
            total = _align(total + 2 * int(np.prod(shape)))
        self.blob_bytes = total
        self._keep = []
        self.synthetic = isinstance(weights, str) and weights == "synthetic"
        self.addresses = weights if isinstance(weights, dict) else None
        if self.addresses is not None:
            missing = [name for name, _ in self.schema if name not in self.addresses]
            assert not missing, missing
            self.blob = None
            base = 0
        elif weights_of is not None:
            assert weights_of.blob_bytes == total and weights_of.profile == p
            self.synthetic = weights_of.synthetic
            self.reservation = getattr(weights_of, "reservation", None)
            self.blob = weights_of.blob
            self._keep.append(weights_of)
            base = weights_of.base
        elif self.synthetic:
            self.reservation = _Reservation(total)
            self.blob = None
            base = self.reservation.address
        else:
            if weights is None:
                weights = np.zeros(total // 2, dtype=np.uint16)
            assert weights.dtype == np.uint16 and weights.nbytes >= total
            self.blob = weights
            base = weights.ctypes.data
        self.base = base

        def w(name):
            if self.addresses is not None:
                return self.addresses[name]
            return base + self.offsets[name]

        h, qw, aw, kvw = p.hidden, p.qkv_rows, p.attention_width, p.kh * p.dim
        f32 = self._f32
        self.state = f32(h)
        self.normalized = f32(h)
        self.logits = f32(p.vocab)
        work_norm, work_branch = f32(h), f32(h)
        work_qkv, work_attn = f32(qw), f32(aw)
        mlp_scratch, mlp_norm, mlp_branch = f32(2 * p.inter), f32(h), f32(h)
        cap_max = max(s.capacity for s in self.specs)
        scores = f32(cap_max)
        cos, sin = f32(p.dim // 2), f32(p.dim // 2)
        self.scales = np.array([s.scale for s in self.specs], dtype=np.float32)
        self.layers = []
        self.caches = []
        layer_ptrs = (ctypes.POINTER(_abi.Layer) * p.layers)()
        for i, spec in enumerate(self.specs):
            prefix = f"model.layers.layers.{i}."
            kc = _abi.Cache(k=f32(spec.capacity * kvw), v=f32(spec.capacity * kvw),
                            capacity=spec.capacity, count=0, width=kvw, sliding=int(spec.sliding))
            freq = np.ascontiguousarray(spec.freq, dtype=np.float32)
            self._keep.append(freq)
            rot = _abi.Rotation(cache=ctypes.pointer(kc), out=f32(spec.capacity * kvw),
                                freq=freq.ctypes.data, cos=cos, sin=sin, heads=p.kh, dim=p.dim,
                                processed_count=0, scale_bits=0)
            q = _abi.Qkv(input=work_norm, weight=w(prefix + "mixer.qkv_proj.weight"),
                         qn=w(prefix + "mixer.q_norm.weight"), kn=w(prefix + "mixer.k_norm.weight"),
                         out=work_qkv, hidden=h, qh=p.qh, kh=p.kh, dim=p.dim)
            g = _abi.Gqa(q=None, k=None, v=None, out=work_attn, scores=scores, tokens=0,
                         dim=p.dim, qh=p.qh, kh=p.kh)
            mix = _abi.Mixer(qkv=ctypes.pointer(q), cache=ctypes.pointer(kc),
                             rotation=ctypes.pointer(rot), gqa=ctypes.pointer(g),
                             weight=w(prefix + "mixer.o_proj.weight"), out=work_branch, hidden=h)
            mlp = _abi.Mlp(state=self.state, pre=w(prefix + "pre_mlp_norm.weight"),
                           post=w(prefix + "post_mlp_norm.weight"),
                           gu=w(prefix + "mlp.gate_up_proj.weight"),
                           down=w(prefix + "mlp.down_proj.weight"), normalized=mlp_norm,
                           branch=mlp_branch, scratch=mlp_scratch, hidden=h,
                           intermediate=p.inter)
            layer = _abi.Layer(state=self.state, pre=w(prefix + "pre_mixer_norm.weight"),
                               post=w(prefix + "post_mixer_norm.weight"), normalized=work_norm,
                               branch=work_branch, mixer=ctypes.pointer(mix),
                               mlp=ctypes.pointer(mlp), hidden=h)
            self._keep += [kc, rot, q, g, mix, mlp, layer]
            self.layers.append(layer)
            self.caches.append(kc)
            layer_ptrs[i] = ctypes.pointer(layer)
        self._keep.append(layer_ptrs)
        head = "model.embed_tokens.weight" if p.tied else "lm_head.weight"
        self.model = _abi.Model(embedding=w("model.embed_tokens.weight"), vocab=p.vocab, hidden=h,
                                state=self.state, layers=layer_ptrs, count=p.layers,
                                scales=self.scales.ctypes.data, norm=w("model.norm.weight"),
                                normalized=self.normalized, head=w(head), logits=self.logits)
        self.ptr = ctypes.pointer(self.model)

    def _f32(self, n):
        a = np.zeros(max(int(n), 1), dtype=np.float32)
        self._keep.append(a)
        return a.ctypes.data

    # ---- host views -------------------------------------------------------
    def view(self, address, count, dtype=np.float32):
        return np.ctypeslib.as_array(ctypes.cast(address, ctypes.POINTER(
            ctypes.c_float if dtype == np.float32 else ctypes.c_uint16)), shape=(count,))

    def tensor(self, name):
        shape = dict(self.schema)[name]
        n = int(np.prod(shape))
        off = self.offsets[name] // 2
        return self.blob[off:off + n].reshape(shape)

    def state_array(self):
        return self.view(self.model.state, self.profile.hidden).copy()

    def logits_array(self):
        return self.view(self.model.logits, self.profile.vocab).copy()

    def normalized_array(self):
        return self.view(self.model.normalized, self.profile.hidden).copy()

    def kv_arrays(self, i):
        """(k, v, rotated k) host rows [0, count) of layer i."""
        kc = self.caches[i]
        kvw = self.profile.kh * self.profile.dim
        n = kc.count * kvw
        rot = self.layers[i].mixer.contents.rotation.contents
        return (self.view(kc.k, n).copy(), self.view(kc.v, n).copy(), self.view(rot.out, n).copy())

    def rotation(self, i):
        return self.layers[i].mixer.contents.rotation.contents

    def reset(self):
        """plamo_reset_request (reference runtime/engine.c:46-55) on the host records."""
        for layer, kc in zip(self.layers, self.caches):
            layer.state = self.model.state
            kc.count = 0
            rot = layer.mixer.contents.rotation.contents
            rot.processed_count = 0
            rot.scale_bits = 0
            layer.mixer.contents.gqa.contents.tokens = 0

    def tensor_ranges(self):
        """(address, element count, name) of every weight tensor."""
        if self.addresses is not None:
            return [(self.addresses[name], int(np.prod(shape)), name) for name, shape in self.schema]
        return [(self.base + self.offsets[name], int(np.prod(shape)), name)
                for name, shape in self.schema]


class Tokenizer:
    """PLaMo-3 tokenizer over a tokenizer.jsonl vocabulary (include/plamo_tokenizer.h;
    reference runtime/tokenizer.h): text -> ids, optionally wrapped in the
    translation prompt (direction 1: English to Japanese, 2: Japanese to
    English), and ids -> bytes."""

    FAIL = 2**64 - 1

    def __init__(self, path):
        self.lib = _abi.load()
        err = ctypes.create_string_buffer(256)
        self.handle = self.lib.plamo_tokenizer_open(os.fsencode(path), err, 256)
        if not self.handle:
            raise ValueError(err.value.decode() or f"cannot open {path}")

    def encode(self, text, direction=0):
        ids = ctypes.POINTER(ctypes.c_uint32)()
        err = ctypes.create_string_buffer(256)
        data = text.encode() if isinstance(text, str) else bytes(text)
        n = self.lib.plamo_tokenizer_encode(self.handle, data, direction, ctypes.byref(ids), err, 256)
        if n == self.FAIL:
            raise ValueError(err.value.decode())
        return np.array([ids[i] for i in range(n)], dtype=np.uint32)

    def prefix(self, direction):
        """The fixed prompt prefix of a source language (0: English, 1: Japanese)."""
        ids = ctypes.POINTER(ctypes.c_uint32)()
        err = ctypes.create_string_buffer(256)
        n = self.lib.plamo_tokenizer_prefix(self.handle, direction, ctypes.byref(ids), err, 256)
        if n == self.FAIL:
            raise ValueError(err.value.decode() or "unsupported prefix direction")
        return np.array([ids[i] for i in range(n)], dtype=np.uint32)

    def decode(self, ids):
        """Bytes of the pieces (BYTE pieces are raw bytes: decode the result as UTF-8)."""
        out = b""
        for i in np.atleast_1d(ids):
            p = ctypes.c_char_p()
            n = self.lib.plamo_tokenizer_decode(self.handle, int(i), ctypes.byref(p))
            if n == self.FAIL:
                raise ValueError(f"token {int(i)} is outside the vocabulary")
            out += ctypes.string_at(p, n)
        return out

    def close(self):
        if self.handle:
            self.lib.plamo_tokenizer_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Checkpoint:
    """Mapped BF16 safetensors shards bound to a profile's weight schema
    (reference src/model_open.s: map every shard, bind every schema entry with
    its exact shape, all or nothing). `model` is the descriptor tree over the
    mapped bytes; Backend.preload_model uploads them."""

    def __init__(self, paths, profile, layer_specs=None, full_capacity=None):
        lib = _abi.load()
        self.maps = (_abi.Mapping * len(paths))()
        self.count = 0
        for i, path in enumerate(paths):
            if not lib.plamo_map_file(os.fsencode(path), ctypes.byref(self.maps[i])):
                self.close()
                raise OSError(f"cannot map {path}")
            self.count = i + 1
        sch = schema(profile)
        self._shapes = [(ctypes.c_uint64 * len(shape))(*shape) for _, shape in sch]
        self._names = [name.encode() for name, _ in sch]
        self._slots = (ctypes.c_void_p * len(sch))()
        specs = (_abi.WeightSpec * (len(sch) + 1))()
        for i, (name, shape) in enumerate(sch):
            specs[i] = _abi.WeightSpec(self._names[i], len(shape), self._shapes[i],
                                       ctypes.cast(ctypes.byref(self._slots, i * ctypes.sizeof(ctypes.c_void_p)),
                                                   ctypes.POINTER(ctypes.c_void_p)))
        if not lib.plamo_bind_weights(self.maps, self.count, specs):
            self.close()
            raise ValueError("checkpoint does not match the profile's weight schema (names, BF16, shapes)")
        addresses = {name: self._slots[i] for i, (name, _) in enumerate(sch)}
        self.model = HostModel(profile, layer_specs, weights=addresses, full_capacity=full_capacity)

    def close(self):
        lib = _abi.load()
        for i in range(self.count):
            lib.plamo_unmap_file(ctypes.byref(self.maps[i]))
        self.count = 0


def write_safetensors(path, tensors, metadata=None):
    """Write {name: uint16 array (BF16 bits)} as one safetensors file (test and
    tooling helper; the loader itself is C)."""
    import json
    header, offset, blobs = {}, 0, []
    if metadata:
        header["__metadata__"] = metadata
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr, dtype=np.uint16)
        header[name] = {"dtype": "BF16", "shape": list(arr.shape), "data_offsets": [offset, offset + arr.nbytes]}
        offset += arr.nbytes
        blobs.append(arr)
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * ((8 - len(text) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(text).to_bytes(8, "little"))
        f.write(text)
        for arr in blobs:
            f.write(arr.tobytes())


def synthetic_parameters(name, std=0.02):
    """(mean, std) of a synthetic tensor: norms are stored as 1.0, projections
    and embeddings draw from N(0, std)."""
    if name.endswith("norm.weight"):
        return 1.0, 0.0
    return 0.0, std


class Backend:
    """Thin owner of one plamo_cuda context."""

    def __init__(self, device=0, max_context=0, max_prefill=0, copy_kv_to_host=False):
        self.lib = _abi.load()
        cfg = _abi.CudaConfig(device=device, max_context=max_context, max_prefill=max_prefill,
                              reserve=0, copy_kv_to_host=int(copy_kv_to_host))
        err = ctypes.create_string_buffer(512)
        self.ctx = self.lib.plamo_cuda_open(ctypes.byref(cfg), err, 512)
        if not self.ctx:
            raise RuntimeError(err.value.decode())

    def close(self):
        if self.ctx:
            self.lib.plamo_cuda_close(self.ctx)
            self.ctx = None

    def info(self):
        info = _abi.CudaInfo()
        self.lib.plamo_cuda_get_info(self.ctx, ctypes.byref(info))
        return info

    def preload_model(self, hm):
        for addr, count, _ in hm.tensor_ranges():
            if not self.lib.plamo_cuda_preload(self.ctx, addr, 2 * count):
                raise RuntimeError(self.info().note.decode())

    def preload_synthetic(self, hm, seed, std=0.02):
        for k, (addr, count, name) in enumerate(hm.tensor_ranges()):
            mean, s = synthetic_parameters(name, std)
            if not self.lib.plamo_cuda_preload_synthetic(self.ctx, addr, count,
                                                         seed * 1000003 + k, mean, s):
                raise RuntimeError(self.info().note.decode())

    def preload_synthetic_tp(self, hm, full, rank, size, seed, std=0.02):
        """Synthetic weights of a tensor-parallel shard `hm` (built from
        tp_shard_profile(full, size)): every tensor is the rank's cut of the
        tensor preload_synthetic generates for the full model, bit for bit."""
        for k, (addr, count, name) in enumerate(hm.tensor_ranges()):
            mean, s = synthetic_parameters(name, std)
            cut = tp_segments(full, size, rank, name)
            if cut is None:
                ok = self.lib.plamo_cuda_preload_synthetic(self.ctx, addr, count, seed * 1000003 + k, mean, s)
            else:
                cols, full_cols, col0, segs = cut
                starts = (ctypes.c_uint64 * len(segs))(*[a for a, _ in segs])
                counts = (ctypes.c_uint64 * len(segs))(*[b for _, b in segs])
                assert sum(b for _, b in segs) * cols == count, name
                ok = self.lib.plamo_cuda_preload_synthetic_rows(self.ctx, addr, cols, full_cols, col0, starts,
                                                                counts, len(segs), seed * 1000003 + k, mean, s)
            if not ok:
                raise RuntimeError(self.info().note.decode())

    def tp_prepare(self, hm, rank, size):
        """Point the shard's head at the rank's vocabulary slice, prepare it and
        return this rank's exchange-buffer handle (bytes)."""
        p = hm.profile
        first, rows = tp_vocab_slice(p.vocab, size, rank)
        head = "model.embed_tokens.weight" if p.tied else "lm_head.weight"
        hm.model.head = hm.base + hm.offsets[head] + first * p.hidden * 2
        handle = _abi.TpHandle()
        if self.lib.plamo_cuda_tp_prepare(self.ctx, hm.ptr, rank, size, first, rows, ctypes.byref(handle)) != 1:
            raise RuntimeError("tp_prepare failed: " + self.info().note.decode())
        return bytes(handle.bytes)

    def tp_connect(self, hm, handles):
        arr = (_abi.TpHandle * len(handles))()
        for i, h in enumerate(handles):
            ctypes.memmove(arr[i].bytes, h, 64)
        if self.lib.plamo_cuda_tp_connect(self.ctx, hm.ptr, arr) != 1:
            raise RuntimeError("tp_connect failed: " + self.info().note.decode())

    def release(self, hm):
        """Drop the device copies of `hm` (its host memory may be reused)."""
        self.lib.plamo_cuda_release_model(self.ctx, hm.ptr)
        if hm.addresses is not None:
            for addr, count, _ in hm.tensor_ranges():
                self.lib.plamo_cuda_release_weights(self.ctx, addr, 2 * count)
        else:
            self.lib.plamo_cuda_release_weights(self.ctx, hm.base, hm.blob_bytes)

    def prepare(self, hm):
        if self.lib.plamo_cuda_prepare_model(self.ctx, hm.ptr) != 1:
            raise RuntimeError("prepare_model failed: " + self.info().note.decode())

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
