"""numpy restatement of include/plamo_synthetic.h (seeded synthetic tensors).

Pins the device generator: plamo_cuda_fill_synthetic_* must produce exactly
these bits. z(seed, i) = (sum of 12 hash bytes - 1530) / 256 with the hash
splitmix64(seed * 0xD1B54A32D192ED03 + 2i [+1]).
"""
import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(x):
    x = (x + np.uint64(0x9E3779B97F4A7C15))
    x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def z(seed, count, start=0):
    with np.errstate(over="ignore"):
        key = np.uint64(seed) * np.uint64(0xD1B54A32D192ED03)
        i = np.arange(start, start + count, dtype=np.uint64)
        a = splitmix64(key + np.uint64(2) * i)
        b = splitmix64(key + np.uint64(2) * i + np.uint64(1))
    s = np.zeros(count, dtype=np.int64)
    for k in range(8):
        s += ((a >> np.uint64(8 * k)) & np.uint64(0xFF)).astype(np.int64)
    for k in range(4):
        s += ((b >> np.uint64(8 * k)) & np.uint64(0xFF)).astype(np.int64)
    return (s - 1530).astype(np.float32) * np.float32(0.00390625)


def f32(seed, count, mean, std):
    prod = np.float32(std) * z(seed, count)
    return (np.float32(mean) + prod).astype(np.float32)


def bf16_round(x):
    bits = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bits = bits + np.uint64(0x7FFF) + ((bits >> np.uint64(16)) & np.uint64(1))
    return (bits >> np.uint64(16)).astype(np.uint16)


def bf16(seed, count, mean, std):
    return bf16_round(f32(seed, count, mean, std))


def bf16_to_f32(u16):
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def fill_model(hm, seed, std=0.02):
    """Host copy of the weights Backend.preload_synthetic(hm, seed) generates."""
    from plamo_b200 import synthetic_parameters
    for k, (_, count, name) in enumerate(hm.tensor_ranges()):
        mean, s = synthetic_parameters(name, std)
        off = hm.offsets[name] // 2
        hm.blob[off:off + count] = bf16(seed * 1000003 + k, count, mean, s)


def lcg_words(seed, count):
    """BF16 patterns 0x3c00 | (s & 0xff) | (s & 0x8000) of the LCG
    s <- s * 1664525 + 1013904223 (reference tests/metal_decode.c:366-375)."""
    a, c, mask = 1664525, 1013904223, 0xFFFFFFFF
    block = 4096
    mul = np.empty(block, dtype=np.uint64)
    add = np.empty(block, dtype=np.uint64)
    m, k = 1, 0
    for i in range(block):  # s_{i+1} = mul[i] * s_0 + add[i]
        m = (m * a) & mask
        k = (k * a + c) & mask
        mul[i], add[i] = m, k
    out = np.empty(count, dtype=np.uint64)
    s = seed
    for start in range(0, count, block):
        n = min(block, count - start)
        vals = (mul[:n] * np.uint64(s) + add[:n]) & np.uint64(mask)
        out[start:start + n] = vals
        s = int(vals[-1])
    return (np.uint64(0x3C00) | (out & np.uint64(0xFF)) | (out & np.uint64(0x8000))).astype(np.uint16)


def lcg_fixture_weights(hm, seed=93):
    """Fill every tensor of `hm`, in schema order, from one LCG word stream."""
    total = sum(c for _, c, _ in hm.tensor_ranges())
    words = lcg_words(seed, total)
    pos = 0
    for _, count, name in hm.tensor_ranges():
        off = hm.offsets[name] // 2
        hm.blob[off:off + count] = words[pos:pos + count]
        pos += count
