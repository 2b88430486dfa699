"""Writes tests/golden/layout.json from the reference's own Python generators.

The reference builds its model descriptors, weight schema and RoPE tables
with Python tools (tools/weight_schema.py, tools/model_layout.py,
tools/rope_constants.py) from per-profile configs (tools/profiles/<name>/
config.json). This script imports those tools from a reference checkout,
runs them for the 0.8B, 2B, 8B and 31B profiles and freezes what the device
path depends on:

  * the profile's shape parameters, as the config states them;
  * the weight schema: every tensor name and shape in slot order;
  * per layer, from the rendered descriptor records: cache capacity, the
    sliding flag, the frequency table it rotates with, its concentration;
  * both frequency tables (FP32) and the global table's concentration.

Usage: python tests/golden/make_layout_golden.py [reference checkout]
(the checkout defaults to the REFERENCE environment variable).
"""
import json
import math
import os
import re
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PROFILES = ("0.8b", "2b", "8b", "31b")


def f32(x):
    return struct.unpack("f", struct.pack("f", x))[0]


def layer_records(text, count):
    """Capacity / sliding flag (cache record), frequency symbol (rotation
    record) per layer and the scale array, from the rendered assembly."""
    quads = {}
    for line in text.splitlines():
        m = re.match(r"(L[cr]\d+): \.quad (.*)$", line)
        if m:
            quads[m.group(1)] = [v.strip() for v in m.group(2).split(",")]
    scales = None
    for line in text.splitlines():
        if line.startswith("Lscales: .float "):
            scales = [float(v) for v in line[len("Lscales: .float "):].split(",")]
    assert scales is not None and len(scales) == count
    layers = []
    for i in range(count):
        cache, rot = quads[f"Lc{i}"], quads[f"Lr{i}"]
        layers.append({"capacity": int(cache[2]), "sliding": bool(int(cache[5])),
                       "table": "global" if rot[2] == "_plamo_rope_global" else "local",
                       "scale": f32(scales[i])})
    return layers


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE", "")
    tools = os.path.join(ref, "tools")
    if not os.path.isdir(tools):
        sys.exit("usage: make_layout_golden.py <reference checkout>")
    sys.path.insert(0, tools)
    import model_layout
    import rope_constants
    import weight_schema

    out = {}
    for name in PROFILES:
        with open(os.path.join(tools, "profiles", name, "config.json")) as f:
            cfg = json.load(f)
        half = cfg["head_dim"] // 2
        local = rope_constants.frequencies(cfg["rope_parameters"]["sliding_attention"], half)
        glob_params = cfg["rope_parameters"]["full_attention"]
        glob = rope_constants.frequencies(glob_params, half)
        out[name] = {
            "config": {k: cfg[k] for k in ("hidden_size", "num_hidden_layers", "num_attention_heads",
                                           "num_key_value_heads", "head_dim", "intermediate_size", "vocab_size",
                                           "window_size", "sliding_window_pattern", "tie_word_embeddings",
                                           "max_position_embeddings")},
            "schema": [[n, list(s)] for n, s in weight_schema.schema(cfg)],
            "layers": layer_records(model_layout.render(cfg), cfg["num_hidden_layers"]),
            "rope_local": [f32(v) for v in local],
            "rope_global": [f32(v) for v in glob],
            "global_concentration": f32(1 + 0.1 * math.log(glob_params["factor"])),
        }
    path = os.path.join(HERE, "layout.json")
    with open(path, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
