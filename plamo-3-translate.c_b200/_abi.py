"""ctypes view of the backend's C ABI (include/plamo_model.h, include/plamo_cuda.h).

The record layouts are the reference's model descriptor ABI
(reference runtime/model.h:7-86, runtime/parallel.h:5-12); the function
table is include/plamo_cuda.h, a drop-in for reference runtime/metal.h:48-88.
The library is loaded from this directory's lib/ (built in-tree by
`make -C plamo-3-translate.c_b200`); importing this module fails loudly when it
is missing, because there is no other implementation to fall back to.
"""
import ctypes
import os
from ctypes import POINTER, c_char, c_char_p, c_double, c_size_t, c_int, c_int64, c_uint, c_uint32, c_uint64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libplamo_cuda.so")
LINEAR_STATIC_FLOATS = 4 << 20  # PLAMO_CUDA_LINEAR_STATIC_FLOATS
PREFIX_LIMIT = 64  # PLAMO_CUDA_PREFIX_LIMIT
VERIFY_MAX = 16  # PLAMO_CUDA_VERIFY_MAX


class Qkv(ctypes.Structure):
    _fields_ = [("input", c_void_p), ("weight", c_void_p), ("qn", c_void_p), ("kn", c_void_p),
                ("out", c_void_p), ("hidden", c_uint64), ("qh", c_uint64), ("kh", c_uint64),
                ("dim", c_uint64)]


class Cache(ctypes.Structure):
    _fields_ = [("k", c_void_p), ("v", c_void_p), ("capacity", c_uint64), ("count", c_uint64),
                ("width", c_uint64), ("sliding", c_uint64)]


class Rotation(ctypes.Structure):
    _fields_ = [("cache", POINTER(Cache)), ("out", c_void_p), ("freq", c_void_p), ("cos", c_void_p),
                ("sin", c_void_p), ("heads", c_uint64), ("dim", c_uint64),
                ("processed_count", c_uint64), ("scale_bits", c_uint64)]


class Gqa(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("out", c_void_p),
                ("scores", c_void_p), ("tokens", c_uint64), ("dim", c_uint64), ("qh", c_uint64),
                ("kh", c_uint64)]


class Mixer(ctypes.Structure):
    _fields_ = [("qkv", POINTER(Qkv)), ("cache", POINTER(Cache)), ("rotation", POINTER(Rotation)),
                ("gqa", POINTER(Gqa)), ("weight", c_void_p), ("out", c_void_p), ("hidden", c_uint64)]


class Mlp(ctypes.Structure):
    _fields_ = [("state", c_void_p), ("pre", c_void_p), ("post", c_void_p), ("gu", c_void_p),
                ("down", c_void_p), ("normalized", c_void_p), ("branch", c_void_p),
                ("scratch", c_void_p), ("hidden", c_uint64), ("intermediate", c_uint64)]


class Layer(ctypes.Structure):
    _fields_ = [("state", c_void_p), ("pre", c_void_p), ("post", c_void_p),
                ("normalized", c_void_p), ("branch", c_void_p), ("mixer", POINTER(Mixer)),
                ("mlp", POINTER(Mlp)), ("hidden", c_uint64)]


class Model(ctypes.Structure):
    _fields_ = [("embedding", c_void_p), ("vocab", c_uint64), ("hidden", c_uint64),
                ("state", c_void_p), ("layers", POINTER(POINTER(Layer))), ("count", c_uint64),
                ("scales", c_void_p), ("norm", c_void_p), ("normalized", c_void_p),
                ("head", c_void_p), ("logits", c_void_p)]


class Matmul(ctypes.Structure):
    _fields_ = [("weights", c_void_p), ("input", c_void_p), ("output", c_void_p),
                ("rows", c_uint64), ("columns", c_uint64), ("tokens", c_uint64),
                ("input_stride", c_uint64), ("output_stride", c_uint64)]


class CudaConfig(ctypes.Structure):
    _fields_ = [("device", c_int), ("max_context", c_uint64), ("max_prefill", c_uint64),
                ("reserve", c_uint64), ("copy_kv_to_host", c_uint)]


class CudaInfo(ctypes.Structure):
    _fields_ = [("device", c_char * 128), ("note", c_char * 256)] + [
        (name, c_uint64) for name in (
            "launches", "graph_launches", "forwards", "prefills", "verification_batches",
            "verified_tokens", "committed_tokens", "declines", "errors", "weight_bytes",
            "kv_bytes", "workspace_bytes", "allocated_bytes", "sm_count")] + [
        ("gpu_seconds", c_double), ("kv_pages_used", c_uint64), ("kv_pages_allocated", c_uint64)]


class CudaTiming(ctypes.Structure):
    _fields_ = [("prefill_seconds", c_double), ("decode_seconds", c_double),
                ("first_token_seconds", c_double), ("prompt_tokens", c_uint64),
                ("completion_tokens", c_uint64), ("decode_steps", c_uint64),
                ("finish_reason", c_char_p)]


class CudaSpeculation(ctypes.Structure):
    _fields_ = [("prefill_seconds", c_double), ("decode_seconds", c_double),
                ("completion_tokens", c_uint64), ("decode_steps", c_uint64),
                ("verify_batches", c_uint64), ("proposed_tokens", c_uint64),
                ("accepted_tokens", c_uint64), ("finish_reason", c_char_p)]


for _struct, _size in ((Qkv, 72), (Cache, 48), (Rotation, 72), (Gqa, 72), (Mixer, 56), (Mlp, 80),
                       (Layer, 64), (Model, 88), (Matmul, 64)):
    assert ctypes.sizeof(_struct) == _size, _struct.__name__

class TpHandle(ctypes.Structure):
    """struct plamo_cuda_tp_handle: a CUDA IPC handle of a rank's exchange buffer."""
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


TP_MAX = 8  # PLAMO_CUDA_TP_MAX
TOKEN_CALLBACK = ctypes.CFUNCTYPE(c_int, c_uint32, c_void_p)
P = c_void_p
M = POINTER(Model)
# name -> (restype, argtypes); exactly the entry points of include/plamo_cuda.h.
SIGNATURES = {
    "plamo_cuda_open": (c_void_p, [POINTER(CudaConfig), c_char_p, ctypes.c_size_t]),
    "plamo_cuda_close": (None, [P]),
    "plamo_cuda_maintain": (None, [P]),
    "plamo_cuda_get_info": (None, [P, POINTER(CudaInfo)]),
    "plamo_cuda_preload": (c_int, [P, P, c_uint64]),
    "plamo_cuda_warm_cache": (c_int, [P]),
    "plamo_cuda_prepare_model": (c_int, [P, M]),
    "plamo_cuda_forward": (c_int, [P, M, c_uint64]),
    "plamo_cuda_prefill": (c_int, [P, M, P, c_uint64, P]),
    "plamo_cuda_verify": (c_int, [P, M, P, c_uint64, P]),
    "plamo_cuda_commit": (c_int, [P, M, c_uint64]),
    "plamo_cuda_linear": (c_int, [P, POINTER(Matmul)]),
    "plamo_cuda_linear_static": (c_int, [P, POINTER(Matmul)]),
    "plamo_cuda_mlp": (c_int, [P, POINTER(Mlp), P, c_uint64]),
    "plamo_cuda_sync_host": (c_int, [P, M]),
    "plamo_cuda_invalidate": (c_int, [P, M]),
    "plamo_cuda_release_model": (c_int, [P, M]),
    "plamo_cuda_release_weights": (c_int, [P, P, c_uint64]),
    "plamo_cuda_forward_greedy": (c_int, [P, M, c_uint64, POINTER(c_uint32)]),
    "plamo_cuda_forward_greedy_margin": (c_int, [P, M, c_uint64, POINTER(c_uint32), POINTER(ctypes.c_float)]),
    "plamo_cuda_prefill_greedy": (c_int, [P, M, P, c_uint64, POINTER(c_uint32)]),
    "plamo_cuda_generate": (c_int64, [P, M, P, c_uint64, c_uint64, P, TOKEN_CALLBACK, P,
                                      POINTER(CudaTiming)]),
    "plamo_cuda_layer": (c_int, [P, M, c_uint64, P]),
    "plamo_cuda_reset_request": (None, [P, M]),
    "plamo_cuda_rollback": (c_int, [P, M, c_uint64]),
    "plamo_cuda_prompt_cache_capture": (c_void_p, [P, M, P, c_uint64]),
    "plamo_cuda_prompt_cache_restore": (c_uint64, [P, P, M, P, c_uint64]),
    "plamo_cuda_prompt_cache_tokens": (c_uint64, [P]),
    "plamo_cuda_prompt_cache_bytes": (c_uint64, [P]),
    "plamo_cuda_prompt_cache_free": (None, [P]),
    "plamo_cuda_generate_speculative": (c_int64, [P, M, M, P, c_uint64, c_uint64, c_uint, P, TOKEN_CALLBACK, P,
                                                  POINTER(CudaSpeculation)]),
    "plamo_cuda_read_weights": (c_int, [P, P, P, c_uint64]),
    "plamo_cuda_gemv_device": (c_int, [P, P, P, P, c_uint64, c_uint64]),
    "plamo_cuda_gemm_device": (c_int, [P, P, c_uint64, P, P, c_uint64, c_uint64, c_uint64, c_uint64]),
    "plamo_cuda_time_gemm": (c_double, [P, P, P, P, c_uint64, c_uint64, c_uint64, c_uint64]),
    "plamo_cuda_device_alloc": (c_void_p, [P, c_uint64]),
    "plamo_cuda_device_free": (None, [P, P]),
    "plamo_cuda_copy_to_device": (c_int, [P, P, P, c_uint64]),
    "plamo_cuda_copy_to_host": (c_int, [P, P, P, c_uint64]),
    "plamo_cuda_synchronize": (c_int, [P]),
    "plamo_cuda_time_decode": (c_double, [P, M, c_uint64]),
    "plamo_cuda_time_gemv": (c_double, [P, P, P, P, c_uint64, c_uint64, c_uint64]),
    "plamo_cuda_time_gemv_copies": (c_double, [P, P, c_uint64, P, P, c_uint64, c_uint64, c_uint64]),
    "plamo_cuda_kernel_launches": (c_uint64, [P]),
    "plamo_cuda_decode_path": (c_char_p, [P, M]),
    "plamo_cuda_read_outputs": (c_int, [P, M]),
    "plamo_cuda_decode_trace": (c_double, [P, M, c_uint64, P, c_uint64]),
    "plamo_cuda_preload_synthetic": (c_int, [P, P, c_uint64, c_uint64, ctypes.c_float,
                                             ctypes.c_float]),
    "plamo_cuda_fill_synthetic_bf16": (c_int, [P, P, c_uint64, c_uint64, ctypes.c_float,
                                               ctypes.c_float]),
    "plamo_cuda_fill_synthetic_f32": (c_int, [P, P, c_uint64, c_uint64, ctypes.c_float,
                                              ctypes.c_float]),
    "plamo_cuda_preload_synthetic_rows": (c_int, [P, P, c_uint64, c_uint64, c_uint64, P, P, c_uint,
                                                  c_uint64, ctypes.c_float, ctypes.c_float]),
    "plamo_cuda_tp_prepare": (c_int, [P, M, c_uint, c_uint, c_uint64, c_uint64,
                                      POINTER(TpHandle)]),
    "plamo_cuda_tp_connect": (c_int, [P, M, POINTER(TpHandle)]),
    "plamo_cuda_batch_open": (c_void_p, [P, P, c_uint]),
    "plamo_cuda_batch_step": (c_int, [P, P, P]),
    "plamo_cuda_time_batch": (c_double, [P, c_uint64]),
    "plamo_cuda_batch_close": (None, [P]),
}

class Mapping(ctypes.Structure):
    """struct plamo_mapping (reference runtime/model.h:65-68)."""
    _fields_ = [("base", c_void_p), ("bytes", c_uint64)]


class WeightSpec(ctypes.Structure):
    """struct plamo_weight_spec (reference runtime/model.h:69-74)."""
    _fields_ = [("name", c_char_p), ("rank", c_uint64), ("shape", POINTER(c_uint64)),
                ("slot", POINTER(c_void_p))]


class Tensor(ctypes.Structure):
    """struct plamo_tensor (reference tests/find.c:4-7)."""
    _fields_ = [("data", c_void_p), ("bytes", c_uint64), ("rank", c_uint64), ("dims", c_uint64 * 4),
                ("reserved", c_uint64)]


assert ctypes.sizeof(Mapping) == 16 and ctypes.sizeof(WeightSpec) == 32 and ctypes.sizeof(Tensor) == 64

# name -> (restype, argtypes); exactly the entry points of include/plamo_safetensors.h.
LOADER_SIGNATURES = {
    "plamo_safetensors_view": (c_int, [P, c_uint64, P]),
    "plamo_parse_u64": (c_int, [P, P, P]),
    "plamo_find_tensor": (c_int, [P, c_uint64, c_char_p, POINTER(Tensor)]),
    "plamo_resolve_weight": (c_void_p, [POINTER(Mapping), c_uint64, c_char_p, c_uint64, POINTER(c_uint64)]),
    "plamo_bind_weights": (c_int, [POINTER(Mapping), c_uint64, POINTER(WeightSpec)]),
    "plamo_map_file": (c_int, [c_char_p, POINTER(Mapping)]),
    "plamo_unmap_file": (None, [POINTER(Mapping)]),
}


class ModelConfig(ctypes.Structure):
    """struct plamo_model_config (include/plamo_layout.h)."""
    _fields_ = [(n, c_uint64) for n in ("hidden", "layers", "query_heads", "kv_heads", "head_dim", "intermediate",
                                         "vocab", "window", "pattern", "max_position", "tied")] + \
               [(n, c_double) for n in ("local_theta", "global_theta", "yarn_factor", "yarn_original", "beta_fast",
                                        "beta_slow")]


# include/plamo_layout.h: run-time model descriptor builder
LAYOUT_SIGNATURES = {
    "plamo_model_config_profile": (c_int, [c_char_p, POINTER(ModelConfig)]),
    "plamo_model_layout_create": (c_void_p, [POINTER(ModelConfig), c_uint64, c_char_p, c_size_t]),
    "plamo_model_layout_schema": (POINTER(WeightSpec), [P]),
    "plamo_model_layout_finish": (c_int, [P]),
    "plamo_model_layout_model": (POINTER(Model), [P]),
    "plamo_model_layout_buffer_bytes": (c_uint64, [P]),
    "plamo_rope_frequencies": (None, [POINTER(ModelConfig), c_int, POINTER(ctypes.c_float)]),
    "plamo_model_layout_destroy": (None, [P]),
}


# include/plamo_tokenizer.h: the engine's tokenizer API (the assembly-level
# pieces are exported too; the reference's own C tests bind those)
TOKENIZER_SIGNATURES = {
    "plamo_tokenizer_open": (c_void_p, [c_char_p, c_char_p, c_size_t]),
    "plamo_tokenizer_close": (None, [P]),
    "plamo_tokenizer_encode": (c_uint64, [P, c_char_p, c_uint, POINTER(POINTER(c_uint32)), c_char_p, c_size_t]),
    "plamo_tokenizer_prefix": (c_uint64, [P, c_uint, POINTER(POINTER(c_uint32)), c_char_p, c_size_t]),
    "plamo_tokenizer_decode": (c_uint64, [P, c_uint32, POINTER(ctypes.c_char_p)]),
    "plamo_translation_prompt": (c_uint64, [c_char_p, c_char_p, c_char_p, c_char_p, c_uint64]),
    "plamo_translation_prefix": (c_uint64, [c_char_p, c_char_p, c_uint64]),
}

_libs = {}


def load(path=LIB_PATH):
    """Load the backend library and bind every entry point (raises if absent)."""
    path = os.path.abspath(path)
    if path in _libs:
        return _libs[path]
    if not os.path.exists(path):
        raise OSError(f"{path} is missing: run `make -C plamo-3-translate.c_b200` (or "
                      "__graft_entry__.build()); there is no non-CUDA implementation")
    lib = ctypes.CDLL(path)
    for name, (restype, argtypes) in (list(SIGNATURES.items()) + list(LOADER_SIGNATURES.items()) +
                                      list(LAYOUT_SIGNATURES.items()) + list(TOKENIZER_SIGNATURES.items())):
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _libs[path] = lib
    return lib
