"""B200-native PLaMo-3 token loop: host-side mirror of the C ABI.

The compute path is the CUDA library built from csrc/ (include/plamo_cuda.h);
this package only binds it (ctypes) and builds the model descriptor records
the reference's engine would hand to its GPU backend.
"""
from . import _abi
from ._abi import load, LIB_PATH
from .model import (PROFILES, Backend, Checkpoint, HostModel, LayerSpec, Profile, Tokenizer, concentration,
                    default_layer_specs, rope_frequencies, schema, synthetic_parameters,
                    tp_all_gather_handles, tp_segments, tp_shard_profile, tp_vocab_slice,
                    write_safetensors)

__all__ = ["_abi", "load", "LIB_PATH", "PROFILES", "Backend", "Checkpoint", "HostModel", "LayerSpec", "Profile", "Tokenizer",
           "concentration", "default_layer_specs", "rope_frequencies", "schema",
           "synthetic_parameters", "tp_all_gather_handles", "tp_segments",
           "tp_shard_profile", "tp_vocab_slice", "write_safetensors"]
