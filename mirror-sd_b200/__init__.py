"""mirror-sd_b200: B200-native DFlash draft-model forward (sm_100a CUDA).

Import with ``importlib.import_module("mirror-sd_b200")`` (the folder name
carries a hyphen).  The compute path is the CUDA library ``lib/libdflash_b200.so``
(C ABI: ``include/dflash_b200.h``), built by ``build.py``.
"""
from . import _native
from .dflash import (DFlashCache, DFlashConfig, DFlashDraftModel, DFlashKVCache, DFlashWeightsF32, DFlashWeightsQ8,
                     F32Layer, Q8Layer,
                     accept, build_target_layer_ids, context_layers, extract_context_feature, key_padding_lengths,
                     quantize_q8, sample)
from .weights import synth_weights_f32, synth_weights_q8, weights_from_q8_numpy
from .generate import SpecDecodeStats, spec_generate
from .loader import load_dflash_model, load_dflash_weights, save_q8_checkpoint
from .serving import DraftServer

__all__ = ["DFlashCache", "DFlashConfig", "DFlashDraftModel", "DFlashKVCache", "DFlashWeightsF32", "DFlashWeightsQ8",
           "F32Layer", "Q8Layer",
           "accept", "build_target_layer_ids", "context_layers", "extract_context_feature", "key_padding_lengths",
           "quantize_q8", "sample",
           "synth_weights_f32", "synth_weights_q8", "weights_from_q8_numpy", "SpecDecodeStats", "spec_generate",
           "load_dflash_model", "load_dflash_weights", "save_q8_checkpoint", "DraftServer"]
