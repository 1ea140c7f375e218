"""ctypes binding of the C ABI in ``include/dflash_b200.h``.

The library is the in-tree ``lib/libdflash_b200.so`` built by ``build.py``.
There is no fallback: if it is missing or fails to load, every entry point
raises.  ctypes releases the GIL around each call.
"""
import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libdflash_b200.so")

DFLASH_OK = 0
DFLASH_ERR_INVALID = 1
DFLASH_ERR_CUDA = 2
DFLASH_ERR_OOM = 3
DFLASH_ERR_DEVICE = 4

c_int32 = ctypes.c_int32
c_float = ctypes.c_float
c_void_p = ctypes.c_void_p
c_size_t = ctypes.c_size_t


class DFlashDims(ctypes.Structure):
    _fields_ = [("hidden_size", c_int32), ("num_hidden_layers", c_int32),
                ("intermediate_size", c_int32), ("num_attention_heads", c_int32),
                ("num_key_value_heads", c_int32), ("head_dim", c_int32),
                ("vocab_size", c_int32), ("num_target_features", c_int32),
                ("rms_norm_eps", c_float), ("rope_theta", c_float),
                ("max_batch", c_int32), ("max_block", c_int32), ("max_ctx", c_int32),
                ("max_ctx_rows", c_int32)]


class DFlashLayerWeights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in
                ["wq", "sq", "wk", "sk", "wv", "sv", "wo", "so", "wg", "sg", "wu", "su", "wd", "sd",
                 "input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"]]


class DFlashWeightsView(ctypes.Structure):
    _fields_ = [("fc", c_void_p), ("hidden_norm", c_void_p), ("norm", c_void_p),
                ("lm_head", c_void_p), ("layers", ctypes.POINTER(DFlashLayerWeights))]


class DFlashLayerWeightsF32(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in
                ["wq", "wk", "wv", "wo", "wg", "wu", "wd",
                 "input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"]]


class DFlashWeightsViewF32(ctypes.Structure):
    _fields_ = [("fc", c_void_p), ("hidden_norm", c_void_p), ("norm", c_void_p),
                ("lm_head", c_void_p), ("layers", ctypes.POINTER(DFlashLayerWeightsF32))]


class DFlashForwardArgs(ctypes.Structure):
    _fields_ = [("batch", c_int32), ("block", c_int32), ("ctx_len", c_int32),
                ("rope_offset", c_int32), ("num_layers", c_int32),
                ("noise", c_void_p), ("target_hidden", c_void_p), ("out_hidden", c_void_p),
                ("out_hidden_fp32", c_int32), ("out_tokens", c_void_p), ("target_tokens", c_void_p),
                ("acc_len", c_void_p), ("correction", c_void_p),
                ("phase_events", ctypes.POINTER(c_void_p)), ("n_phase_events", c_int32),
                ("ctx_lens", ctypes.POINTER(c_int32)), ("rope_offsets", ctypes.POINTER(c_int32)),
                ("cache", c_void_p),
                ("anchor_logits", c_void_p), ("anchor_logits_ld", ctypes.c_int64),
                ("anchor_logits_bf16", c_int32), ("anchor_top_k", c_int32),
                ("target_layers", ctypes.POINTER(c_void_p)), ("target_layers_ld", ctypes.c_int64),
                ("cache_seqs", ctypes.POINTER(c_int32))]


DFLASH_PHASES = 8
PHASE_NAMES = ["start", "rope+init", "fc_gemm", "hidden_norm", "ctx_kv_gemm", "layers",
               "final_norm", "lm_head_argmax"]


EXPORTS = {
    "dflash_create": (c_int32, [ctypes.POINTER(DFlashDims), ctypes.POINTER(DFlashWeightsView),
                                ctypes.c_int, ctypes.POINTER(c_void_p)]),
    "dflash_create_f32": (c_int32, [ctypes.POINTER(DFlashDims), ctypes.POINTER(DFlashWeightsViewF32),
                                    ctypes.c_int, ctypes.POINTER(c_void_p)]),
    "dflash_forward": (c_int32, [c_void_p, ctypes.POINTER(DFlashForwardArgs), c_void_p]),
    "dflash_accept": (c_int32, [c_void_p, c_void_p, ctypes.c_int, ctypes.c_int, c_void_p, c_void_p,
                                c_void_p]),
    "dflash_quantize_q8": (c_int32, [c_void_p, ctypes.c_int, ctypes.c_int, c_void_p, c_void_p,
                                     c_void_p]),
    "dflash_device_status": (c_int32, [c_void_p, c_void_p]),
    "dflash_probe_bounded_wait": (c_int32, [c_void_p, ctypes.c_uint32, c_void_p]),
    "dflash_cache_create": (c_int32, [c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.POINTER(c_void_p)]),
    "dflash_cache_trim": (c_int32, [c_void_p, ctypes.c_int, ctypes.c_int]),
    "dflash_cache_reset": (c_int32, [c_void_p]),
    "dflash_cache_trim_seqs": (c_int32, [c_void_p, ctypes.c_int, ctypes.POINTER(c_int32),
                                         ctypes.POINTER(c_int32), ctypes.c_int]),
    "dflash_cache_reset_seqs": (c_int32, [c_void_p, ctypes.POINTER(c_int32), ctypes.c_int]),
    "dflash_cache_state": (c_int32, [c_void_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(c_int32),
                                     ctypes.POINTER(c_int32)]),
    "dflash_cache_read": (c_int32, [c_void_p, ctypes.c_int, ctypes.c_int, c_void_p, c_void_p,
                                    c_void_p]),
    "dflash_cache_destroy": (c_int32, [c_void_p]),
    "dflash_destroy": (c_int32, [c_void_p]),
    "dflash_last_launch_count": (c_int32, [c_void_p]),
    "dflash_last_error": (c_int32, [ctypes.c_char_p, c_size_t]),
    "dflash_version": (c_int32, []),
    "dflash_w8_linear": (c_int32, [c_void_p, c_void_p, ctypes.c_int, ctypes.c_int, c_void_p,
                                   ctypes.c_int, c_void_p, c_void_p]),
    "dflash_tc_gemm": (c_int32, [c_void_p, c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, c_void_p, c_void_p]),
    "dflash_soft_anchor_workspace_size": (c_size_t, [ctypes.c_int]),
    "dflash_soft_anchor": (c_int32, [c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                     ctypes.c_int, c_void_p, ctypes.c_int, c_void_p, c_void_p, c_size_t,
                                     c_void_p]),
    "dflash_attention_workspace_size": (c_size_t, [ctypes.c_int] * 5),
    "dflash_attention": (c_int32, [c_void_p, c_void_p, c_void_p, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   c_void_p, c_void_p, c_float, ctypes.c_int, ctypes.c_int,
                                   c_float, c_void_p, c_void_p, c_size_t, c_void_p]),
    "dflash_attention_noalloc": (c_int32, [c_void_p, c_void_p, c_void_p, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, c_void_p, c_void_p, c_float, ctypes.c_int,
                                           ctypes.c_int, c_float, c_void_p, c_void_p]),
    "dflash_lm_head_workspace_size": (c_size_t, [ctypes.c_int] * 4),
    "dflash_lm_head_argmax": (c_int32, [c_void_p, c_void_p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_size_t, c_void_p]),
}

_lib = None
_lock = threading.Lock()


def load():
    """Load the CUDA library (raises if it is missing: there is no fallback)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"CUDA library not built: {LIB_PATH} (run mirror-sd_b200/build.py)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in EXPORTS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error():
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.dflash_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status, what):
    """Map a status code to the reference's error types (ValueError for bad
    arguments, RuntimeError otherwise; ane/src/wrapper.rs:204-209, :397-405)."""
    if status == DFLASH_OK:
        return
    msg = f"{what} failed: {last_error()}"
    if status == DFLASH_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


def ptr(t):
    """Device pointer of a torch tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())
