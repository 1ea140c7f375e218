"""Host side of the B200 DFlash draft model, mirroring ``mirror_sd.dflash``.

Same names, arguments and error behaviour as the reference's
``mirror_sd/dflash.py`` so a decode loop written against it
(``generate.py:591-606``) can hold this object instead:

* ``DFlashConfig`` (dflash.py:34-105) with ``from_dict`` / ``qwen3_8b`` /
  ``qwen3_4b``; ``build_target_layer_ids`` (:108-119);
  ``extract_context_feature`` (:122-130); ``sample`` (:133-136).
* ``DFlashDraftModel.__call__(noise_embedding, target_hidden, mask=None,
  cache=None)`` -> final-normed hidden states ``[b, q, H]`` (:384-403), with
  ``block_size``, ``mask_token_id``, ``config`` and a settable
  ``num_draft_layers`` (:380-382, generate.py:419-440).
* The fused draft step the reference exposes through its ANE split API
  (``prepare_forward`` / ``run_kernels`` / ``read_output`` /
  ``read_draft_tokens``, ane_model.py:538-604): lm_head + greedy argmax (+
  acceptance) inside the same call.

Every compute call goes through the CUDA library (``_native``); there is no
CPU or PyTorch fallback.  torch is used for device memory and streams only.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional

import torch

from . import _native as N


# ----------------------------------------------------------------------------
# config (mirror_sd/dflash.py:34-105)
# ----------------------------------------------------------------------------
@dataclass
class DFlashConfig:
    hidden_size: int = 4096
    num_hidden_layers: int = 5
    intermediate_size: int = 12288
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_position_embeddings: int = 40960
    vocab_size: int = 151936
    block_size: int = 16
    mask_token_id: int = 151669
    target_layer_ids: List[int] = field(default_factory=lambda: [4, 12, 19, 26, 33])
    num_target_layers: int = 36
    rope_scaling: Optional[dict] = None

    @classmethod
    def qwen3_8b(cls, num_target_layers: int = 36) -> "DFlashConfig":
        cfg = cls(num_target_layers=num_target_layers)
        cfg.target_layer_ids = build_target_layer_ids(num_target_layers, cfg.num_hidden_layers)
        return cfg

    @classmethod
    def qwen3_4b(cls, num_target_layers: int = 36) -> "DFlashConfig":
        cfg = cls(hidden_size=2560, num_hidden_layers=5, intermediate_size=6912,
                  num_attention_heads=20, num_key_value_heads=4, head_dim=128, vocab_size=151936)
        cfg.num_target_layers = num_target_layers
        cfg.target_layer_ids = build_target_layer_ids(num_target_layers, cfg.num_hidden_layers)
        return cfg

    @classmethod
    def from_dict(cls, d: dict) -> "DFlashConfig":
        """HF ``config.json`` -> config, with the reference's fall-back
        defaults (dflash.py:77-105)."""
        dc = d.get("dflash_config", {})
        nhl = d.get("num_hidden_layers", dc.get("num_hidden_layers", 5))
        ntl = dc.get("num_target_layers", d.get("num_target_layers", 36))
        cfg = cls(hidden_size=d.get("hidden_size", 4096), num_hidden_layers=nhl,
                  intermediate_size=d.get("intermediate_size", 10944),
                  num_attention_heads=d.get("num_attention_heads", 32),
                  num_key_value_heads=d.get("num_key_value_heads", 2),
                  head_dim=d.get("head_dim", 128), rms_norm_eps=d.get("rms_norm_eps", 1e-6),
                  rope_theta=d.get("rope_theta", 10000.0),
                  max_position_embeddings=d.get("max_position_embeddings", 4096),
                  vocab_size=d.get("vocab_size", 151936),
                  block_size=dc.get("block_size", d.get("block_size", 16)),
                  mask_token_id=dc.get("mask_token_id", d.get("mask_token_id", 151667)),
                  num_target_layers=ntl)
        cfg.target_layer_ids = (dc["target_layer_ids"] if "target_layer_ids" in dc
                                else build_target_layer_ids(cfg.num_target_layers, cfg.num_hidden_layers))
        if "rope_scaling" in d:
            cfg.rope_scaling = d["rope_scaling"]
        return cfg

    def to_dict(self) -> dict:
        """HF-style ``config.json`` content that ``from_dict`` reads back
        unchanged (the draft fields under ``dflash_config``)."""
        d = {"hidden_size": self.hidden_size, "num_hidden_layers": self.num_hidden_layers,
             "intermediate_size": self.intermediate_size, "num_attention_heads": self.num_attention_heads,
             "num_key_value_heads": self.num_key_value_heads, "head_dim": self.head_dim,
             "rms_norm_eps": self.rms_norm_eps, "rope_theta": self.rope_theta,
             "max_position_embeddings": self.max_position_embeddings, "vocab_size": self.vocab_size,
             "dflash_config": {"block_size": self.block_size, "mask_token_id": self.mask_token_id,
                               "num_target_layers": self.num_target_layers,
                               "target_layer_ids": list(self.target_layer_ids)}}
        if getattr(self, "rope_scaling", None) is not None:
            d["rope_scaling"] = self.rope_scaling
        return d


def build_target_layer_ids(num_target_layers: int, num_draft_layers: int) -> List[int]:
    """Evenly spaced target layers in [1, n-3] (dflash.py:108-119)."""
    if num_draft_layers == 1:
        return [num_target_layers // 2]
    start, end = 1, num_target_layers - 3
    span = end - start
    return [int(round(start + (i * span) / (num_draft_layers - 1))) for i in range(num_draft_layers)]


def extract_context_feature(hidden_states, layer_ids):
    """Concatenate captured target layers on the feature axis (dflash.py:122-130)."""
    if len(hidden_states) == len(layer_ids):
        return torch.cat(list(hidden_states), dim=-1)
    return torch.cat([hidden_states[lid + 1] for lid in layer_ids], dim=-1)


def context_layers(hidden_states, layer_ids):
    """The layers ``extract_context_feature`` would concatenate (dflash.py:122-130),
    left where they are: pass the list as ``target_hidden`` and the fc GEMM
    reads them directly, with no [*, F*H] copy."""
    if len(hidden_states) == len(layer_ids):
        return list(hidden_states)
    return [hidden_states[lid + 1] for lid in layer_ids]


def sample(logits: torch.Tensor, temperature: float = 0.0) -> torch.Tensor:
    """Greedy argmax, first index on ties (dflash.py:133-136).  Sampling with
    temperature is part of the target-side loop and is not on this path."""
    if temperature < 1e-5:
        return torch.argmax(logits, dim=-1)
    raise NotImplementedError("temperature sampling is outside the draft forward")


# ----------------------------------------------------------------------------
# weights in the reference's W8A16 format (ane_model.py:265-344)
# ----------------------------------------------------------------------------
PROJ = ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]


def key_padding_lengths(mask, batch: int, q_len: int, ctx_len: int) -> Optional[List[int]]:
    """Map the ``mask`` that ``DFlashDraftModel.__call__`` passes to SDPA
    (dflash.py:315, over the stateless step's keys ``[context ; block]``) to
    left padding: ``None`` when every key is kept, else the number of context
    rows each sequence keeps, its last ones (the block is always kept).

    Additive masks may hold 0 (kept) and values <= -1e4 or -inf (masked: their
    exponentials underflow to exactly 0 in fp32, as in the reference's ANE
    padding masks, ane_model.py:529-536); boolean masks keep True entries.  The
    mask broadcasts to [batch, heads, q_len, ctx_len + q_len] as SDPA
    broadcasts it and must be the same for every head and query.  Other masks
    (biases, right padding, masked block keys) raise NotImplementedError: left
    padding keeps every kept key at its own RoPE position once the kept rows are
    packed and each sequence's positions start at ``ctx_len - kept``."""
    m = torch.as_tensor(mask).detach().cpu()
    if m.dtype == torch.bool:
        keep = m
    else:
        mf = m.to(torch.float64)
        if not bool(((mf == 0) | (mf <= -1e4)).all()):
            raise NotImplementedError("additive masks may hold only 0 (kept) and <= -1e4 / -inf (masked)")
        keep = mf == 0
    L = ctx_len + q_len
    if keep.dim() > 4 or keep.shape[-1] != L:
        raise ValueError(f"mask must broadcast to [batch, heads, {q_len}, {L}], got {tuple(keep.shape)}")
    while keep.dim() < 4:
        keep = keep.unsqueeze(0)
    try:
        keep = keep.expand(batch, keep.shape[1], q_len, L)
    except RuntimeError as e:
        raise ValueError(f"mask must broadcast to [batch, heads, {q_len}, {L}], got {tuple(m.shape)}") from e
    rows = keep[:, :1, :1, :].expand_as(keep)
    if not bool((keep == rows).all()):
        raise NotImplementedError("the mask must be the same for every head and query row")
    rows = keep[:, 0, 0, :]
    if bool(rows.all()):
        return None
    if not bool(rows[:, ctx_len:].all()):
        raise NotImplementedError("block keys cannot be masked (the draft block attends to itself)")
    lens = []
    for i in range(batch):
        kept = int(rows[i, :ctx_len].sum())
        if kept and not bool(rows[i, ctx_len - kept:ctx_len].all()):
            raise NotImplementedError("only left padding of the context is supported (kept rows last)")
        lens.append(kept)
    return lens


@dataclass
class Q8Layer:
    """One decoder layer: int8 [out, in] + fp16 [out] per projection, fp32 norms."""
    q: dict            # name -> int8 tensor (device)
    s: dict            # name -> fp16 tensor (device)
    input_layernorm: torch.Tensor
    post_attention_layernorm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


@dataclass
class DFlashWeightsQ8:
    fc: torch.Tensor             # bf16 [H, F*H]
    hidden_norm: torch.Tensor    # fp32 [H]
    norm: torch.Tensor           # fp32 [H]
    layers: List[Q8Layer]


@dataclass
class F32Layer:
    """One decoder layer in fp32: name -> [out, in] fp32 tensor for each of
    PROJ, plus the four norm weights."""
    w: dict
    input_layernorm: torch.Tensor
    post_attention_layernorm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


@dataclass
class DFlashWeightsF32:
    """fp32 weights for the fp32-accumulate mode (a checkpoint stored in fp32,
    or a W8A16 one dequantised exactly with ``from_q8``)."""
    fc: torch.Tensor             # fp32 [H, F*H]
    hidden_norm: torch.Tensor    # fp32 [H]
    norm: torch.Tensor           # fp32 [H]
    layers: List[F32Layer]

    @staticmethod
    def from_q8(w: "DFlashWeightsQ8") -> "DFlashWeightsF32":
        """Exact fp32 copies of W8A16 weights: q * fp16(s) per output channel
        (both factors are exact in fp32, and so is their product)."""
        layers = [F32Layer(w={k: l.q[k].float() * l.s[k].float()[:, None] for k in PROJ},
                           input_layernorm=l.input_layernorm.float(),
                           post_attention_layernorm=l.post_attention_layernorm.float(),
                           q_norm=l.q_norm.float(), k_norm=l.k_norm.float()) for l in w.layers]
        return DFlashWeightsF32(fc=w.fc.float(), hidden_norm=w.hidden_norm.float(), norm=w.norm.float(),
                                layers=layers)


def quantize_q8(w: torch.Tensor):
    """Symmetric per-output-channel int8 with fp16 scales on the GPU, bit-exact
    with ``ANEDraftModel._quantize_weight_q8`` (ane_model.py:265-279).
    ``w``: [oc, ic] CUDA tensor.  Returns ``(q int8 [oc, ic], s fp16 [oc])``."""
    if not w.is_cuda:
        raise ValueError("quantize_q8 expects a CUDA tensor")
    lib = N.load()
    w32 = w.detach().to(torch.float32).contiguous()
    oc, ic = w32.shape
    q = torch.empty((oc, ic), dtype=torch.int8, device=w.device)
    s = torch.empty((oc,), dtype=torch.float16, device=w.device)
    st = torch.cuda.current_stream(w.device).cuda_stream
    N.check(lib.dflash_quantize_q8(N.ptr(w32), oc, ic, N.ptr(q), N.ptr(s), ctypes.c_void_p(st)),
            "dflash_quantize_q8")
    return q, s


# ----------------------------------------------------------------------------
# draft KV cache (dflash.py:139-212)
# ----------------------------------------------------------------------------
class _CacheStore:
    """The device cache behind one ``make_cache()`` list: K/V rows of every
    layer and sequence in device rings (include/dflash_b200.h, dflash_cache_*)."""

    def __init__(self, model, num_layers, sink_size, window_size, max_len, max_batch):
        self._lib = model._lib
        self.model = model          # keeps the handle alive while the cache exists
        self.num_layers = num_layers
        self.batch = 1              # sequences of the last forward
        ptr = ctypes.c_void_p()
        N.check(self._lib.dflash_cache_create(model._handle, num_layers, max_batch, int(sink_size),
                                              int(window_size), int(max_len), ctypes.byref(ptr)),
                "dflash_cache_create")
        self.ptr = ptr

    def close(self):
        if getattr(self, "ptr", None) is not None and self.ptr.value:
            N.check(self._lib.dflash_cache_destroy(self.ptr), "dflash_cache_destroy")
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def state(self, layer, seq=0):
        off, ln = ctypes.c_int32(), ctypes.c_int32()
        N.check(self._lib.dflash_cache_state(self.ptr, layer, seq, ctypes.byref(off), ctypes.byref(ln)),
                "dflash_cache_state")
        return off.value, ln.value

    def trim(self, layer, n):
        N.check(self._lib.dflash_cache_trim(self.ptr, layer, int(n)), "dflash_cache_trim")

    def trim_seqs(self, layer, seqs, counts):
        seqs, counts = [int(s) for s in seqs], [int(c) for c in counts]
        if len(seqs) != len(counts):
            raise ValueError("seqs and counts differ in length")
        sa = (ctypes.c_int32 * len(seqs))(*seqs)
        ca = (ctypes.c_int32 * len(counts))(*counts)
        N.check(self._lib.dflash_cache_trim_seqs(self.ptr, layer, sa, ca, len(seqs)), "dflash_cache_trim_seqs")

    def reset(self):
        N.check(self._lib.dflash_cache_reset(self.ptr), "dflash_cache_reset")

    def reset_seqs(self, seqs):
        seqs = [int(s) for s in seqs]
        sa = (ctypes.c_int32 * len(seqs))(*seqs)
        N.check(self._lib.dflash_cache_reset_seqs(self.ptr, sa, len(seqs)), "dflash_cache_reset_seqs")

    def read(self, layer):
        """(keys, values) f16 [b, NKV, len, 128] in logical order, or a list of
        per-sequence [NKV, len_s, 128] tensors when the lengths differ."""
        cfg = self.model.config
        ks, vs = [], []
        st = torch.cuda.current_stream(self.model.device)
        for seq in range(self.batch):
            ln = self.state(layer, seq)[1]
            k = torch.empty((cfg.num_key_value_heads, ln, cfg.head_dim), dtype=torch.float16,
                            device=self.model.device)
            v = torch.empty_like(k)
            N.check(self._lib.dflash_cache_read(self.ptr, layer, seq, N.ptr(k), N.ptr(v),
                                                ctypes.c_void_p(st.cuda_stream)), "dflash_cache_read")
            ks.append(k)
            vs.append(v)
        if len({k.shape[1] for k in ks}) == 1:
            return torch.stack(ks), torch.stack(vs)
        return ks, vs


class DFlashKVCache:
    """One layer of the draft cache (dflash.py:139-212): ``offset``, ``keys`` /
    ``values`` and ``trim(n)`` with the reference's meaning.  Appending, with
    the sink + window eviction of ``update_and_fetch``, happens inside the
    draft forward on the device."""

    def __init__(self, store: _CacheStore, layer: int, sink_size: int, window_size: int):
        self._store = store
        self.layer = layer
        self.sink_size = int(sink_size)
        self.window_size = int(window_size)

    @property
    def offset(self) -> int:
        return self._store.state(self.layer, 0)[0]

    def _kv(self):
        if all(self._store.state(self.layer, s)[1] == 0 for s in range(self._store.batch)):
            return None, None
        return self._store.read(self.layer)

    @property
    def keys(self):
        return self._kv()[0]

    @property
    def values(self):
        return self._kv()[1]

    def trim(self, n: int):
        self._store.trim(self.layer, n)

    def state(self):
        k, v = self._kv()
        return [] if k is None else [k, v]


class DFlashCache(list):
    """``make_cache()`` result: one ``DFlashKVCache`` per draft layer over one
    device store (``generate.py`` trims each entry after every draft step)."""

    def __init__(self, store: _CacheStore, sink_size: int, window_size: int):
        super().__init__(DFlashKVCache(store, l, sink_size, window_size)
                         for l in range(store.num_layers))
        self.store = store

    def reset(self):
        self.store.reset()

    def trim_seqs(self, seqs, counts):
        """Per-sequence rollback on every layer: cache sequence seqs[i] drops
        its last counts[i] rows (one entry per sequence of a batched decode)."""
        self.store.trim_seqs(-1, seqs, counts)

    def reset_seqs(self, seqs):
        """Empty the listed sequences (offset 0, no rows)."""
        self.store.reset_seqs(seqs)


# ----------------------------------------------------------------------------
# the draft model
# ----------------------------------------------------------------------------
class DFlashDraftModel:
    """B200 DFlash draft model with the reference's call signature.

    ``lm_head`` is the target's (tied) embedding matrix [V, H] in bf16; it is
    referenced, not copied (generate.py:435-436: the draft does not own it).

    Capacities: ``max_batch`` sequences of up to ``max_block`` block rows and
    ``max_ctx`` new context rows each per step; ``max_ctx_rows`` bounds the
    context rows of one step over all sequences (0: max_batch * max_ctx).
    Above 64 block rows per step the projections run as dense tensor-core
    GEMMs over f16 copies of the int8 weights (twice their memory).

    With ``DFlashWeightsF32`` weights (and an fp32 ``lm_head``) the model runs
    in fp32-accumulate mode: fp32 weights, activations and sums on the CUDA
    cores, inputs taken as fp32, hidden states returned in fp32.  That mode
    is stateless (no cache, soft anchor or in-place target layers).
    """

    def __init__(self, config: DFlashConfig, weights, lm_head: torch.Tensor,
                 max_batch: int = 1, max_ctx: int = 4096, max_block: Optional[int] = None,
                 device=None, max_ctx_rows: int = 0):
        self.config = config
        self.block_size = config.block_size
        self.mask_token_id = config.mask_token_id
        self.num_draft_layers = config.num_hidden_layers
        self.device = torch.device(device) if device is not None else weights.fc.device
        if self.device.type != "cuda":
            raise ValueError("DFlashDraftModel runs on a CUDA device only")
        self._lib = N.load()
        self.fp32 = isinstance(weights, DFlashWeightsF32)
        self._act_dtype = torch.float32 if self.fp32 else torch.bfloat16
        self._lm_head = lm_head.to(device=self.device, dtype=self._act_dtype).contiguous()
        self._weights = weights
        H, F = config.hidden_size, len(config.target_layer_ids)
        if tuple(weights.fc.shape) != (H, F * H):
            raise ValueError(f"fc weight shape {tuple(weights.fc.shape)} != {(H, F * H)}")
        if tuple(self._lm_head.shape) != (config.vocab_size, H):
            raise ValueError(f"lm_head shape {tuple(self._lm_head.shape)} != {(config.vocab_size, H)}")
        self.max_batch = int(max_batch)
        self.max_ctx = int(max_ctx)
        self.max_block = int(max_block or config.block_size)
        dims = N.DFlashDims(
            hidden_size=H, num_hidden_layers=config.num_hidden_layers,
            intermediate_size=config.intermediate_size,
            num_attention_heads=config.num_attention_heads,
            num_key_value_heads=config.num_key_value_heads, head_dim=config.head_dim,
            vocab_size=config.vocab_size, num_target_features=F,
            rms_norm_eps=config.rms_norm_eps, rope_theta=config.rope_theta,
            max_batch=self.max_batch, max_block=self.max_block, max_ctx=self.max_ctx,
            max_ctx_rows=int(max_ctx_rows))
        keep = []  # tensors whose pointers the create call reads

        def dev(t, dtype):
            t = t.to(device=self.device, dtype=dtype).contiguous()
            keep.append(t)
            return t.data_ptr()

        if len(weights.layers) != config.num_hidden_layers:
            raise ValueError(f"{len(weights.layers)} layers of weights for {config.num_hidden_layers} layers")
        handle = ctypes.c_void_p()
        if self.fp32:
            layers = (N.DFlashLayerWeightsF32 * config.num_hidden_layers)()
            for i, lw in enumerate(weights.layers):
                L = layers[i]
                for name in PROJ:
                    setattr(L, name, dev(lw.w[name], torch.float32))
                L.input_layernorm = dev(lw.input_layernorm, torch.float32)
                L.post_attention_layernorm = dev(lw.post_attention_layernorm, torch.float32)
                L.q_norm = dev(lw.q_norm, torch.float32)
                L.k_norm = dev(lw.k_norm, torch.float32)
            view = N.DFlashWeightsViewF32(fc=dev(weights.fc, torch.float32),
                                          hidden_norm=dev(weights.hidden_norm, torch.float32),
                                          norm=dev(weights.norm, torch.float32),
                                          lm_head=self._lm_head.data_ptr(), layers=layers)
            torch.cuda.synchronize(self.device)
            N.check(self._lib.dflash_create_f32(ctypes.byref(dims), ctypes.byref(view),
                                                self.device.index or 0, ctypes.byref(handle)),
                    "dflash_create_f32")
        else:
            layers = (N.DFlashLayerWeights * config.num_hidden_layers)()
            for i, lw in enumerate(weights.layers):
                L = layers[i]
                for name in PROJ:
                    setattr(L, name, dev(lw.q[name], torch.int8))
                    setattr(L, "s" + name[1], dev(lw.s[name], torch.float16))
                L.input_layernorm = dev(lw.input_layernorm, torch.float32)
                L.post_attention_layernorm = dev(lw.post_attention_layernorm, torch.float32)
                L.q_norm = dev(lw.q_norm, torch.float32)
                L.k_norm = dev(lw.k_norm, torch.float32)
            view = N.DFlashWeightsView(fc=dev(weights.fc, torch.bfloat16),
                                       hidden_norm=dev(weights.hidden_norm, torch.float32),
                                       norm=dev(weights.norm, torch.float32),
                                       lm_head=self._lm_head.data_ptr(), layers=layers)
            torch.cuda.synchronize(self.device)
            N.check(self._lib.dflash_create(ctypes.byref(dims), ctypes.byref(view),
                                            self.device.index or 0, ctypes.byref(handle)),
                    "dflash_create")
        self._handle = handle
        # ANE-style split API state
        self._pending = None
        self._out_hidden = None
        self._out_tokens = None
        self.b_logits = True  # lm_head + argmax is fused (read_draft_tokens is valid)

    # -- lifecycle -----------------------------------------------------------
    def close(self):
        if getattr(self, "_handle", None) is not None and self._handle.value:
            N.check(self._lib.dflash_destroy(self._handle), "dflash_destroy")
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def make_cache(self, sink_size: int = 64, window_size: int = 1024,
                   max_len: Optional[int] = None, max_batch: Optional[int] = None) -> "DFlashCache":
        """Per-layer draft caches (dflash.py:405-406).  Eviction runs when both
        sink_size and window_size are positive; otherwise the cache holds up to
        ``max_len`` rows per sequence (default: 4 * (max_ctx + max_block))."""
        if max_len is None:
            max_len = 4 * (self.max_ctx + self.max_block)
        store = _CacheStore(self, self.num_draft_layers, sink_size, window_size, max_len,
                            max_batch or self.max_batch)
        return DFlashCache(store, sink_size, window_size)

    def device_status(self) -> None:
        """Reads and clears the handle's device error word: raises
        RuntimeError when a bounded device-side wait gave up since the last
        check (every mbarrier wait of the kernels is bounded)."""
        N.check(self._lib.dflash_device_status(self._handle, self._stream()), "dflash_device_status")

    def probe_bounded_wait(self, polls: int = 1 << 14) -> None:
        """Failure-reporting self test: enqueue one bounded wait that nothing
        completes; the next device_status() raises, and the context stays
        usable."""
        N.check(self._lib.dflash_probe_bounded_wait(self._handle, int(polls), self._stream()),
                "dflash_probe_bounded_wait")

    def set_block_size(self, new_block: int) -> None:
        """Change the active block size (ane_model.py:611-630: ValueError
        outside [1, capacity])."""
        if new_block < 1 or new_block > self.max_block:
            raise ValueError(f"new_seq_q={new_block} must be in [1, {self.max_block}]")
        self.block_size = new_block
        self.config.block_size = new_block

    # -- core step -----------------------------------------------------------
    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _layer_rows(self, t, H):
        """One target layer as [rows, H] bf16 rows on the device with unit
        column stride and a 16-byte row pitch (a view when it already is)."""
        t = t.to(self.device, torch.bfloat16) if (t.device != self.device or t.dtype != torch.bfloat16) else t
        if t.shape[-1] != H:
            raise ValueError(f"target layer width {t.shape[-1]} differs from hidden size {H}")
        try:
            r = t.view(-1, H)
        except RuntimeError:
            r = t.reshape(-1, H).contiguous()
        if r.stride(1) != 1 or r.stride(0) % 8 or r.data_ptr() % 16:
            r = r.contiguous()
        return r

    def _as_dev(self, t, dtype):
        if t.device != self.device:
            t = t.to(self.device, non_blocking=True)
        return t.to(dtype).contiguous()

    def draft_step(self, noise_embedding, target_hidden, rope_offset: int = 0,
                   target_tokens=None, want_hidden: bool = True, want_tokens: bool = True,
                   out_hidden=None, out_tokens=None, acc_len=None, correction=None,
                   hidden_fp32: bool = False, phase_events=None, cache=None, ctx_lens=None,
                   rope_offsets=None, anchor_logits=None, anchor_top_k: int = 8, cache_seqs=None):
        """One draft step on the device: final-normed hidden states (bf16, or
        fp32 with ``hidden_fp32``), greedy draft ids for rows 1..q-1 and, given
        the verifier's posterior ``target_tokens`` [b, q], the accepted length
        and correction token.

        ``target_hidden`` is [b, ctx, F*H], or with ``ctx_lens`` (one count per
        sequence) the packed rows [sum(ctx_lens), F*H].  With ``cache`` (from
        ``make_cache``) the rows are appended to it and the step attends to
        everything it holds; without, positions start at ``rope_offset`` (or
        ``rope_offsets`` per sequence).  ``phase_events``: optional list of 8
        ``torch.cuda.Event`` recorded at the phase boundaries.

        ``anchor_logits`` [b, V] (fp32 or bf16; the previous verify step's
        logits at each sequence's correction position) replaces row 0 of every
        block with the soft anchor: the softmax-weighted sum of the
        ``anchor_top_k`` most likely tokens' embeddings (generate.py:1422-1436),
        computed on the device inside the step.

        ``cache_seqs`` (with ``cache``): the cache sequence each of the b
        sequences of this step reads and extends (distinct indices below the
        cache's max_batch), so a step may cover any subset of the cache's
        sequences; default 0..b-1."""
        noise = self._as_dev(noise_embedding, self._act_dtype)
        if noise.dim() != 3:
            raise ValueError("noise_embedding [b, q, H] expected")
        b, q, H = noise.shape
        F = len(self.config.target_layer_ids)
        layers = None
        if self.fp32 and (isinstance(target_hidden, (list, tuple)) or cache is not None
                          or anchor_logits is not None):
            raise ValueError("the fp32-accumulate mode is stateless: no cache, anchor_logits or "
                             "in-place target layers")
        if isinstance(target_hidden, (list, tuple)):
            # the F selected target layers, each [b, ctx, H] (or packed rows
            # with ctx_lens): the fc GEMM reads them in place
            if len(target_hidden) != F:
                raise ValueError(f"target_hidden needs {F} layers, got {len(target_hidden)}")
            layers = [self._layer_rows(t, H) for t in target_hidden]
            if len({tuple(t.shape) for t in layers}) != 1:
                raise ValueError("target layers differ in shape")
            if len({t.stride(0) for t in layers}) != 1:
                layers = [t.contiguous() for t in layers]
            th = layers[0].new_empty((0,))
            rows = layers[0].shape[0]
            src_shape = tuple(target_hidden[0].shape)
        else:
            th = self._as_dev(target_hidden, self._act_dtype)
            if th.shape[-1] != F * H:
                raise ValueError("hidden size mismatch")
            rows = th.reshape(-1, th.shape[-1]).shape[0]
            src_shape = tuple(th.shape)
        lens_arr = offs_arr = None
        if ctx_lens is not None:
            lens = [int(c) for c in ctx_lens]
            if len(lens) != b:
                raise ValueError(f"ctx_lens needs {b} entries")
            if layers is None:
                th = th.reshape(-1, th.shape[-1])
            if rows != sum(lens):
                raise ValueError(f"packed target_hidden has {rows} rows, ctx_lens sum to {sum(lens)}")
            lens_arr = (ctypes.c_int32 * b)(*lens)
            ctx_len = max(lens) if lens else 0
        else:
            if len(src_shape) != 3 or src_shape[0] != b:
                raise ValueError("noise_embedding [b, q, H] and target_hidden [b, ctx, F*H] "
                                 "(or F layers [b, ctx, H]) expected")
            ctx_len = src_shape[1]
        if H != self.config.hidden_size:
            raise ValueError("hidden size mismatch")
        if rope_offsets is not None:
            if len(rope_offsets) != b:
                raise ValueError(f"rope_offsets needs {b} entries")
            offs_arr = (ctypes.c_int32 * b)(*[int(o) for o in rope_offsets])
        store = None
        if cache is not None:
            store = getattr(cache, "store", None)
            if not isinstance(store, _CacheStore):
                raise ValueError("cache must come from this model's make_cache()")
        if self.fp32:
            hidden_fp32 = True
        if want_hidden and out_hidden is None:
            out_hidden = torch.empty((b, q, H), dtype=torch.float32 if hidden_fp32 else torch.bfloat16,
                                     device=self.device)
        if out_hidden is not None:
            hidden_fp32 = out_hidden.dtype == torch.float32
            if self.fp32 and not hidden_fp32:
                raise ValueError("an fp32-accumulate model writes fp32 hidden states")
        if (want_tokens or target_tokens is not None) and out_tokens is None:
            out_tokens = torch.empty((b, q - 1), dtype=torch.int32, device=self.device)
        al = None
        if anchor_logits is not None:
            al = anchor_logits if anchor_logits.dim() == 2 else anchor_logits.reshape(b, -1)
            if al.dtype not in (torch.float32, torch.bfloat16):
                al = al.to(torch.float32)
            if al.device != self.device:
                al = al.to(self.device)
            if al.stride(-1) != 1:
                al = al.contiguous()
            if al.shape != (b, self.config.vocab_size):
                raise ValueError(f"anchor_logits must be [{b}, {self.config.vocab_size}], got {tuple(al.shape)}")
        tt = None
        if target_tokens is not None:
            tt = self._as_dev(target_tokens, torch.int32)
            if acc_len is None:
                acc_len = torch.empty((b,), dtype=torch.int32, device=self.device)
            if correction is None:
                correction = torch.empty((b,), dtype=torch.int32, device=self.device)
        args = N.DFlashForwardArgs(
            batch=b, block=q, ctx_len=ctx_len, rope_offset=int(rope_offset),
            num_layers=int(self.num_draft_layers),
            noise=noise.data_ptr(),
            target_hidden=th.data_ptr() if layers is None and th.numel() else None,
            out_hidden=out_hidden.data_ptr() if out_hidden is not None else None,
            out_hidden_fp32=int(bool(hidden_fp32)),
            out_tokens=out_tokens.data_ptr() if out_tokens is not None else None,
            target_tokens=tt.data_ptr() if tt is not None else None,
            acc_len=acc_len.data_ptr() if acc_len is not None else None,
            correction=correction.data_ptr() if correction is not None else None,
            ctx_lens=lens_arr, rope_offsets=offs_arr, cache=store.ptr if store is not None else None,
            anchor_logits=al.data_ptr() if al is not None else None,
            anchor_logits_ld=al.stride(0) if al is not None else 0,
            anchor_logits_bf16=int(al is not None and al.dtype == torch.bfloat16),
            anchor_top_k=int(anchor_top_k))
        if layers is not None and rows > 0:
            ptrs = (ctypes.c_void_p * F)(*[t.data_ptr() for t in layers])
            args.target_layers = ctypes.cast(ptrs, ctypes.POINTER(ctypes.c_void_p))
            args.target_layers_ld = layers[0].stride(0)
        if cache_seqs is not None:
            cs = [int(c) for c in cache_seqs]
            if len(cs) != b:
                raise ValueError(f"cache_seqs needs {b} entries")
            cs_arr = (ctypes.c_int32 * b)(*cs)
            args.cache_seqs = cs_arr
        if phase_events is not None:
            if len(phase_events) < N.DFLASH_PHASES:
                raise ValueError(f"phase_events needs {N.DFLASH_PHASES} events")
            arr = (ctypes.c_void_p * len(phase_events))(*[ctypes.c_void_p(e.cuda_event) for e in phase_events])
            args.phase_events = ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))
            args.n_phase_events = len(phase_events)
        N.check(self._lib.dflash_forward(self._handle, ctypes.byref(args), self._stream()),
                "dflash_forward")
        if store is not None:
            store.batch = max(store.batch, b if cache_seqs is None else max(int(c) for c in cache_seqs) + 1)
        return out_hidden, out_tokens, acc_len, correction

    def __call__(self, noise_embedding, target_hidden, mask=None, cache=None, **kwargs):
        """``DFlashDraftModel.__call__`` (dflash.py:384-403): returns the
        final-normed hidden states [b, q, H] (bf16; fp32 in fp32-accumulate mode)."""
        if mask is not None:
            b, q = int(noise_embedding.shape[0]), int(noise_embedding.shape[1])
            if cache is not None or isinstance(target_hidden, (list, tuple)):
                # with a cache (or target layers read in place) only masks that
                # keep every key are taken
                m = torch.as_tensor(mask)
                if not bool((m if m.dtype == torch.bool else m == 0).all()):
                    raise NotImplementedError("a masking mask needs cache=None and a [b, ctx, F*H] target_hidden")
            else:
                C = int(target_hidden.shape[1])
                lens = key_padding_lengths(mask, b, q, C)
                if lens is not None:
                    th = target_hidden if isinstance(target_hidden, torch.Tensor) else torch.as_tensor(target_hidden)
                    packed = torch.cat([th[i, C - c:] for i, c in enumerate(lens)], dim=0)
                    hidden, _, _, _ = self.draft_step(noise_embedding, packed, ctx_lens=lens,
                                                      rope_offsets=[C - c for c in lens],
                                                      want_hidden=True, want_tokens=False)
                    return hidden
        hidden, _, _, _ = self.draft_step(noise_embedding, target_hidden, cache=cache,
                                          want_hidden=True, want_tokens=False)
        return hidden

    def draft_tokens(self, noise_embedding, target_hidden, rope_offset: int = 0, cache=None,
                     anchor_logits=None, anchor_top_k: int = 8):
        """lm_head + greedy argmax fused on the device: ids [b, q-1] for rows
        1..q-1 (generate.py:604-606); ``anchor_logits`` as in draft_step."""
        _, toks, _, _ = self.draft_step(noise_embedding, target_hidden, rope_offset,
                                        want_hidden=False, want_tokens=True, cache=cache,
                                        anchor_logits=anchor_logits, anchor_top_k=anchor_top_k)
        return toks

    # -- ANE-style split API (ane_model.py:538-604) ---------------------------
    def prepare_forward(self, noise_embedding, precomputed_context, cache, target_hidden):
        if precomputed_context is not None:
            raise ValueError("precomputed_context is not used: fc + hidden_norm run on the device")
        self._pending = (noise_embedding, target_hidden, cache)

    def run_kernels(self):
        if self._pending is None:
            raise RuntimeError("prepare_forward() must be called first")
        noise, th, cache = self._pending
        self._out_hidden, self._out_tokens, _, _ = self.draft_step(noise, th, cache=cache)
        self._pending = None

    def read_output(self):
        if self._out_hidden is None:
            raise RuntimeError("run_kernels() has not produced an output")
        return self._out_hidden

    def read_draft_tokens(self):
        """[1, q] ids like the reference (position 0 is the anchor row, whose
        id is not computed and reads as -1); callers slice [:, 1:q]."""
        if self._out_tokens is None:
            raise RuntimeError("run_kernels() has not produced tokens")
        b = self._out_tokens.shape[0]
        head = torch.full((b, 1), -1, dtype=torch.int32, device=self.device)
        return torch.cat([head, self._out_tokens], dim=1)


def accept(draft_tokens: torch.Tensor, target_tokens: torch.Tensor):
    """Longest matching prefix on the device (generate.py:722-728).
    draft [b, q-1], target [b, q] int32 CUDA tensors -> (acc_len [b], correction [b])."""
    lib = N.load()
    d = draft_tokens.to(torch.int32).contiguous()
    t = target_tokens.to(torch.int32).contiguous()
    if d.dim() == 1:
        d, t = d[None], t[None]
    b, q = t.shape
    if d.shape != (b, q - 1):
        raise ValueError("draft must be [b, q-1] for target [b, q]")
    acc = torch.empty((b,), dtype=torch.int32, device=t.device)
    cor = torch.empty((b,), dtype=torch.int32, device=t.device)
    st = ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
    N.check(lib.dflash_accept(N.ptr(d), N.ptr(t), b, q, N.ptr(acc), N.ptr(cor), st), "dflash_accept")
    return acc, cor
