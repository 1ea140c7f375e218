"""CPU oracle for the DFlash draft-model forward.  TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU in fp32 (or fp64), the algorithm of the
reference's DFlash draft model so the CUDA path can be checked against it.
It is imported only by ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``; the product
(the ``mirror-sd_b200`` package and its CUDA library) never imports it.

Pinning.  The reference runs on MLX, which is not installable here.  The
composition of the forward (projection order, concat of context and block
rows, per-head norms, RoPE offsets, GQA repeat, residuals, cache window and
trim) is pinned by running the reference's own ``mirror_sd/dflash.py``
through an MLX-API shim and freezing the outputs as fixtures
(``tests/golden/gen_golden.py``).  The W8A16 quantiser is pinned bit-exactly
against the reference's own ``ANEDraftModel._quantize_weight_q8`` (pure
numpy).  The numerics of the MLX primitives themselves
(``mx.fast.rms_norm``, ``mx.fast.rope``, ``mx.fast.scaled_dot_product_attention``)
are restated from their documented semantics and are NOT pinned against MLX.

All line citations are ``mirror_sd/...`` paths inside the reference project.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch


# --------------------------------------------------------------------------
# configuration (mirror_sd/dflash.py:34-105)
# --------------------------------------------------------------------------
@dataclass
class OracleConfig:
    hidden_size: int = 4096
    num_hidden_layers: int = 5
    intermediate_size: int = 12288
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    vocab_size: int = 151936
    block_size: int = 16
    mask_token_id: int = 151669
    num_target_features: int = 5
    target_layer_ids: List[int] = field(default_factory=lambda: [4, 12, 19, 26, 33])


def build_target_layer_ids(num_target_layers: int, num_draft_layers: int) -> List[int]:
    """mirror_sd/dflash.py:108-119 (python round = half-to-even, as there)."""
    if num_draft_layers == 1:
        return [num_target_layers // 2]
    start, end = 1, num_target_layers - 3
    span = end - start
    return [int(round(start + (i * span) / (num_draft_layers - 1)))
            for i in range(num_draft_layers)]


def extract_context_feature(hidden_states, layer_ids):
    """mirror_sd/dflash.py:122-130: concat on the feature axis; when the list
    holds every layer (embedding first) select ``layer_ids`` shifted by one."""
    if len(hidden_states) == len(layer_ids):
        return torch.cat(list(hidden_states), dim=-1)
    return torch.cat([hidden_states[i + 1] for i in layer_ids], dim=-1)


# --------------------------------------------------------------------------
# W8A16 quantiser (mirror_sd/ane_model.py:265-279)
# --------------------------------------------------------------------------
def quantize_q8(w: np.ndarray):
    """Symmetric per-output-channel int8 with fp16 scales.

    ``s = max|w_row| / 127`` in fp32 (an all-zero row uses ``1/127``);
    ``q = clip(round_half_even(w / s), -127, 127)`` with the fp32 scale; the
    scale is then stored as fp16.  Returns ``(q int8 [oc, ic], s fp16 [oc])``.
    """
    w = np.asarray(w, dtype=np.float32)
    maxv = np.abs(w).max(axis=1)
    maxv = np.where(maxv == 0, np.float32(1.0), maxv).astype(np.float32)
    s = (maxv / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.round(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s.astype(np.float16)


def dequantize_q8(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """``w ~= q * fp16(s)`` evaluated in fp32 (the oracle's weight view)."""
    return q.astype(np.float32) * s.astype(np.float32)[:, None]


# --------------------------------------------------------------------------
# MLX primitive restatements
# --------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """``mx.fast.rms_norm`` as used by ``nn.RMSNorm``: x * rsqrt(mean(x^2)+eps) * w
    over the last axis (dflash.py:251-252, :338-339, :378-379)."""
    ms = (x * x).mean(dim=-1, keepdim=True)
    return x * torch.rsqrt(ms + eps) * w


def rope_inv_freq(head_dim: int, theta: float, dtype=torch.float32) -> torch.Tensor:
    """inv_freq_i = theta^(-2i/d), i < d/2, evaluated in fp64 then cast."""
    i = torch.arange(head_dim // 2, dtype=torch.float64)
    return (theta ** (-2.0 * i / head_dim)).to(dtype)


def rope_neox(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """``mx.fast.rope(traditional=False, scale=1)`` (dflash.py:263-275):
    split-half rotation on the last axis, angle = position * inv_freq.
    ``x`` is [..., S, D]; ``positions`` is [S]."""
    d = x.shape[-1]
    half = d // 2
    inv = rope_inv_freq(d, theta, x.dtype)
    ang = positions.to(x.dtype)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


def sdpa(q, k, v, scale, mask=None):
    """``mx.fast.scaled_dot_product_attention`` (dflash.py:315-317): full,
    non-causal attention; an additive ``mask`` is added to the scores and a
    boolean one keeps its True entries, broadcast to [b, heads, q, keys]."""
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    if mask is not None:
        m = torch.as_tensor(mask)
        s = s.masked_fill(~m, float("-inf")) if m.dtype == torch.bool else s + m.to(s.dtype)
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, v)


def silu(x):
    return x * torch.sigmoid(x)


# --------------------------------------------------------------------------
# KV cache (mirror_sd/dflash.py:139-212)
# --------------------------------------------------------------------------
class OracleKVCache:
    """Append, sink+window eviction after append, and ``trim(n)``."""

    def __init__(self, sink_size: int = 0, window_size: int = 0):
        self.keys = None
        self.values = None
        self.offset = 0
        self.sink_size = int(sink_size)
        self.window_size = int(window_size)

    def update_and_fetch(self, k, v):          # dflash.py:168-177
        if self.keys is None:
            self.keys, self.values = k, v
        else:
            self.keys = torch.cat([self.keys, k], dim=2)
            self.values = torch.cat([self.values, v], dim=2)
        self.offset += k.shape[2]
        self._apply_window()
        return self.keys, self.values

    def _apply_window(self):                   # dflash.py:179-193
        if self.sink_size <= 0 or self.window_size <= 0 or self.keys is None:
            return
        n = self.keys.shape[2]
        if n <= self.sink_size + self.window_size:
            return
        self.keys = torch.cat([self.keys[:, :, :self.sink_size],
                               self.keys[:, :, -self.window_size:]], dim=2)
        self.values = torch.cat([self.values[:, :, :self.sink_size],
                                 self.values[:, :, -self.window_size:]], dim=2)

    def trim(self, n: int):                    # dflash.py:195-207
        if self.keys is not None and n > 0:
            keep = max(self.keys.shape[2] - n, 0)
            self.keys = self.keys[..., :keep, :]
            self.values = self.values[..., :keep, :]
            self.offset -= n


# --------------------------------------------------------------------------
# weights
# --------------------------------------------------------------------------
@dataclass
class OracleLayer:
    wq: torch.Tensor
    wk: torch.Tensor
    wv: torch.Tensor
    wo: torch.Tensor
    wg: torch.Tensor
    wu: torch.Tensor
    wd: torch.Tensor
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


@dataclass
class OracleWeights:
    fc: torch.Tensor            # [H, F*H]
    hidden_norm: torch.Tensor   # [H]
    norm: torch.Tensor          # [H]
    lm_head: torch.Tensor       # [V, H] (tied embedding)
    layers: List[OracleLayer]

    def to(self, dtype):
        cv = lambda t: t.to(dtype)
        return OracleWeights(
            cv(self.fc), cv(self.hidden_norm), cv(self.norm), cv(self.lm_head),
            [OracleLayer(*[cv(getattr(l, f)) for f in OracleLayer.__dataclass_fields__])
             for l in self.layers])


# --------------------------------------------------------------------------
# forward (mirror_sd/dflash.py:236-403)
# --------------------------------------------------------------------------
def attention(cfg: OracleConfig, lw: OracleLayer, h, ctx, cache=None, mask=None):
    """Qwen3DFlashAttention.__call__ (dflash.py:277-319)."""
    b, q_len, _ = h.shape
    c_len = ctx.shape[1]
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    kv_in = torch.cat([ctx, h], dim=1)                         # :287
    kv_len = c_len + q_len
    q = h @ lw.wq.T                                            # :290
    q = rms_norm(q.reshape(b, q_len, nh, hd), lw.q_norm, cfg.rms_norm_eps).transpose(1, 2)
    k = kv_in @ lw.wk.T                                        # :293
    v = kv_in @ lw.wv.T
    k = rms_norm(k.reshape(b, kv_len, nkv, hd), lw.k_norm, cfg.rms_norm_eps).transpose(1, 2)
    v = v.reshape(b, kv_len, nkv, hd).transpose(1, 2)
    off = cache.offset if cache is not None else 0             # :299-302
    q = rope_neox(q, torch.arange(q_len) + off + c_len, cfg.rope_theta)   # :304
    k = rope_neox(k, torch.arange(kv_len) + off, cfg.rope_theta)          # :305
    if cache is not None:
        k, v = cache.update_and_fetch(k, v)                    # :307-308
    rep = nh // nkv
    if rep > 1:                                                # :310-313 (mx.repeat)
        k = torch.repeat_interleave(k, rep, dim=1)
        v = torch.repeat_interleave(v, rep, dim=1)
    o = sdpa(q, k, v, hd ** -0.5, mask)                        # :315-317
    o = o.transpose(1, 2).reshape(b, q_len, nh * hd)
    return o @ lw.wo.T                                         # :319


def mlp(lw: OracleLayer, x):
    """Qwen3MLP (dflash.py:329-330)."""
    return (silu(x @ lw.wg.T) * (x @ lw.wu.T)) @ lw.wd.T


def decoder_layer(cfg, lw, h, ctx, cache=None, mask=None):
    """Qwen3DFlashDecoderLayer.__call__ (dflash.py:341-362)."""
    h = h + attention(cfg, lw, rms_norm(h, lw.in_norm, cfg.rms_norm_eps), ctx, cache, mask)
    return h + mlp(lw, rms_norm(h, lw.post_norm, cfg.rms_norm_eps))


def context_projection(cfg, w: OracleWeights, target_hidden):
    """ctx = hidden_norm(fc(target_hidden)) (dflash.py:392)."""
    return rms_norm(target_hidden @ w.fc.T, w.hidden_norm, cfg.rms_norm_eps)


def draft_forward(cfg: OracleConfig, w: OracleWeights, noise, target_hidden,
                  cache: Optional[list] = None, num_layers: Optional[int] = None, mask=None):
    """DFlashDraftModel.__call__ (dflash.py:384-403): returns the final-normed
    hidden states [b, q_len, H]."""
    h = noise
    ctx = context_projection(cfg, w, target_hidden)
    n = len(w.layers) if num_layers is None else num_layers
    for i in range(n):
        h = decoder_layer(cfg, w.layers[i], h, ctx, None if cache is None else cache[i], mask)
    return rms_norm(h, w.norm, cfg.rms_norm_eps)


# --------------------------------------------------------------------------
# lm_head, greedy argmax, acceptance
# --------------------------------------------------------------------------
def draft_logits(w: OracleWeights, hidden, block_size: int):
    """Tied lm_head on the last block_size-1 rows (generate.py:604-605)."""
    return hidden[:, -(block_size - 1):, :] @ w.lm_head.T


def greedy(logits):
    """argmax over the vocab, first index on ties (dflash.py:133-136;
    ANE read_argmax with a strict '>' in ane/src/wrapper.rs:108-140)."""
    return torch.argmax(logits, dim=-1).to(torch.int32)


def top2_margin(logits):
    """top-1 minus top-2 logit per row (diagnostic for argmax near-ties)."""
    t = torch.topk(logits, 2, dim=-1).values
    return t[..., 0] - t[..., 1]


def accept(draft_tokens, target_tokens):
    """Longest matching prefix (generate.py:722-728): ``draft`` has B-1
    entries, ``target`` (the verifier's posterior) has B; returns
    ``(acc, correction=target[acc])``."""
    acc = 0
    for i in range(len(draft_tokens)):
        if int(draft_tokens[i]) == int(target_tokens[i]):
            acc += 1
        else:
            break
    return acc, int(target_tokens[acc])


def soft_anchor(logits: np.ndarray, E: np.ndarray, k: int = 8):
    """Soft anchor (generate.py:1422-1436): for one row of logits [V] and the
    embedding table E [V, H] (fp32 holding bf16 values), the k largest logits
    (a stable argsort of -logits: lower index first on ties), their fp32
    softmax, and the fp32 weighted sum of their embedding rows, summed in
    order q = 0..k-1.  Returns (ids [k], weights [k], anchor [H] fp32); the
    reference casts the anchor to the noise dtype (bf16) afterwards."""
    x = np.asarray(logits, dtype=np.float32)
    ids = np.argsort(-x, kind="stable")[:k]
    top = x[ids].astype(np.float32)
    e = np.exp(top - top.max())
    w = (e / e.sum()).astype(np.float32)
    rows = np.asarray(E, dtype=np.float32)[ids]
    anchor = np.zeros(rows.shape[1], dtype=np.float32)
    for q in range(k):
        anchor = anchor + w[q] * rows[q]
    return ids, w, anchor


# --------------------------------------------------------------------------
# seeded synthetic weights / inputs (the configs' N(0, 0.02) recipe)
# --------------------------------------------------------------------------
def synth_weights(cfg: OracleConfig, seed: int = 0, std: float = 0.02,
                  random_norms: bool = True):
    """Returns ``(q8, dense)`` where ``q8`` holds the int8 + fp16-scale
    projections (what the CUDA path receives) and ``dense`` the fp32
    ``OracleWeights`` built from their dequantised values, with bf16-rounded
    fc / lm_head (both stay bf16 in the W8A16 configs)."""
    g = np.random.default_rng(seed)
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nh, nkv, F, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.num_target_features, cfg.vocab_size

    def randn(*shape):
        return (g.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def norm_w(n):
        if random_norms:
            return (1.0 + 0.1 * g.standard_normal(n, dtype=np.float32)).astype(np.float32)
        return np.ones(n, dtype=np.float32)

    def bf16(a):
        return torch.from_numpy(a).to(torch.bfloat16).to(torch.float32)

    q8_layers, layers = [], []
    for _ in range(cfg.num_hidden_layers):
        raw = dict(wq=randn(nh * hd, H), wk=randn(nkv * hd, H), wv=randn(nkv * hd, H),
                   wo=randn(H, nh * hd), wg=randn(I, H), wu=randn(I, H), wd=randn(H, I))
        ql = {k: quantize_q8(v) for k, v in raw.items()}
        norms = dict(in_norm=norm_w(H), post_norm=norm_w(H), q_norm=norm_w(hd), k_norm=norm_w(hd))
        q8_layers.append(dict(ql, **norms))
        layers.append(OracleLayer(
            **{k: torch.from_numpy(dequantize_q8(*ql[k])) for k in raw},
            **{k: torch.from_numpy(v) for k, v in norms.items()}))
    fc = bf16(randn(H, F * H))
    lm = bf16(randn(V, H))
    hn, fn = norm_w(H), norm_w(H)
    dense = OracleWeights(fc, torch.from_numpy(hn), torch.from_numpy(fn), lm, layers)
    q8 = dict(layers=q8_layers, fc=fc, lm_head=lm, hidden_norm=hn, norm=fn)
    return q8, dense


def synth_inputs(cfg: OracleConfig, batch: int, ctx_len: int, block: int, seed: int = 1):
    """noise embedding rows (bf16-rounded N(0,1)*0.02 like test_ane_e2e.py:36-40)
    and target_hidden N(0,1) (bf16-rounded), as fp32 tensors."""
    g = torch.Generator().manual_seed(seed)
    H, F = cfg.hidden_size, cfg.num_target_features
    noise = (torch.randn(batch, block, H, generator=g) * 0.02).to(torch.bfloat16).float()
    th = torch.randn(batch, ctx_len, F * H, generator=g).to(torch.bfloat16).float()
    return noise, th
