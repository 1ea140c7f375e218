"""Weight containers: from numpy W8A16 arrays, or seeded synthetic weights
generated directly on the GPU (N(0, std) per projection, quantised with the
reference rule by the CUDA quantiser, ane_model.py:265-279)."""
from __future__ import annotations

import numpy as np
import torch

from .dflash import PROJ, DFlashConfig, DFlashWeightsF32, DFlashWeightsQ8, F32Layer, Q8Layer, quantize_q8


def weights_from_q8_numpy(q8: dict, device) -> DFlashWeightsQ8:
    """``q8``: {"layers": [{name: (int8 [oc, ic], fp16 [oc]) for name in PROJ,
    "in_norm", "post_norm", "q_norm", "k_norm": fp32}], "fc": [H, F*H],
    "hidden_norm": [H], "norm": [H]} (numpy or torch)."""
    dev = torch.device(device)
    t = lambda a, dt: torch.as_tensor(np.asarray(a) if not torch.is_tensor(a) else a).to(dev, dt)
    layers = []
    for L in q8["layers"]:
        layers.append(Q8Layer(q={k: t(L[k][0], torch.int8) for k in PROJ},
                              s={k: t(L[k][1], torch.float16) for k in PROJ},
                              input_layernorm=t(L["in_norm"], torch.float32),
                              post_attention_layernorm=t(L["post_norm"], torch.float32),
                              q_norm=t(L["q_norm"], torch.float32),
                              k_norm=t(L["k_norm"], torch.float32)))
    return DFlashWeightsQ8(fc=t(q8["fc"], torch.bfloat16), hidden_norm=t(q8["hidden_norm"], torch.float32),
                           norm=t(q8["norm"], torch.float32), layers=layers)


@torch.no_grad()
def synth_weights_q8(cfg: DFlashConfig, seed: int = 0, device="cuda", std: float = 0.02,
                     random_norms: bool = False, num_target_features: int = 5):
    """Seeded N(0, std) weights of the given dims, generated on the GPU.
    Projections are quantised to int8 + fp16 scales; fc and the tied lm_head
    stay bf16; norm weights are ones (or 1 + N(0, 0.1) with random_norms).
    Returns ``(DFlashWeightsQ8, lm_head [V, H] bf16)``."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nh, nkv, F = cfg.num_attention_heads, cfg.num_key_value_heads, num_target_features
    shapes = {"wq": (nh * hd, H), "wk": (nkv * hd, H), "wv": (nkv * hd, H), "wo": (H, nh * hd),
              "wg": (I, H), "wu": (I, H), "wd": (H, I)}

    def randn(*shape):
        return torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std

    def norm_w(n):
        if random_norms:
            return 1.0 + 0.1 * torch.randn((n,), generator=g, device=dev)
        return torch.ones((n,), device=dev)

    layers = []
    for _ in range(cfg.num_hidden_layers):
        q, s = {}, {}
        for k, shp in shapes.items():
            w = randn(*shp)
            q[k], s[k] = quantize_q8(w)
            del w
        layers.append(Q8Layer(q=q, s=s, input_layernorm=norm_w(H), post_attention_layernorm=norm_w(H),
                              q_norm=norm_w(hd), k_norm=norm_w(hd)))
    fc = randn(H, F * H).to(torch.bfloat16)
    lm = torch.empty((cfg.vocab_size, H), dtype=torch.bfloat16, device=dev)
    for i in range(0, cfg.vocab_size, 16384):  # chunked to bound the fp32 temporary
        j = min(cfg.vocab_size, i + 16384)
        lm[i:j] = randn(j - i, H).to(torch.bfloat16)
    w = DFlashWeightsQ8(fc=fc, hidden_norm=norm_w(H), norm=norm_w(H), layers=layers)
    return w, lm


@torch.no_grad()
def synth_weights_f32(cfg: DFlashConfig, seed: int = 0, device="cuda", std: float = 0.02,
                      random_norms: bool = False, num_target_features: int = 5):
    """Seeded fp32 N(0, std) weights of the given dims for the fp32-accumulate
    mode (the CPU plumbing config: every weight fp32 N(0, 0.02), norm weights
    ones or 1 + N(0, 0.1) with random_norms), generated on the GPU.
    Returns ``(DFlashWeightsF32, lm_head [V, H] fp32)``; the lm_head is the
    tied embedding, so it also embeds the block ids."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nh, nkv, F = cfg.num_attention_heads, cfg.num_key_value_heads, num_target_features
    shapes = {"wq": (nh * hd, H), "wk": (nkv * hd, H), "wv": (nkv * hd, H), "wo": (H, nh * hd),
              "wg": (I, H), "wu": (I, H), "wd": (H, I)}

    def randn(*shape):
        return torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std

    def norm_w(n):
        if random_norms:
            return 1.0 + 0.1 * torch.randn((n,), generator=g, device=dev)
        return torch.ones((n,), device=dev)

    layers = [F32Layer(w={k: randn(*shp) for k, shp in shapes.items()}, input_layernorm=norm_w(H),
                       post_attention_layernorm=norm_w(H), q_norm=norm_w(hd), k_norm=norm_w(hd))
              for _ in range(cfg.num_hidden_layers)]
    fc = randn(H, F * H)
    lm = randn(cfg.vocab_size, H)
    return DFlashWeightsF32(fc=fc, hidden_norm=norm_w(H), norm=norm_w(H), layers=layers), lm
