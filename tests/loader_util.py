"""Synthetic HuggingFace-style DFlash checkpoints for the loader tests."""
import json
import os

import numpy as np
import torch
from safetensors.torch import save_file

from oracle import dflash_oracle as O

PROJ_NAMES = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj",
              "wo": "self_attn.o_proj", "wg": "mlp.gate_proj", "wu": "mlp.up_proj", "wd": "mlp.down_proj"}


def make_checkpoint(path, ocfg: O.OracleConfig, seed=0, layout="single", prefix="", dtype=torch.bfloat16):
    """Writes config.json and seeded float weights; returns the tensors written
    (unprefixed names -> fp32 CPU tensors of the values stored)."""
    os.makedirs(path, exist_ok=True)
    g = torch.Generator().manual_seed(seed)
    H, I, hd = ocfg.hidden_size, ocfg.intermediate_size, ocfg.head_dim
    nh, nkv, F = ocfg.num_attention_heads, ocfg.num_key_value_heads, ocfg.num_target_features
    shapes = {"wq": (nh * hd, H), "wk": (nkv * hd, H), "wv": (nkv * hd, H), "wo": (H, nh * hd),
              "wg": (I, H), "wu": (I, H), "wd": (H, I)}
    t = {"fc.weight": torch.randn(H, F * H, generator=g) * 0.02,
         "hidden_norm.weight": 1 + 0.1 * torch.randn(H, generator=g),
         "norm.weight": 1 + 0.1 * torch.randn(H, generator=g)}
    for i in range(ocfg.num_hidden_layers):
        p = f"layers.{i}."
        for k, shp in shapes.items():
            t[p + PROJ_NAMES[k] + ".weight"] = torch.randn(*shp, generator=g) * 0.02
        t[p + "input_layernorm.weight"] = 1 + 0.1 * torch.randn(H, generator=g)
        t[p + "post_attention_layernorm.weight"] = 1 + 0.1 * torch.randn(H, generator=g)
        t[p + "self_attn.q_norm.weight"] = 1 + 0.1 * torch.randn(hd, generator=g)
        t[p + "self_attn.k_norm.weight"] = 1 + 0.1 * torch.randn(hd, generator=g)
    stored = {k: v.to(dtype) for k, v in t.items()}
    named = {prefix + k: v for k, v in stored.items()}
    keys = sorted(named)
    if layout == "single":
        save_file(named, os.path.join(path, "model.safetensors"))
    elif layout == "sharded":
        half = len(keys) // 2
        shards = {"model-00001-of-00002.safetensors": keys[:half],
                  "model-00002-of-00002.safetensors": keys[half:]}
        wmap = {}
        for fname, ks in shards.items():
            save_file({k: named[k] for k in ks}, os.path.join(path, fname))
            wmap.update({k: fname for k in ks})
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {}, "weight_map": wmap}, f)
    else:  # any *.safetensors names
        half = len(keys) // 2
        save_file({k: named[k] for k in keys[:half]}, os.path.join(path, "a.safetensors"))
        save_file({k: named[k] for k in keys[half:]}, os.path.join(path, "b.safetensors"))
    cfg = {"hidden_size": H, "num_hidden_layers": ocfg.num_hidden_layers, "intermediate_size": I,
           "num_attention_heads": nh, "num_key_value_heads": nkv, "head_dim": hd,
           "rms_norm_eps": ocfg.rms_norm_eps, "rope_theta": ocfg.rope_theta, "vocab_size": ocfg.vocab_size,
           "dflash_config": {"block_size": ocfg.block_size, "mask_token_id": ocfg.mask_token_id,
                             "target_layer_ids": list(range(F)), "num_target_layers": 36}}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    return {k: v.float() for k, v in stored.items()}


def oracle_weights(ocfg, tensors, lm_head):
    """Dense oracle weights from the stored values: projections through the
    oracle quantiser (the reference rule), fc / lm_head as stored."""
    layers = []
    for i in range(ocfg.num_hidden_layers):
        p = f"layers.{i}."
        deq = {}
        for k, path in PROJ_NAMES.items():
            q, s = O.quantize_q8(tensors[p + path + ".weight"].numpy())
            deq[k] = torch.from_numpy(O.dequantize_q8(q, s))
        layers.append(O.OracleLayer(**deq, in_norm=tensors[p + "input_layernorm.weight"],
                                    post_norm=tensors[p + "post_attention_layernorm.weight"],
                                    q_norm=tensors[p + "self_attn.q_norm.weight"],
                                    k_norm=tensors[p + "self_attn.k_norm.weight"]))
    return O.OracleWeights(tensors["fc.weight"], tensors["hidden_norm.weight"], tensors["norm.weight"],
                           lm_head.float(), layers)
