"""Checkpoint loading for the B200 draft model (mirror_sd/loader.py:20-116).

A DFlash draft checkpoint is a HuggingFace directory: ``config.json`` and
safetensors weights, one file, shards listed by
``model.safetensors.index.json``, or any ``*.safetensors`` (the three layouts
``_load_safetensors`` accepts).  Parameter names follow the reference module
tree (dflash.py:246-379):

    fc.weight, hidden_norm.weight, norm.weight,
    layers.{i}.self_attn.{q,k,v,o}_proj.weight,
    layers.{i}.self_attn.{q,k}_norm.weight,
    layers.{i}.mlp.{gate,up,down}_proj.weight,
    layers.{i}.{input,post_attention}_layernorm.weight

(an optional ``model.`` prefix is accepted).  The seven projections of every
layer are quantised on the GPU with the reference's int8 rule
(ane_model.py:265-279, bit-exact); fc stays bf16, norms fp32.

``save_q8_checkpoint`` writes that quantised form (int8 weights, fp16 scales:
the ``Q8LayerWeights`` bytes of ane/src/wrapper.rs:363-428) so a later load
skips the quantisation; ``load_dflash_weights`` reads either form.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Dict, Optional, Tuple

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from .dflash import PROJ, DFlashConfig, DFlashDraftModel, DFlashWeightsQ8, Q8Layer, quantize_q8

# our projection keys -> the reference module paths inside a layer
PROJ_PATH = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj",
             "wo": "self_attn.o_proj", "wg": "mlp.gate_proj", "wu": "mlp.up_proj",
             "wd": "mlp.down_proj"}
NORM_PATH = {"input_layernorm": "input_layernorm",
             "post_attention_layernorm": "post_attention_layernorm",
             "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm"}
Q8_SCALE_SUFFIX = ".scales"      # fp16 [out] beside an int8 ".weight"


def load_config(model_path, overrides: Optional[Dict] = None) -> DFlashConfig:
    """DFlashConfig from ``config.json`` (loader.py:61-72)."""
    path = Path(model_path) / "config.json"
    if not path.exists():
        raise FileNotFoundError(f"No config.json found at {path}")
    with open(path) as f:
        cfg = json.load(f)
    if overrides:
        cfg.update(overrides)
    return DFlashConfig.from_dict(cfg)


def weight_files(model_path) -> list:
    """The safetensors files of a checkpoint directory, in the order
    loader.py:84-112 reads them: the shards of the index, else
    ``model.safetensors``, else every ``*.safetensors`` sorted."""
    root = Path(model_path)
    index = root / "model.safetensors.index.json"
    if index.exists():
        with open(index) as f:
            names = sorted(set(json.load(f)["weight_map"].values()))
        return [root / n for n in names]
    single = root / "model.safetensors"
    if single.exists():
        return [single]
    files = sorted(root.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"No safetensors weights found in {root}")
    return files


def read_tensors(model_path) -> Dict[str, torch.Tensor]:
    """Every tensor of the checkpoint on the CPU (dtype as stored), with a
    leading ``model.`` stripped from the names."""
    out = {}
    for fpath in weight_files(model_path):
        with safe_open(str(fpath), framework="pt", device="cpu") as f:
            for k in f.keys():
                name = k[len("model."):] if k.startswith("model.") else k
                out[name] = f.get_tensor(k)
    return out


def _need(t: Dict[str, torch.Tensor], name: str) -> torch.Tensor:
    if name not in t:
        raise KeyError(f"checkpoint has no tensor {name!r}")
    return t[name]


@torch.no_grad()
def load_dflash_weights(model_path, config: Optional[DFlashConfig] = None,
                        device="cuda") -> Tuple[DFlashWeightsQ8, DFlashConfig]:
    """The draft weights in the W8A16 form the device path runs on.

    Projections stored as floats are quantised on ``device`` (the reference
    rule, bit-exact); projections already stored as int8 with ``.scales``
    (``save_q8_checkpoint``) are taken as they are."""
    cfg = config or load_config(model_path)
    dev = torch.device(device)
    t = read_tensors(model_path)
    H, F = cfg.hidden_size, len(cfg.target_layer_ids)
    fc = _need(t, "fc.weight")
    if tuple(fc.shape) != (H, F * H):
        raise ValueError(f"fc.weight has shape {tuple(fc.shape)}, expected {(H, F * H)}")
    layers = []
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        q, s = {}, {}
        for key, path in PROJ_PATH.items():
            w = _need(t, p + path + ".weight")
            sc = t.get(p + path + ".weight" + Q8_SCALE_SUFFIX)
            if w.dtype == torch.int8:
                if sc is None:
                    raise KeyError(f"int8 tensor {p + path}.weight has no {Q8_SCALE_SUFFIX}")
                q[key], s[key] = w.to(dev), sc.to(dev, torch.float16)
            else:
                q[key], s[key] = quantize_q8(w.to(dev, torch.float32))
        norms = {k: _need(t, p + v + ".weight").to(dev, torch.float32) for k, v in NORM_PATH.items()}
        layers.append(Q8Layer(q=q, s=s, **norms))
    w = DFlashWeightsQ8(fc=fc.to(dev, torch.bfloat16),
                        hidden_norm=_need(t, "hidden_norm.weight").to(dev, torch.float32),
                        norm=_need(t, "norm.weight").to(dev, torch.float32), layers=layers)
    return w, cfg


def load_dflash_model(model_path, lm_head: torch.Tensor, config_overrides: Optional[Dict] = None,
                      device="cuda", max_batch: int = 1, max_ctx: int = 4096,
                      max_block: Optional[int] = None) -> Tuple[DFlashDraftModel, DFlashConfig]:
    """``load_dflash_model`` (loader.py:20-58) on the device: the draft
    model and its config.  The draft does not own the lm_head; ``lm_head`` is
    the target's (tied) embedding [V, H] (generate.py:435-436)."""
    cfg = load_config(model_path, config_overrides)
    w, cfg = load_dflash_weights(model_path, cfg, device)
    model = DFlashDraftModel(cfg, w, lm_head, max_batch=max_batch, max_ctx=max_ctx, max_block=max_block,
                             device=device)
    return model, cfg


def save_q8_checkpoint(weights: DFlashWeightsQ8, config: DFlashConfig, output_dir) -> Path:
    """Write the quantised weights (int8 projections + fp16 ``.scales``, bf16
    fc, fp32 norms) and the config, as ``convert_dflash_to_mlx``
    (loader.py:117-170) writes a converted checkpoint."""
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    tensors = {"fc.weight": weights.fc, "hidden_norm.weight": weights.hidden_norm,
               "norm.weight": weights.norm}
    for i, L in enumerate(weights.layers):
        p = f"layers.{i}."
        for key, path in PROJ_PATH.items():
            tensors[p + path + ".weight"] = L.q[key]
            tensors[p + path + ".weight" + Q8_SCALE_SUFFIX] = L.s[key]
        for k, v in NORM_PATH.items():
            tensors[p + v + ".weight"] = getattr(L, k)
    save_file({k: v.detach().contiguous().cpu() for k, v in tensors.items()},
              str(out / "model.safetensors"))
    with open(out / "config.json", "w") as f:
        json.dump(config.to_dict(), f, indent=2)
    return out
