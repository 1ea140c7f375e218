"""Test helpers shared by the GPU parity tests (oracle <-> CUDA path glue)."""
import numpy as np
import torch

from oracle import dflash_oracle as O


def tiny_cfg(**kw):
    d = dict(hidden_size=256, num_hidden_layers=2, intermediate_size=256, num_attention_heads=4,
             num_key_value_heads=2, head_dim=128, vocab_size=1000, block_size=8)
    d.update(kw)
    return O.OracleConfig(**d)


def pkg_config(pkg, ocfg: O.OracleConfig):
    c = pkg.DFlashConfig(hidden_size=ocfg.hidden_size, num_hidden_layers=ocfg.num_hidden_layers,
                         intermediate_size=ocfg.intermediate_size,
                         num_attention_heads=ocfg.num_attention_heads,
                         num_key_value_heads=ocfg.num_key_value_heads, head_dim=ocfg.head_dim,
                         rms_norm_eps=ocfg.rms_norm_eps, rope_theta=ocfg.rope_theta,
                         vocab_size=ocfg.vocab_size, block_size=ocfg.block_size,
                         mask_token_id=ocfg.mask_token_id)
    c.target_layer_ids = list(range(ocfg.num_target_features))
    return c


def gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=64, max_block=None, device="cuda"):
    w = pkg.weights_from_q8_numpy(q8, device)
    lm = torch.as_tensor(q8["lm_head"]).to(device, torch.bfloat16)
    return pkg.DFlashDraftModel(pkg_config(pkg, ocfg), w, lm, max_batch=max_batch, max_ctx=max_ctx,
                                max_block=max_block or ocfg.block_size, device=device)


def cosine(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def check_hidden(gpu, ref, cos_min=0.9995, max_abs=2e-2):
    """North-star tolerance for bf16/fp16 hidden states."""
    g = gpu.float().cpu()
    r = ref.float().cpu()
    c = cosine(g, r)
    m = float((g - r).abs().max())
    assert c >= cos_min and m <= max_abs, f"cosine {c:.6f} (min {cos_min}), max-abs {m:.4g} (max {max_abs})"
    return c, m


def check_tokens(gpu_tokens, ref_logits, margin_tol):
    """Draft ids must equal the oracle's argmax wherever the oracle's top-1 /
    top-2 logit margin exceeds ``margin_tol`` (a near-tie within the numeric
    tolerance of the bf16/f16 path may legitimately resolve either way).
    Returns (n_equal, n_total, n_near_ties)."""
    ref_ids = O.greedy(ref_logits)
    margin = O.top2_margin(ref_logits)
    g = gpu_tokens.cpu().to(torch.int32)
    eq = g == ref_ids
    near = margin <= margin_tol
    bad = (~eq) & (~near)
    assert not bool(bad.any()), (
        f"draft ids differ at rows with margin > {margin_tol}: "
        f"{[(tuple(i.tolist()), float(margin[tuple(i)])) for i in bad.nonzero()[:5]]}")
    return int(eq.sum()), int(eq.numel()), int(near.sum())


def bf16_value(bits):
    """bf16 bit patterns (uint16, as stored in the golden fixtures) -> fp64."""
    bits = np.asarray(bits)
    if bits.dtype != np.uint16:
        return bits.astype(np.float64)
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def fixture_case(z):
    """(OracleConfig, q8 dict for the GPU model, fp64 OracleWeights) from the
    reference-generated fixture."""
    import json
    cfgd = json.loads(str(z["cfg"]))
    ocfg = O.OracleConfig(**cfgd)
    f64 = lambda a: torch.from_numpy(bf16_value(a))
    layers, q8_layers = [], []
    for i in range(ocfg.num_hidden_layers):
        p = f"w.l{i}."
        deq = {k: torch.from_numpy(z[p + k + ".q"].astype(np.float64) * z[p + k + ".s"].astype(np.float64)[:, None])
               for k in ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]}
        norms = {k: f64(z[p + k]) for k in ["in_norm", "post_norm", "q_norm", "k_norm"]}
        layers.append(O.OracleLayer(**deq, **norms))
        L = {k: (z[p + k + ".q"], z[p + k + ".s"]) for k in ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]}
        L.update({k: v.float().numpy() for k, v in norms.items()})
        q8_layers.append(L)
    dense = O.OracleWeights(f64(z["w.fc"]), f64(z["w.hidden_norm"]), f64(z["w.norm"]), f64(z["w.lm_head"]),
                            layers)
    q8 = dict(layers=q8_layers, fc=dense.fc.float(), lm_head=dense.lm_head.float(),
              hidden_norm=dense.hidden_norm.float().numpy(), norm=dense.norm.float().numpy())
    return ocfg, q8, dense
