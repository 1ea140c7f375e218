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


# Per-case parity records, printed as a table at the end of the pytest run
# (conftest.pytest_terminal_summary): hidden-state cosine / max-abs and the
# draft-id comparison of every case that calls check_hidden / check_tokens
# with a label.
PARITY = {}


def _record(label, **kw):
    if label:
        PARITY.setdefault(label, {}).update(kw)


def check_hidden(gpu, ref, cos_min=0.9995, max_abs=2e-2, label=None):
    """North-star tolerance for bf16/fp16 hidden states."""
    g = gpu.float().cpu()
    r = ref.float().cpu()
    c = cosine(g, r)
    m = float((g - r).abs().max())
    _record(label, cosine=c, max_abs=m)
    assert c >= cos_min and m <= max_abs, f"cosine {c:.6f} (min {cos_min}), max-abs {m:.4g} (max {max_abs})"
    return c, m


def token_stats(gpu_tokens, ref_logits):
    """Compare device draft ids with the oracle's logits row by row.  For a
    row whose id differs, ``gap`` is the oracle's top-1 logit minus the
    oracle's logit at the device's id: how far the device's choice is from
    the oracle's maximum.  Returns (rows, n_diff, max_gap, diffs) with diffs
    a list of (row index, oracle id, device id, gap)."""
    ref_logits = ref_logits.double()
    ref_ids = O.greedy(ref_logits)
    g = gpu_tokens.cpu().to(torch.int64).reshape(ref_ids.shape)
    flat_l = ref_logits.reshape(-1, ref_logits.shape[-1])
    flat_g = g.reshape(-1)
    flat_r = ref_ids.reshape(-1).to(torch.int64)
    top = flat_l.gather(1, flat_r[:, None])[:, 0]
    at_g = flat_l.gather(1, flat_g.clamp(0, flat_l.shape[1] - 1)[:, None])[:, 0]
    gap = top - at_g
    diff = (flat_g != flat_r).nonzero().flatten().tolist()
    diffs = [(i, int(flat_r[i]), int(flat_g[i]), float(gap[i])) for i in diff]
    return int(flat_g.numel()), len(diffs), max([d[3] for d in diffs], default=0.0), diffs


def check_tokens(gpu_tokens, ref_logits, margin_tol, label=None, max_diff_frac=None):
    """Draft ids must equal the oracle's argmax, except where the device's
    choice is within ``margin_tol`` of the oracle's maximum logit (a near-tie
    that the bf16/f16 path may resolve either way).  With ``max_diff_frac``
    the number of such rows is bounded too (at most max(1, frac * rows)).
    Returns (n_equal, n_total, n_diff)."""
    rows, n_diff, max_gap, diffs = token_stats(gpu_tokens, ref_logits)
    margin = O.top2_margin(ref_logits.double()).reshape(-1)
    _record(label, rows=rows, ids_differ=n_diff, max_gap=max_gap, tol=margin_tol,
            min_margin=float(margin.min()))
    bad = [d for d in diffs if not d[3] <= margin_tol]
    assert not bad, f"draft ids differ by more than {margin_tol} of oracle logit: {bad[:5]}"
    if max_diff_frac is not None:
        assert n_diff <= max(1, int(max_diff_frac * rows)), f"{n_diff} of {rows} ids differ: {diffs[:5]}"
    return rows - n_diff, rows, n_diff


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


def oracle_weights_from_q8(w, lm):
    """fp32 CPU ``OracleWeights`` holding exactly what a device handle built
    from ``w`` (DFlashWeightsQ8) and ``lm`` (bf16 [V, H]) computes with: the
    dequantised int8 * fp16-scale projections, the bf16 fc and lm_head."""
    deq = lambda l, k: (l.q[k].float() * l.s[k].float()[:, None]).cpu()
    layers = [O.OracleLayer(**{k: deq(l, k) for k in ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]},
                            in_norm=l.input_layernorm.float().cpu(),
                            post_norm=l.post_attention_layernorm.float().cpu(),
                            q_norm=l.q_norm.float().cpu(), k_norm=l.k_norm.float().cpu()) for l in w.layers]
    return O.OracleWeights(w.fc.float().cpu(), w.hidden_norm.float().cpu(), w.norm.float().cpu(),
                           lm.float().cpu(), layers)


def oracle_weights_from_f32(w, lm):
    """fp32 CPU ``OracleWeights`` copy of an fp32-mode model's weights
    (DFlashWeightsF32 and the fp32 lm_head)."""
    layers = [O.OracleLayer(**{k: l.w[k].float().cpu() for k in ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]},
                            in_norm=l.input_layernorm.float().cpu(),
                            post_norm=l.post_attention_layernorm.float().cpu(),
                            q_norm=l.q_norm.float().cpu(), k_norm=l.k_norm.float().cpu()) for l in w.layers]
    return O.OracleWeights(w.fc.float().cpu(), w.hidden_norm.float().cpu(), w.norm.float().cpu(),
                           lm.float().cpu(), layers)
