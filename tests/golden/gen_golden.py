"""Generate the golden fixtures in this folder from the REFERENCE's own code.

Run in the development container (it needs the reference checkout, which the
GPU box does not have):

    python tests/golden/gen_golden.py /path/to/reference

It imports the reference's unmodified ``mirror_sd/dflash.py`` and
``mirror_sd/ane_model.py`` through the numpy MLX-API shim in ``mlx_shim/``
(MLX itself is not installable here), runs them on seeded tiny configs and
writes:

* ``dflash_forward_small.npz``: inputs and weights (bf16 bit patterns, int8 +
  fp16 scales) and the fp64 outputs of
  ``DFlashDraftModel.__call__`` (dflash.py:384-403) for a stateless call
  (cache=None) at batch 1 and 2, and a three-step cached sequence with a
  sink/window cache (dflash.py:139-212) including ``trim``;
* ``quantizer_q8.npz``: the int8 / fp16 bytes that
  ``ANEDraftModel._quantize_weight_q8`` (ane_model.py:265-279) returns for a
  matrix with a zero row, exact half-way ties and random rows;
* ``layer_ids.json``: ``build_target_layer_ids`` (dflash.py:108-119) values;
* ``soft_anchor.npz``: the block embedding that ``_make_soft_anchor``
  (scripts/bench_ane_pipeline.py:76-84, the restatement of
  generate.py:1422-1436 the reference benchmarks) returns for seeded logits
  and a bf16-valued embedding table, fp32 and bf16-valued logits, k = 8, 1, 16.

The shim only restates MLX primitive semantics; the fixtures pin the
reference's composition of them, and the quantiser bit-exactly.
"""
import importlib
import importlib.util
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# tiny DFlash dims (head_dim stays 128 as in every reference config)
TINY = dict(hidden_size=256, num_hidden_layers=2, intermediate_size=256,
            num_attention_heads=4, num_key_value_heads=2, head_dim=128,
            rms_norm_eps=1e-6, rope_theta=1000000.0, vocab_size=256,
            block_size=8, mask_token_id=255)
N_FEAT = 5


def load_reference(ref_root):
    sys.path.insert(0, os.path.join(HERE, "mlx_shim"))
    pkg = types.ModuleType("mirror_sd")
    pkg.__path__ = [os.path.join(ref_root, "mirror_sd")]
    sys.modules["mirror_sd"] = pkg          # skip the package __init__ (needs mlx_lm)
    dflash = importlib.import_module("mirror_sd.dflash")
    ane_model = importlib.import_module("mirror_sd.ane_model")
    return dflash, ane_model


def bf16_bits(a):
    """Round to bf16 (nearest-even) and return the raw 16-bit patterns."""
    u = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_value(bits):
    """bf16 bit patterns -> exact fp64 values."""
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def make_weights(rng, cfg, quantize):
    """Projection weights are int8 + fp16 scales from the reference's own
    quantiser (stored that way, 1 byte each); fc / lm_head / norms are
    bf16-representable values stored as bf16 bit patterns.  The model sees
    their exact fp64 values, so any engine fed these arrays gets identical
    operands."""
    H, I, hd = cfg["hidden_size"], cfg["intermediate_size"], cfg["head_dim"]
    nh, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    r = lambda *s: bf16_bits(rng.standard_normal(s) * 0.02)
    nw = lambda n: bf16_bits(1.0 + 0.1 * rng.standard_normal(n))
    stored = {"fc": r(H, N_FEAT * H), "hidden_norm": nw(H), "norm": nw(H),
              "lm_head": r(cfg["vocab_size"], H)}
    dense = {k: bf16_value(v) for k, v in stored.items()}
    shapes = {"wq": (nh * hd, H), "wk": (nkv * hd, H), "wv": (nkv * hd, H),
              "wo": (H, nh * hd), "wg": (I, H), "wu": (I, H), "wd": (H, I)}
    for i in range(cfg["num_hidden_layers"]):
        p = f"l{i}."
        for k, shp in shapes.items():
            q, s = quantize(rng.standard_normal(shp).astype(np.float32) * np.float32(0.02))
            stored[p + k + ".q"], stored[p + k + ".s"] = q, s
            dense[p + k] = q.astype(np.float64) * s.astype(np.float64)[:, None]
        for k, n in [("in_norm", H), ("post_norm", H), ("q_norm", hd), ("k_norm", hd)]:
            stored[p + k] = nw(n)
            dense[p + k] = bf16_value(stored[p + k])
    return stored, dense


def build_model(dflash, cfg, w):
    c = dflash.DFlashConfig(**cfg)
    c.target_layer_ids = [0, 1, 2, 3, 4]
    m = dflash.DFlashDraftModel(c)
    m.fc.weight = w["fc"]
    m.hidden_norm.weight = w["hidden_norm"]
    m.norm.weight = w["norm"]
    for i, L in enumerate(m.layers):
        p = f"l{i}."
        a = L.self_attn
        a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.o_proj.weight = (
            w[p + "wq"], w[p + "wk"], w[p + "wv"], w[p + "wo"])
        a.q_norm.weight, a.k_norm.weight = w[p + "q_norm"], w[p + "k_norm"]
        L.mlp.gate_proj.weight, L.mlp.up_proj.weight, L.mlp.down_proj.weight = (
            w[p + "wg"], w[p + "wu"], w[p + "wd"])
        L.input_layernorm.weight, L.post_attention_layernorm.weight = (
            w[p + "in_norm"], w[p + "post_norm"])
    return m


def main(ref_root):
    dflash, ane_model = load_reference(ref_root)
    rng = np.random.default_rng(20260101)
    cfg = dict(TINY)
    def quantize(m):
        qb, sb, oc, ic = ane_model.ANEDraftModel._quantize_weight_q8(None, m)
        return (np.frombuffer(qb, dtype=np.int8).reshape(oc, ic),
                np.frombuffer(sb, dtype=np.float16))

    stored, w = make_weights(rng, cfg, quantize)
    model = build_model(dflash, cfg, w)
    H, B = cfg["hidden_size"], cfg["block_size"]
    out = {f"w.{k}": v for k, v in stored.items()}

    # stateless calls (cache=None), batch 1 and 2
    for name, (bsz, ctx) in {"s1": (1, 12), "s2": (2, 20)}.items():
        nb = bf16_bits(rng.standard_normal((bsz, B, H)) * 0.02)
        tb = bf16_bits(rng.standard_normal((bsz, ctx, N_FEAT * H)))
        noise, th = bf16_value(nb), bf16_value(tb)
        hid = model(noise_embedding=noise, target_hidden=th, cache=None)
        logits = hid[:, -(B - 1):, :] @ w["lm_head"].T
        out.update({f"{name}.noise": nb, f"{name}.th": tb, f"{name}.hidden": hid,
                    f"{name}.tokens": dflash.sample(logits).astype(np.int32)})

    # cached decode sequence: sink 4 + window 16, trim(B) after each draft,
    # new context rows = accepted prefix + 1 (generate.py:599-609, :773)
    cache = model.make_cache(sink_size=4, window_size=16)
    for step, ctx in enumerate([12, 5, 9]):
        nb = bf16_bits(rng.standard_normal((1, B, H)) * 0.02)
        tb = bf16_bits(rng.standard_normal((1, ctx, N_FEAT * H)))
        noise, th = bf16_value(nb), bf16_value(tb)
        hid = model(noise_embedding=noise, target_hidden=th, cache=cache)
        p = f"c{step}."
        out.update({p + "noise": nb, p + "th": tb, p + "hidden": hid,
                    p + "offset_after_call": np.int64(cache[0].offset),
                    p + "len_after_call": np.int64(cache[0].keys.shape[2])})
        for c in cache:
            c.trim(B)
        out.update({p + "offset_after_trim": np.int64(cache[0].offset),
                    p + "len_after_trim": np.int64(cache[0].keys.shape[2]),
                    p + "k0_after_trim": cache[0].keys, p + "v1_after_trim": cache[1].values})
    out["cfg"] = np.array(json.dumps(cfg))
    np.savez_compressed(os.path.join(HERE, "dflash_forward_small.npz"), **out)

    # quantiser (ane_model.py:265-279): zero row, exact .5 ties, random rows
    qrng = np.random.default_rng(7)
    m = (qrng.standard_normal((16, 96)) * 0.02).astype(np.float32)
    m[3] = 0.0
    row = np.array([(k + 0.5) for k in range(-48, 48)], dtype=np.float32)
    row[-1] = 127.0
    m[5] = row * np.float32(0.01)
    m[6] = np.float32(1e-30) * qrng.standard_normal(96).astype(np.float32)  # subnormal-scale row
    m[7, :] = -m[7, :]
    qb, sb, oc, ic = ane_model.ANEDraftModel._quantize_weight_q8(None, m)
    np.savez_compressed(os.path.join(HERE, "quantizer_q8.npz"), w=m,
                        q=np.frombuffer(qb, dtype=np.int8).reshape(oc, ic),
                        s=np.frombuffer(sb, dtype=np.float16))

    ids = {f"{nt},{nd}": dflash.build_target_layer_ids(nt, nd)
           for nt, nd in [(36, 5), (64, 5), (40, 5), (28, 3), (36, 1), (48, 4)]}
    with open(os.path.join(HERE, "layer_ids.json"), "w") as f:
        json.dump(ids, f, indent=1, sort_keys=True)
    soft_anchor_fixture(ref_root)
    print("wrote fixtures to", HERE)


def soft_anchor_fixture(ref_root):
    """``soft_anchor.npz`` from the reference's ``_make_soft_anchor``.  The
    embedding table holds bf16 values (stored as bit patterns, used as fp32,
    which is what MLX promotes bf16 * fp32 to); the noise rows are fp32, so
    the returned row 0 is the fp32 sum before the cast to the noise dtype."""
    sys.path.insert(0, os.path.join(HERE, "mlx_shim"))
    spec = importlib.util.spec_from_file_location(
        "bench_ane_pipeline", os.path.join(ref_root, "scripts", "bench_ane_pipeline.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    rng = np.random.default_rng(4242)
    out = {}
    cases = {"a": (256, 256, 4, 8, False, 3.0), "b": (1000, 64, 3, 8, True, 2.0),
             "c": (777, 128, 2, 1, False, 1.0), "d": (777, 128, 2, 16, False, 0.5)}
    for name, (V, H, rows, k, bf16_logits, scale) in cases.items():
        eb = bf16_bits(rng.standard_normal((V, H)) * 0.05)
        E = bf16_value(eb).astype(np.float32)
        logits = (rng.standard_normal((rows, V)) * scale).astype(np.float32)
        if bf16_logits:
            logits = bf16_value(bf16_bits(logits)).astype(np.float32)
        noise = np.zeros((1, 4, H), dtype=np.float32)
        anchors = []
        for r in range(rows):
            blk = bench._make_soft_anchor(noise, logits[r], lambda ids: E[ids], top_k=k)
            anchors.append(np.asarray(blk)[0, 0])
        out.update({f"{name}.E": eb, f"{name}.logits": logits, f"{name}.k": np.int64(k),
                    f"{name}.bf16_logits": np.int64(bf16_logits),
                    f"{name}.anchor": np.stack(anchors).astype(np.float32)})
    np.savez_compressed(os.path.join(HERE, "soft_anchor.npz"), **out)


if __name__ == "__main__":
    ref = next((a for a in sys.argv[1:] if not a.startswith("--")), None)
    if ref is None:
        sys.exit("usage: python tests/golden/gen_golden.py /path/to/reference [--only-soft-anchor]")
    if "--only-soft-anchor" in sys.argv:
        soft_anchor_fixture(ref)
    else:
        main(ref)
