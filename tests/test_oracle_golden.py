"""The CPU oracle against fixtures produced by the reference's own code.

The fixtures (tests/golden/gen_golden.py) come from running the reference's
``mirror_sd/dflash.py`` and ``ANEDraftModel._quantize_weight_q8`` through an
MLX-API shim; these tests pin the oracle's composition of the forward, its
cache semantics and its quantiser to them.
"""
import json
import os

import numpy as np
import torch

from oracle import dflash_oracle as O
from helpers import bf16_value, fixture_case


def _load(golden_dir):
    z = np.load(os.path.join(golden_dir, "dflash_forward_small.npz"))
    cfg, _, w = fixture_case(z)
    return z, cfg, w


def test_stateless_forward_matches_reference(golden_dir):
    z, cfg, w = _load(golden_dir)
    for name in ["s1", "s2"]:
        noise = torch.from_numpy(bf16_value(z[f"{name}.noise"]))
        th = torch.from_numpy(bf16_value(z[f"{name}.th"]))
        out = O.draft_forward(cfg, w, noise, th)
        ref = z[f"{name}.hidden"]
        assert np.abs(out.numpy() - ref).max() < 1e-9
        toks = O.greedy(O.draft_logits(w, out, cfg.block_size))
        assert np.array_equal(toks.numpy(), z[f"{name}.tokens"])


def test_stateless_forward_fp32_close(golden_dir):
    z, cfg, w = _load(golden_dir)
    w32 = w.to(torch.float32)
    noise = torch.from_numpy(bf16_value(z["s2.noise"])).float()
    th = torch.from_numpy(bf16_value(z["s2.th"])).float()
    out = O.draft_forward(cfg, w32, noise, th)
    assert np.abs(out.numpy() - z["s2.hidden"]).max() < 2e-4


def test_cached_sequence_matches_reference(golden_dir):
    z, cfg, w = _load(golden_dir)
    cache = [O.OracleKVCache(sink_size=4, window_size=16) for _ in range(cfg.num_hidden_layers)]
    for step in range(3):
        p = f"c{step}."
        noise = torch.from_numpy(bf16_value(z[p + "noise"]))
        th = torch.from_numpy(bf16_value(z[p + "th"]))
        out = O.draft_forward(cfg, w, noise, th, cache=cache)
        assert np.abs(out.numpy() - z[p + "hidden"]).max() < 1e-9
        assert cache[0].offset == int(z[p + "offset_after_call"])
        assert cache[0].keys.shape[2] == int(z[p + "len_after_call"])
        for c in cache:
            c.trim(cfg.block_size)
        assert cache[0].offset == int(z[p + "offset_after_trim"])
        assert cache[0].keys.shape[2] == int(z[p + "len_after_trim"])
        assert np.abs(cache[0].keys.numpy() - z[p + "k0_after_trim"]).max() < 1e-9
        assert np.abs(cache[1].values.numpy() - z[p + "v1_after_trim"]).max() < 1e-9


def test_quantizer_bit_exact(golden_dir):
    z = np.load(os.path.join(golden_dir, "quantizer_q8.npz"))
    q, s = O.quantize_q8(z["w"])
    assert np.array_equal(q, z["q"])
    assert np.array_equal(s.view(np.uint16), z["s"].view(np.uint16))


def test_build_target_layer_ids(golden_dir):
    with open(os.path.join(golden_dir, "layer_ids.json")) as f:
        ids = json.load(f)
    for key, val in ids.items():
        nt, nd = map(int, key.split(","))
        assert O.build_target_layer_ids(nt, nd) == val


def test_accept_prefix():
    assert O.accept([5, 6, 7], [5, 6, 7, 8]) == (3, 8)
    assert O.accept([5, 6, 7], [5, 9, 7, 8]) == (1, 9)
    assert O.accept([5, 6, 7], [1, 6, 7, 8]) == (0, 1)
    assert O.accept([], [4]) == (0, 4)


def test_greedy_first_index_on_ties():
    logits = torch.tensor([[0.0, 3.0, 3.0, 1.0], [2.0, 2.0, 2.0, 2.0]])
    assert O.greedy(logits).tolist() == [1, 0]


def test_soft_anchor_matches_reference(golden_dir):
    """The oracle's soft anchor equals the reference's ``_make_soft_anchor``
    (scripts/bench_ane_pipeline.py:76-84) bit for bit, ties included (case b
    has a tie at the k-th place, broken by the lower index)."""
    z = np.load(os.path.join(golden_dir, "soft_anchor.npz"))
    for c in "abcd":
        E = bf16_value(z[f"{c}.E"]).astype(np.float32)
        logits, k = z[f"{c}.logits"], int(z[f"{c}.k"])
        for r in range(logits.shape[0]):
            ids, w, anchor = O.soft_anchor(logits[r], E, k)
            assert len(ids) == k and abs(float(w.sum()) - 1.0) < 1e-6
            assert np.array_equal(anchor, z[f"{c}.anchor"][r])
