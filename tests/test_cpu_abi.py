"""CPU-only checks of the boundary: the C-ABI library loads and exports every
function include/dflash_b200.h declares (no compute call without a GPU), and
the host-side mirror of the reference interface."""
import ctypes
import json
import os
import re

import pytest

from oracle import dflash_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    with open(os.path.join(ROOT, "include", "dflash_b200.h")) as f:
        src = f.read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dflash_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ["dflash_create", "dflash_forward", "dflash_accept", "dflash_destroy",
              "dflash_last_error", "dflash_quantize_q8"]:
        assert n in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._native.load()
    for name in _declared():
        assert hasattr(lib, name), name
        assert name in pkg._native.EXPORTS, f"{name} has no ctypes binding"


def test_version_and_error_string_without_gpu(pkg):
    lib = pkg._native.load()
    assert lib.dflash_version() >= 1
    # argument validation runs before any CUDA call
    h = ctypes.c_void_p()
    dims = pkg._native.DFlashDims(hidden_size=256, num_hidden_layers=1, intermediate_size=256,
                                  num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                  vocab_size=10, num_target_features=5, rms_norm_eps=1e-6,
                                  rope_theta=1e6, max_batch=1, max_block=8, max_ctx=8)
    st = lib.dflash_create(ctypes.byref(dims), None, 0, ctypes.byref(h))
    assert st == pkg._native.DFLASH_ERR_INVALID
    assert "head_dim" in pkg._native.last_error()
    with pytest.raises(ValueError):
        pkg._native.check(st, "dflash_create")
    assert lib.dflash_forward(None, None, None) == pkg._native.DFLASH_ERR_INVALID


def test_config_from_dict_defaults_match_reference(pkg):
    # dflash.py:77-105 fall-backs differ from the dataclass defaults
    c = pkg.DFlashConfig.from_dict({})
    assert (c.rope_theta, c.mask_token_id, c.intermediate_size, c.num_key_value_heads) == \
        (10000.0, 151667, 10944, 2)
    c = pkg.DFlashConfig.from_dict({"hidden_size": 5120, "dflash_config": {
        "block_size": 32, "mask_token_id": 5, "target_layer_ids": [1, 2, 3, 4, 5]}})
    assert (c.block_size, c.mask_token_id, c.target_layer_ids) == (32, 5, [1, 2, 3, 4, 5])
    d = pkg.DFlashConfig()
    assert (d.rope_theta, d.mask_token_id, d.target_layer_ids) == (1e6, 151669, [4, 12, 19, 26, 33])


def test_target_layer_ids_match_fixture(pkg, golden_dir):
    with open(os.path.join(golden_dir, "layer_ids.json")) as f:
        ids = json.load(f)
    for key, val in ids.items():
        nt, nd = map(int, key.split(","))
        assert pkg.build_target_layer_ids(nt, nd) == val


def test_extract_context_feature_and_sample(pkg):
    import torch
    hs = [torch.full((1, 3, 2), float(i)) for i in range(6)]
    out = pkg.extract_context_feature(hs, [0, 2, 4])    # embedding first -> shift by one
    assert out[0, 0].tolist() == [1, 1, 3, 3, 5, 5]
    out = pkg.extract_context_feature(hs[:3], [7, 8, 9])
    assert out.shape == (1, 3, 6)
    assert pkg.sample(torch.tensor([[1.0, 3.0, 3.0]])).tolist() == [1]


def _attn_splits(batch, nkv, kv_len, sms, rows):
    """Restatement of the library's KV split choice (attention.cu
    attn_pick_split): with more than 128 query rows per kv head (one CTA per
    SM) minimise waves * (kv tiles per CTA + 6); otherwise cover the SMs once."""
    per = batch * nkv
    tiles = -(-kv_len // 64)
    s = -(-sms // per)
    if rows > 128:
        cap, best = max(s, 8), None
        for c in range(1, min(cap, tiles) + 1):
            per_cta = -(-tiles // c)
            se = -(-tiles // per_cta)
            cost = -(-(per * se) // sms) * (per_cta + 6)
            if best is None or cost < best:
                best, s = cost, se
    s = max(1, min(s, tiles))
    ch = -(-(-(-kv_len // s)) // 64) * 64
    return -(-kv_len // ch)


def test_attention_split_waves(pkg):
    """The attention workspace (C entry dflash_attention_workspace_size) holds
    batch * NKV * splits partial rows: the split count avoids a partial second
    wave of one-CTA-per-SM grids (27B dims: 40 / 8 heads, block 32)."""
    import torch
    lib = pkg._native.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148

    def ws(batch, nq, nkv, block, kv_len, splits):
        rows = batch * nkv * splits * (nq // nkv) * block
        return rows * 130 * 4 + (kv_len + block) * 64 * 8 + 64 * 4 + 256

    for batch, nq, nkv, block, kv_len in [(1, 40, 8, 32, 32800), (16, 40, 8, 32, 32800), (1, 40, 8, 32, 4128),
                                          (16, 40, 8, 32, 8224), (4, 40, 8, 32, 16416), (1, 32, 8, 16, 2064),
                                          (256, 32, 8, 16, 1104)]:
        s = _attn_splits(batch, nkv, kv_len, sms, (nq // nkv) * block)
        assert lib.dflash_attention_workspace_size(batch, nq, nkv, block, kv_len) == ws(batch, nq, nkv, block,
                                                                                       kv_len, s)
    if sms == 148:
        assert _attn_splits(1, 8, 32800, 148, 160) == 18      # 144 CTAs, one wave (19 left 4 in a second)
        assert _attn_splits(16, 8, 32800, 148, 160) == 8      # 1024 CTAs, 6.9 waves
        assert _attn_splits(16, 8, 8224, 148, 160) == 1
        assert _attn_splits(16, 8, 16416, 148, 160) == 1
        assert _attn_splits(1, 8, 4128, 148, 160) == 17       # the c3 step: 136 CTAs


def test_attention_split_model_properties(pkg):
    """Across random shapes, the library's attention workspace equals the
    restated split choice, and the splits tile the kv rows: chunks are whole
    64-row tiles, every split holds at least one kv row, and together they
    cover kv_len."""
    from hypothesis import given, settings, strategies as st
    import torch
    lib = pkg._native.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148

    @settings(max_examples=300, deadline=None, derandomize=True)
    @given(batch=st.integers(1, 300), nkv=st.sampled_from([1, 2, 4, 8]), g=st.integers(1, 8),
           block=st.integers(1, 64), kv_len=st.integers(1, 40000))
    def check(batch, nkv, g, block, kv_len):
        rows = g * block
        if rows > 256:
            return
        s = _attn_splits(batch, nkv, kv_len, sms, rows)
        per = batch * nkv * s * rows
        want = per * 130 * 4 + (kv_len + block) * 64 * 8 + 64 * 4 + 256
        assert lib.dflash_attention_workspace_size(batch, g * nkv, nkv, block, kv_len) == want
        ch = -(-(-(-kv_len // s)) // 64) * 64
        assert ch % 64 == 0 and s >= 1
        assert (s - 1) * ch < kv_len <= s * ch

    check()


def test_key_padding_lengths(pkg):
    """The masks DFlashDraftModel.__call__ takes (dflash.py:315 passes them to
    SDPA): all-kept -> None, left padding -> kept context counts, anything the
    device path cannot express exactly -> NotImplementedError."""
    import torch
    f = pkg.key_padding_lengths
    b, q, C = 3, 4, 6
    L = C + q
    assert f(torch.zeros(L), b, q, C) is None
    assert f(torch.ones(1, 1, q, L, dtype=torch.bool), b, q, C) is None
    keep = torch.ones(b, 1, 1, L, dtype=torch.bool)
    keep[0, 0, 0, :2] = False          # sequence 0 keeps its last 4 context rows
    keep[2, 0, 0, :C] = False          # sequence 2 keeps no context
    assert f(keep, b, q, C) == [4, 6, 0]
    add = torch.where(keep, torch.tensor(0.0), torch.tensor(-1e4))        # the ANE padding value
    assert f(add, b, q, C) == [4, 6, 0]
    assert f(torch.where(keep, 0.0, float("-inf")), b, q, C) == [4, 6, 0]
    right = torch.ones(b, 1, 1, L, dtype=torch.bool)
    right[1, 0, 0, C - 2:C] = False    # right padding: kept rows first
    with pytest.raises(NotImplementedError):
        f(right, b, q, C)
    with pytest.raises(NotImplementedError):
        f(torch.full((L,), 0.5), b, q, C)                                 # a bias
    blk = torch.ones(L, dtype=torch.bool)
    blk[C] = False
    with pytest.raises(NotImplementedError):
        f(blk, b, q, C)                                                   # a masked block key
    perq = torch.ones(1, 1, q, L, dtype=torch.bool)
    perq[0, 0, 1, 0] = False
    with pytest.raises(NotImplementedError):
        f(perq, b, q, C)                                                  # query-dependent
    with pytest.raises(ValueError):
        f(torch.zeros(L + 1), b, q, C)


def test_oracle_masked_sdpa_matches_truncation():
    """The oracle's SDPA mask (dflash.py:315): masking keys equals dropping
    them, additive -1e4 included."""
    import torch
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(2, 4, n, 16, generator=g, dtype=torch.float64) for n in (5, 9, 9))
    keep = torch.ones(2, 1, 1, 9, dtype=torch.bool)
    keep[1, :, :, :3] = False
    full = O.sdpa(q, k, v, 0.25, torch.where(keep, 0.0, -1e4).double())
    assert torch.allclose(full[0], O.sdpa(q[:1], k[:1], v[:1], 0.25)[0], atol=1e-12)
    assert torch.allclose(full[1], O.sdpa(q[1:], k[1:, :, 3:], v[1:, :, 3:], 0.25)[0], atol=1e-12)
