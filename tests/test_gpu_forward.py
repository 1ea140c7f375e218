"""End-to-end parity of the draft step (C-ABI dflash_forward) against the CPU
oracle on identical seeded weights and inputs, and against the golden
fixture produced by the reference's own dflash.py.

Tolerances (north star): final hidden states cosine >= 0.9995 and
max-abs <= 2e-2 (bf16/f16 activations, fp32 accumulation); draft ids equal to
the oracle's greedy ids wherever the oracle's top-1/top-2 logit margin is
above the stated near-tie bound; acceptance is integer work and must match
exactly given the ids.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import dflash_oracle as O
from helpers import bf16_value, check_hidden, check_tokens, fixture_case, gpu_model, pkg_config, tiny_cfg

pytestmark = pytest.mark.gpu

MARGIN = 0.05   # logits: near-ties below this may flip under bf16/f16 rounding


def _run_case(pkg, ocfg, batch, ctx, seed, num_layers=None):
    q8, dense = O.synth_weights(ocfg, seed=seed)
    model = gpu_model(pkg, ocfg, q8, max_batch=batch, max_ctx=max(ctx, 1))
    noise, th = O.synth_inputs(ocfg, batch, ctx, ocfg.block_size, seed=seed + 1)
    if num_layers is not None:
        model.num_draft_layers = num_layers
    hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    ref = O.draft_forward(ocfg, dense, noise, th, num_layers=num_layers)
    logits = O.draft_logits(dense, ref, ocfg.block_size)
    torch.cuda.synchronize()
    c, m = check_hidden(hid, ref)
    eq, tot, near = check_tokens(toks, logits, MARGIN)
    model.close()
    return c, m, eq, tot, near


@pytest.mark.parametrize("batch,ctx", [(1, 12), (2, 33), (1, 0), (4, 130)])
def test_forward_tiny(pkg, batch, ctx):
    _run_case(pkg, tiny_cfg(), batch, ctx, seed=batch * 100 + ctx)


def test_forward_mid_ragged_tiles(pkg):
    # hidden 1024, GQA 4, vocab not a multiple of 32, ctx not a multiple of 128
    ocfg = tiny_cfg(hidden_size=1024, intermediate_size=2816, num_attention_heads=8,
                    num_key_value_heads=2, vocab_size=5003, block_size=16, num_hidden_layers=2)
    _run_case(pkg, ocfg, 2, 300, seed=5)


def test_forward_heads_not_multiple_of_8(pkg):
    # 12 query heads: the split merge that writes the o-projection's limbs runs
    # as clusters of two CTAs per row, the second holding 4 heads; 3 sequences
    # of block 8 leave 8 padding rows in the 32-row limb tile
    ocfg = tiny_cfg(num_attention_heads=12, num_key_value_heads=4)
    _run_case(pkg, ocfg, 3, 150, seed=12)


def test_forward_num_draft_layers(pkg):
    _run_case(pkg, tiny_cfg(num_hidden_layers=3), 1, 40, seed=9, num_layers=2)


def test_forward_27b_dims_one_layer(pkg):
    """The bench config's dims (hidden 5120, 40/8 heads, FFN 17408, full vocab,
    block 32) at one layer and ctx 200 so the CPU oracle stays quick."""
    ocfg = O.OracleConfig(hidden_size=5120, num_hidden_layers=1, intermediate_size=17408,
                          num_attention_heads=40, num_key_value_heads=8, vocab_size=151936,
                          block_size=32)
    pcfg = pkg_config(pkg, ocfg)
    w, lm = pkg.synth_weights_q8(pcfg, seed=3, random_norms=True)
    model = pkg.DFlashDraftModel(pcfg, w, lm, max_batch=1, max_ctx=200, max_block=32)
    noise, th = O.synth_inputs(ocfg, 1, 200, 32, seed=4)
    hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    torch.cuda.synchronize()
    # oracle weights: exact dequantised copies of what the GPU holds
    deq = lambda l, k: (l.q[k].float() * l.s[k].float()[:, None]).cpu()
    layers = [O.OracleLayer(**{k: deq(l, k) for k in ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]},
                            in_norm=l.input_layernorm.cpu(), post_norm=l.post_attention_layernorm.cpu(),
                            q_norm=l.q_norm.cpu(), k_norm=l.k_norm.cpu()) for l in w.layers]
    dense = O.OracleWeights(w.fc.float().cpu(), w.hidden_norm.cpu(), w.norm.cpu(), lm.float().cpu(), layers)
    ref = O.draft_forward(ocfg, dense, noise, th)
    check_hidden(hid, ref)
    check_tokens(toks, O.draft_logits(dense, ref, 32), MARGIN)
    model.close()


@pytest.mark.parametrize("layers", [1, 2])
def test_forward_4b_dims_c1_shape(pkg, layers):
    """The CPU-plumbing config's dims (Qwen3-4B class: hidden 2560, 32/8
    heads, FFN 9728, full vocab, block 16, ctx 64, batch 1) through the W8A16
    device path; the oracle gets the exact dequantised weights."""
    ocfg = O.OracleConfig(hidden_size=2560, num_hidden_layers=layers, intermediate_size=9728,
                          num_attention_heads=32, num_key_value_heads=8, vocab_size=151936,
                          block_size=16)
    pcfg = pkg_config(pkg, ocfg)
    w, lm = pkg.synth_weights_q8(pcfg, seed=13, random_norms=True)
    model = pkg.DFlashDraftModel(pcfg, w, lm, max_batch=1, max_ctx=64, max_block=16)
    noise, th = O.synth_inputs(ocfg, 1, 64, 16, seed=14)
    hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    torch.cuda.synchronize()
    deq = lambda l, k: (l.q[k].float() * l.s[k].float()[:, None]).cpu()
    ls = [O.OracleLayer(**{k: deq(l, k) for k in ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]},
                        in_norm=l.input_layernorm.cpu(), post_norm=l.post_attention_layernorm.cpu(),
                        q_norm=l.q_norm.cpu(), k_norm=l.k_norm.cpu()) for l in w.layers]
    dense = O.OracleWeights(w.fc.float().cpu(), w.hidden_norm.cpu(), w.norm.cpu(), lm.float().cpu(), ls)
    ref = O.draft_forward(ocfg, dense, noise, th)
    check_hidden(hid, ref)
    check_tokens(toks, O.draft_logits(dense, ref, 16), MARGIN)
    model.close()


def test_forward_accept_fused(pkg):
    ocfg = tiny_cfg()
    q8, dense = O.synth_weights(ocfg, seed=21)
    model = gpu_model(pkg, ocfg, q8, max_batch=2, max_ctx=16)
    noise, th = O.synth_inputs(ocfg, 2, 16, ocfg.block_size, seed=22)
    _, toks, _, _ = model.draft_step(noise.cuda(), th.cuda())
    t = torch.cat([toks.cpu(), torch.full((2, 1), 7, dtype=torch.int32)], dim=1)
    t[1, 2] = (t[1, 2] + 1) % ocfg.vocab_size
    _, toks2, acc, cor = model.draft_step(noise.cuda(), th.cuda(), target_tokens=t.cuda())
    assert torch.equal(toks2.cpu(), toks.cpu())
    want = [O.accept(d.tolist(), tt.tolist()) for d, tt in zip(toks.cpu(), t)]
    assert acc.cpu().tolist() == [w[0] for w in want] == [ocfg.block_size - 1, 2]
    assert cor.cpu().tolist() == [w[1] for w in want]
    model.close()


def test_forward_matches_reference_fixture(pkg, golden_dir):
    """The golden fixture's weights and inputs (generated by the reference's own
    dflash.py; bf16-exact fc / lm_head / inputs) through the CUDA path, against
    the reference's fp64 outputs and its greedy ids."""
    z = np.load(os.path.join(golden_dir, "dflash_forward_small.npz"))
    ocfg, q8, dense = fixture_case(z)
    model = gpu_model(pkg, ocfg, q8, max_batch=2, max_ctx=20)
    for name in ["s1", "s2"]:
        noise = torch.from_numpy(bf16_value(z[f"{name}.noise"])).float()
        th = torch.from_numpy(bf16_value(z[f"{name}.th"])).float()
        hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
        torch.cuda.synchronize()
        ref = torch.from_numpy(z[f"{name}.hidden"])
        check_hidden(hid, ref)
        check_tokens(toks, O.draft_logits(dense, ref, ocfg.block_size), MARGIN)
    model.close()


@pytest.mark.parametrize("batch,bf16", [(1, False), (3, True)])
def test_forward_soft_anchor(pkg, batch, bf16):
    """With anchor_logits the step embeds block row 0 as the soft anchor
    (generate.py:1422-1436) inside the forward, reading the lm_head tiles it
    holds: bit-identical to a step fed noise whose row 0 is the standalone
    soft anchor over the row-major table, and within the north-star
    tolerance of the oracle forward on that noise."""
    import importlib
    K = importlib.import_module("mirror-sd_b200.kernels")
    ocfg = tiny_cfg(vocab_size=3001, block_size=8)
    q8, dense = O.synth_weights(ocfg, seed=77)
    model = gpu_model(pkg, ocfg, q8, max_batch=batch, max_ctx=40)
    noise, th = O.synth_inputs(ocfg, batch, 40, ocfg.block_size, seed=78)
    g = torch.Generator().manual_seed(79)
    logits = torch.randn(batch, ocfg.vocab_size, generator=g) * 3.0
    if bf16:
        logits = logits.to(torch.bfloat16)
    E = torch.as_tensor(q8["lm_head"]).to(torch.bfloat16)
    hid_a, tok_a, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True,
                                          anchor_logits=logits.cuda())
    anchor = K.soft_anchor(logits.cuda(), E.cuda(), 8)
    noise2 = noise.clone().to(torch.bfloat16)
    noise2[:, 0] = anchor.cpu()
    hid_b, tok_b, _, _ = model.draft_step(noise2.cuda(), th.cuda(), hidden_fp32=True)
    torch.cuda.synchronize()
    assert torch.equal(hid_a, hid_b) and torch.equal(tok_a, tok_b)
    ref = O.draft_forward(ocfg, dense, noise2.float(), th)
    check_hidden(hid_a, ref)
    # without anchor_logits the noise row 0 is used again (nothing persists)
    hid_c, _, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    hid_d, _, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True,
                                      anchor_logits=None)
    assert torch.equal(hid_c, hid_d) and not torch.equal(hid_c, hid_a)
    with pytest.raises(Exception):
        model.draft_step(noise.cuda(), th.cuda(), anchor_logits=logits[:, :10].cuda())
    with pytest.raises(Exception):
        model.draft_step(noise.cuda(), th.cuda(), anchor_logits=logits.cuda(), anchor_top_k=17)
    model.close()


def test_forward_target_layers_in_place(pkg):
    """extract_context_feature fused into the fc GEMM (dflash.py:122-130): the
    F target layers passed as a list (contiguous, as column slices of a wider
    buffer with a longer row pitch, and packed ragged with ctx_lens) give the
    same bits as the concatenated [*, F*H] input."""
    ocfg = tiny_cfg(num_hidden_layers=2)
    q8, _ = O.synth_weights(ocfg, seed=91)
    model = gpu_model(pkg, ocfg, q8, max_batch=3, max_ctx=150)
    H, F = ocfg.hidden_size, ocfg.num_target_features
    noise, th = O.synth_inputs(ocfg, 2, 150, ocfg.block_size, seed=92)
    noise, th = noise.cuda(), th.cuda().to(torch.bfloat16)
    want, wtok, _, _ = model.draft_step(noise, th, hidden_fp32=True)
    layers = [th[..., f * H:(f + 1) * H].contiguous() for f in range(F)]
    got, gtok, _, _ = model.draft_step(noise, layers, hidden_fp32=True)
    assert torch.equal(got, want) and torch.equal(gtok, wtok)
    wide = torch.zeros(2, 150, F, H + 64, dtype=torch.bfloat16, device="cuda")
    for f in range(F):
        wide[:, :, f, :H] = layers[f]
    strided = [wide[:, :, f, :H] for f in range(F)]         # row pitch F*(H+64)
    got2, _, _, _ = model.draft_step(noise, strided, hidden_fp32=True)
    assert torch.equal(got2, want)
    views = [th[..., f * H:(f + 1) * H] for f in range(F)]   # column slices of the concat itself
    got3, _, _, _ = model.draft_step(noise, views, hidden_fp32=True)
    assert torch.equal(got3, want)
    # ragged packed rows (ctx_lens), three sequences
    lens = [7, 0, 131]
    n3, th3 = O.synth_inputs(ocfg, 3, 131, ocfg.block_size, seed=93)
    packed = torch.cat([th3[s, :lens[s]] for s in range(3)]).cuda().to(torch.bfloat16)
    want4, _, _, _ = model.draft_step(n3.cuda(), packed, hidden_fp32=True, ctx_lens=lens)
    got4, _, _, _ = model.draft_step(n3.cuda(), [packed[:, f * H:(f + 1) * H] for f in range(F)],
                                     hidden_fp32=True, ctx_lens=lens)
    assert torch.equal(got4, want4)
    with pytest.raises(ValueError):
        model.draft_step(noise, layers[:-1])
    model.close()


def test_forward_rejects_bad_shapes(pkg):
    ocfg = tiny_cfg()
    q8, _ = O.synth_weights(ocfg, seed=1)
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=8)
    noise, th = O.synth_inputs(ocfg, 1, 9, ocfg.block_size, seed=2)
    with pytest.raises(ValueError):
        model.draft_step(noise.cuda(), th.cuda())          # ctx 9 > max_ctx 8
    noise2, th2 = O.synth_inputs(ocfg, 2, 4, ocfg.block_size, seed=2)
    with pytest.raises(ValueError):
        model.draft_step(noise2.cuda(), th2.cuda())        # batch 2 > max_batch 1
    with pytest.raises(ValueError):
        model.set_block_size(ocfg.block_size + 1)
    model.close()


def test_bounded_wait_expiry_is_reported_and_the_context_survives(pkg):
    """Failure detection without a fault: a bounded mbarrier wait that
    nothing completes gives up after its poll limit, records the timeout in
    the handle's error word (device_status raises, then reads clean), and the
    next draft step on the same context is still correct."""
    import time
    ocfg = tiny_cfg()
    q8, dense = O.synth_weights(ocfg, seed=81)
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=16)
    noise, th = O.synth_inputs(ocfg, 1, 16, ocfg.block_size, seed=82)
    model.device_status()                     # clean before
    t0 = time.time()
    model.probe_bounded_wait(1 << 14)
    with pytest.raises(RuntimeError, match="wait limit"):
        model.device_status()
    assert time.time() - t0 < 10.0
    model.device_status()                     # cleared by the read
    hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    torch.cuda.synchronize()
    ref = O.draft_forward(ocfg, dense, noise, th)
    check_hidden(hid, ref)
    check_tokens(toks, O.draft_logits(dense, ref, ocfg.block_size), MARGIN)
    model.device_status()
    model.close()


def test_forward_activations_beyond_f16_range(pkg):
    """Projection inputs of about 1e5 and SiLU * up products of about 1e8 (a
    post-attention norm weight of 3e4): the W8A16 path splits its fp32 rows
    into limbs directly, so nothing overflows where f16 (max 65504) would,
    and the hidden states stay within the north-star tolerance of the fp32
    oracle (the reference's MLP intermediates are bf16, dflash.py:322-330)."""
    ocfg = tiny_cfg(hidden_size=1024, intermediate_size=2816, num_attention_heads=8, num_key_value_heads=2,
                    vocab_size=5003, block_size=16, num_hidden_layers=2)
    q8, dense = O.synth_weights(ocfg, seed=31)
    big = (3e4 * (1.0 + 0.1 * np.random.default_rng(32).standard_normal(ocfg.hidden_size))).astype(np.float32)
    q8["layers"][0]["post_norm"] = big
    dense.layers[0].post_norm = torch.from_numpy(big)
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=64)
    noise, th = O.synth_inputs(ocfg, 1, 64, ocfg.block_size, seed=33)
    hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = O.draft_forward(ocfg, dense, noise, th)
        # the magnitudes this case drives through layer 0's MLP
        lw = dense.layers[0]
        h = noise + O.attention(ocfg, lw, O.rms_norm(noise, lw.in_norm, 1e-6),
                                O.context_projection(ocfg, dense, th))
        x2 = O.rms_norm(h, lw.post_norm, 1e-6)
        act = O.silu(x2 @ lw.wg.T) * (x2 @ lw.wu.T)
    assert float(x2.abs().max()) > 1e5 and float(act.abs().max()) > 1e7
    assert torch.isfinite(hid).all()
    check_hidden(hid, ref, label="W8A16, activations beyond the f16 range")
    check_tokens(toks, O.draft_logits(dense, ref, ocfg.block_size), MARGIN)
    model.close()


@pytest.mark.parametrize("additive", [False, True])
def test_forward_left_padding_mask(pkg, additive):
    """``__call__`` with a key-padding mask (dflash.py:315 passes it to SDPA):
    3 sequences in one [b, ctx, F*H] buffer keeping their last 40 / 75 / 0
    context rows, against the oracle's masked SDPA over the padded inputs (each
    kept key at its own position), as a boolean mask and as the ANE's additive
    -1e4 padding."""
    ocfg = tiny_cfg()
    b, C, B = 3, 75, ocfg.block_size
    q8, dense = O.synth_weights(ocfg, seed=21)
    model = gpu_model(pkg, ocfg, q8, max_batch=b, max_ctx=C)
    noise, th = O.synth_inputs(ocfg, b, C, B, seed=22)
    keep = torch.ones(b, 1, 1, C + B, dtype=torch.bool)
    keep[0, :, :, :C - 40] = False
    keep[2, :, :, :C] = False
    mask = torch.where(keep, 0.0, -1e4) if additive else keep
    hid = model(noise.to(torch.bfloat16).cuda(), th.to(torch.bfloat16).cuda(), mask=mask)
    torch.cuda.synchronize()
    ref = O.draft_forward(ocfg, dense, noise.to(torch.bfloat16).float(), th.to(torch.bfloat16).float(),
                          mask=mask.double() if additive else keep)
    check_hidden(hid, ref, label=f"left-padding mask ({'additive' if additive else 'boolean'})")
    with pytest.raises(NotImplementedError):
        right = torch.ones(C + B, dtype=torch.bool)
        right[C - 5:C] = False
        model(noise.to(torch.bfloat16).cuda(), th.to(torch.bfloat16).cuda(), mask=right)
    model.close()
