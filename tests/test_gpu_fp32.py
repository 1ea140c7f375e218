"""The fp32-accumulate mode (dflash_create_f32): fp32 weights, activations and
accumulation on the CUDA cores, against the fp32 CPU oracle.

draft token ids and accepted lengths bit-exact under
fp32-accumulate mode.  A differing id is allowed only where the oracle's own
top-1 / top-2 logit margin is at most 1e-4 (the two fp32 evaluations sum in
different orders, so an exact tie within rounding may go either way); every
such row is listed in the parity table.  Hidden states: cosine >= 0.99999 and
max-abs <= 1e-3 (fp32 against fp32).

c1 is BASELINE's CPU plumbing config: Qwen3-4B-class dims (hidden 2560, 32/8
heads, FFN 9728, 5 layers, vocab 151936, tied lm_head), every weight fp32
N(0, 0.02), block 16, ctx 64, batch 1, target_hidden N(0, 1), block ids
uniform over the vocabulary with position 0 the mask id, seed 0.
"""
import pytest
import torch

from oracle import dflash_oracle as O
from helpers import PARITY, check_hidden, oracle_weights_from_f32, pkg_config, tiny_cfg, token_stats

pytestmark = pytest.mark.gpu

TIE = 1e-4      # oracle margin below which a differing id is a tie within fp32 rounding
COS, MAXABS = 0.99999, 1e-3


def _check_ids(toks, logits, label):
    rows, n_diff, max_gap, diffs = token_stats(toks, logits)
    margin = O.top2_margin(logits.double()).reshape(-1)
    PARITY.setdefault(label, {}).update(rows=rows, ids_differ=n_diff, max_gap=max_gap, tol=TIE,
                                        min_margin=float(margin.min()))
    bad = [d for d in diffs if float(margin[d[0]]) > TIE]
    assert not bad, f"fp32 draft ids differ from the oracle at clear maxima: {bad}"


def _accept_exact(model, noise, th, toks, ref_ids, **kw):
    """Fused acceptance against targets that keep a prefix of the oracle's ids:
    the accepted length and correction equal the oracle's own acceptance."""
    b, n = ref_ids.shape
    g = torch.Generator().manual_seed(5)
    cut = torch.randint(0, n + 1, (b,), generator=g)
    tgt = torch.cat([ref_ids.clone(), torch.full((b, 1), 3, dtype=torch.int32)], dim=1)
    for i in range(b):
        if cut[i] < n:
            tgt[i, cut[i]] = (tgt[i, cut[i]] + 1) % 1000
    _, t2, acc, cor = model.draft_step(noise, th, target_tokens=tgt.cuda(), want_hidden=False, **kw)
    assert torch.equal(t2.cpu(), toks.cpu())
    # exact given the ids; equal to the oracle's own acceptance whenever the
    # ids are (they may differ only at an fp32 tie, checked by _check_ids)
    got = [(int(a), int(c)) for a, c in zip(acc.cpu(), cor.cpu())]
    assert got == [O.accept(r.tolist(), t.tolist()) for r, t in zip(toks.cpu(), tgt)]
    if torch.equal(toks.cpu().to(torch.int32), ref_ids.to(torch.int32)):
        assert got == [O.accept(r.tolist(), t.tolist()) for r, t in zip(ref_ids, tgt)]


def test_c1_fp32_ids_and_accept_bit_exact(pkg):
    ocfg = O.OracleConfig(hidden_size=2560, num_hidden_layers=5, intermediate_size=9728, num_attention_heads=32,
                          num_key_value_heads=8, vocab_size=151936, block_size=16)
    cfg = pkg_config(pkg, ocfg)
    w, lm = pkg.synth_weights_f32(cfg, seed=0)
    model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=1, max_ctx=64, max_block=16)
    assert model.fp32
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, ocfg.vocab_size, (1, 16), generator=g)
    ids[0, 0] = ocfg.mask_token_id
    noise = lm[ids.cuda()]                                   # the tied embedding of the block ids
    th = torch.randn(1, 64, 5 * ocfg.hidden_size, generator=g)
    hid, toks, _, _ = model.draft_step(noise, th.cuda())
    torch.cuda.synchronize()
    assert hid.dtype == torch.float32
    dense = oracle_weights_from_f32(w, lm)
    with torch.no_grad():
        ref = O.draft_forward(ocfg, dense, noise.cpu(), th)
        logits = O.draft_logits(dense, ref, 16)
    label = "c1 4B fp32-accumulate (5 layers, ctx 64)"
    check_hidden(hid, ref, cos_min=COS, max_abs=MAXABS, label=label)
    _check_ids(toks, logits, label)
    _accept_exact(model, noise, th.cuda(), toks, O.greedy(logits))
    model.close()


@pytest.mark.parametrize("seed", [1, 2])
def test_fp32_ragged_batch_random_norms(pkg, seed):
    """Three sequences with ragged contexts (one empty) and RoPE offsets,
    random norm weights, a vocabulary that is not a multiple of 128, and
    12 query heads over 4 kv heads."""
    ocfg = tiny_cfg(hidden_size=512, num_hidden_layers=3, intermediate_size=1280, num_attention_heads=12,
                    num_key_value_heads=4, vocab_size=5003, block_size=8)
    cfg = pkg_config(pkg, ocfg)
    w, lm = pkg.synth_weights_f32(cfg, seed=seed, random_norms=True)
    lens, offs = [0, 5, 70], [3, 0, 100]
    model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=3, max_ctx=70, max_block=8)
    g = torch.Generator().manual_seed(seed)
    noise = torch.randn(3, 8, ocfg.hidden_size, generator=g) * 0.02
    th = [torch.randn(c, 5 * ocfg.hidden_size, generator=g) for c in lens]
    hid, toks, _, _ = model.draft_step(noise.cuda(), torch.cat(th).cuda(), ctx_lens=lens, rope_offsets=offs)
    torch.cuda.synchronize()
    dense = oracle_weights_from_f32(w, lm)
    refs, logits = [], []
    with torch.no_grad():
        for i in range(3):
            cache = [O.OracleKVCache() for _ in range(ocfg.num_hidden_layers)]
            for c in cache:
                c.offset = offs[i]
            r = O.draft_forward(ocfg, dense, noise[i:i + 1], th[i][None], cache=cache)
            refs.append(r)
            logits.append(O.draft_logits(dense, r, 8))
    label = f"fp32 ragged 3 seqs, seed {seed}"
    check_hidden(hid, torch.cat(refs), cos_min=COS, max_abs=MAXABS, label=label)
    _check_ids(toks, torch.cat(logits), label)
    _accept_exact(model, noise.cuda(), torch.cat(th).cuda(), toks, O.greedy(torch.cat(logits)),
                  ctx_lens=lens, rope_offsets=offs)
    model.close()


def test_fp32_from_q8_matches_dequantised_oracle(pkg):
    """A W8A16 checkpoint run in fp32-accumulate mode (DFlashWeightsF32.from_q8:
    the exact fp32 values q * fp16(s)) at the 27B dims, one layer, ctx 200."""
    ocfg = O.OracleConfig(hidden_size=5120, num_hidden_layers=1, intermediate_size=17408, num_attention_heads=40,
                          num_key_value_heads=8, vocab_size=151936, block_size=32)
    cfg = pkg_config(pkg, ocfg)
    wq, lmq = pkg.synth_weights_q8(cfg, seed=3, random_norms=True)
    w = pkg.DFlashWeightsF32.from_q8(wq)
    lm = lmq.float()
    del wq, lmq
    model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=1, max_ctx=200, max_block=32)
    noise, th = O.synth_inputs(ocfg, 1, 200, 32, seed=4)
    hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda())
    torch.cuda.synchronize()
    dense = oracle_weights_from_f32(w, lm)
    with torch.no_grad():
        ref = O.draft_forward(ocfg, dense, noise, th)
        logits = O.draft_logits(dense, ref, 32)
    label = "27B dims fp32-accumulate from int8 (1 layer, ctx 200)"
    check_hidden(hid, ref, cos_min=COS, max_abs=MAXABS, label=label)
    _check_ids(toks, logits, label)
    model.close()


def test_fp32_rejects_stateful_arguments(pkg):
    ocfg = tiny_cfg()
    cfg = pkg_config(pkg, ocfg)
    w, lm = pkg.synth_weights_f32(cfg, seed=0)
    model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=1, max_ctx=8, max_block=8)
    noise = torch.zeros(1, 8, ocfg.hidden_size, device="cuda")
    th = torch.zeros(1, 4, 5 * ocfg.hidden_size, device="cuda")
    with pytest.raises(ValueError):
        model.draft_step(noise, th, anchor_logits=torch.zeros(1, ocfg.vocab_size, device="cuda"))
    with pytest.raises(ValueError):
        model.draft_step(noise, [th[..., :ocfg.hidden_size]] * 5)
    model.close()
