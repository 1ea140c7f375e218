"""Stateful draft KV cache and ragged batches on the device, against the
reference fixture and the CPU oracle.

The cache follows dflash.py:139-212:
- append the step's [context; block] K/V rows;
- keep the sink rows and the last window rows once the list outgrows them;
- ``trim(n)`` drops the last n rows and moves the offset back.

The device keeps the rows in rings and moves only a start index.  These tests
drive many steps, so the ring wraps several times, and compare every step's
hidden states and draft ids with the oracle's.

Tolerances as in test_gpu_forward.py:
- hidden states: cosine >= 0.9995 and max-abs <= 2e-2;
- draft ids: equal wherever the oracle's top-2 margin exceeds 0.05;
- offsets and lengths: exact.
"""
import os

import numpy as np
import pytest
import torch

from oracle import dflash_oracle as O
from helpers import bf16_value, check_hidden, check_tokens, fixture_case, gpu_model, tiny_cfg

pytestmark = pytest.mark.gpu

MARGIN = 0.05


def _oracle_cache(ocfg, sink, window, offset=0):
    cache = [O.OracleKVCache(sink_size=sink, window_size=window) for _ in range(ocfg.num_hidden_layers)]
    for c in cache:
        c.offset = offset
    return cache


def test_cache_matches_reference_fixture(pkg, golden_dir):
    """The three-step cached sequence frozen from the reference's own
    DFlashKVCache (sink 4, window 16; eviction in steps 2 and 3)."""
    z = np.load(os.path.join(golden_dir, "dflash_forward_small.npz"))
    ocfg, q8, dense = fixture_case(z)
    B = ocfg.block_size
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=16)
    cache = model.make_cache(sink_size=4, window_size=16)
    for step in range(3):
        p = f"c{step}."
        noise = torch.from_numpy(bf16_value(z[p + "noise"])).float()
        th = torch.from_numpy(bf16_value(z[p + "th"])).float()
        hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), cache=cache, hidden_fp32=True)
        torch.cuda.synchronize()
        ref = torch.from_numpy(z[p + "hidden"])
        check_hidden(hid, ref)
        check_tokens(toks, O.draft_logits(dense, ref, B), MARGIN)
        assert cache[0].offset == int(z[p + "offset_after_call"])
        assert cache[0].keys.shape[2] == int(z[p + "len_after_call"])
        for c in cache:
            c.trim(B)
        assert cache[0].offset == int(z[p + "offset_after_trim"])
        assert cache[0].keys.shape[2] == int(z[p + "len_after_trim"])
        # stored K (layer 0) and V (layer 1) rows, logical order, f16 on the device
        k0 = cache[0].keys.float().cpu()
        v1 = cache[1].values.float().cpu()
        assert (k0 - torch.from_numpy(z[p + "k0_after_trim"]).float()).abs().max() < 2e-2
        assert (v1 - torch.from_numpy(z[p + "v1_after_trim"]).float()).abs().max() < 2e-2
    model.close()


def _decode_run(pkg, ocfg, sink, window, ctx_seq, batch=1, seed=0, max_len=None):
    """Replays a decode-like sequence: prefill, then steps with a few new
    context rows each, trim(B) after every draft."""
    B = ocfg.block_size
    q8, dense = O.synth_weights(ocfg, seed=seed)
    model = gpu_model(pkg, ocfg, q8, max_batch=batch, max_ctx=max(ctx_seq))
    cache = model.make_cache(sink_size=sink, window_size=window, max_len=max_len)
    ocache = _oracle_cache(ocfg, sink, window)
    for step, ctx in enumerate(ctx_seq):
        noise, th = O.synth_inputs(ocfg, batch, ctx, B, seed=seed * 1000 + step)
        hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), cache=cache, hidden_fp32=True)
        ref = O.draft_forward(ocfg, dense, noise, th, cache=ocache)
        torch.cuda.synchronize()
        check_hidden(hid, ref)
        check_tokens(toks, O.draft_logits(dense, ref, B), MARGIN)
        assert cache[0].offset == ocache[0].offset
        assert cache[-1].keys.shape[2] == ocache[-1].keys.shape[2]
        for c, oc in zip(cache, ocache):
            c.trim(B)
            oc.trim(B)
        assert cache[0].offset == ocache[0].offset
    # logical rows after the last trim: same K/V as the oracle's cache
    k = cache[0].keys.float().cpu()
    assert k.shape == ocache[0].keys.shape
    assert (k - ocache[0].keys.float()).abs().max() < 2e-2
    return model, cache


def test_cache_eviction_ring_wraps(pkg):
    """sink 8 / window 40: eviction from the first step, and 30 steps wrap the
    ring (window + max_ctx + max_block = 40 + 70 + 8 slots) several times."""
    ctx_seq = [70] + [1 + (i * 5) % 8 for i in range(29)]
    model, _ = _decode_run(pkg, tiny_cfg(), 8, 40, ctx_seq, seed=3)
    model.close()


def test_cache_batch2_default_window(pkg):
    """Two sequences stepping together (the reference's batched cache), with
    the reference's default sink 64 / window 1024."""
    ctx_seq = [300, 3, 9, 1, 5]
    model, _ = _decode_run(pkg, tiny_cfg(), 64, 1024, ctx_seq, batch=2, seed=4)
    model.close()


def test_cache_without_eviction_and_overflow(pkg):
    """sink 0 disables eviction (dflash.py:180-181); a step that would exceed
    max_len rows is rejected and leaves the cache unchanged."""
    ocfg = tiny_cfg()
    model, cache = _decode_run(pkg, ocfg, 0, 0, [20, 4, 7], seed=5, max_len=50)
    before = (cache[0].offset, cache[0].keys.shape[2])   # 31 rows held
    noise, th = O.synth_inputs(ocfg, 1, 20, ocfg.block_size, seed=6)   # 31 + 28 > 50
    with pytest.raises(ValueError, match="cache full"):
        model.draft_step(noise.cuda(), th.cuda(), cache=cache)
    assert (cache[0].offset, cache[0].keys.shape[2]) == before
    model.close()


def test_cache_layers_trimmed_differently_is_rejected(pkg):
    ocfg = tiny_cfg()
    q8, _ = O.synth_weights(ocfg, seed=7)
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=16)
    cache = model.make_cache(sink_size=4, window_size=16)
    noise, th = O.synth_inputs(ocfg, 1, 10, ocfg.block_size, seed=8)
    model.draft_step(noise.cuda(), th.cuda(), cache=cache)
    cache[0].trim(ocfg.block_size)      # layer 1 left untrimmed
    with pytest.raises(ValueError, match="trim every layer alike"):
        model.draft_step(noise.cuda(), th.cuda(), cache=cache)
    model.close()


def test_ragged_stateless_batch(pkg):
    """Per-sequence context lengths and RoPE offsets in one launch (packed
    context rows), against the oracle run one sequence at a time."""
    ocfg = tiny_cfg()
    B = ocfg.block_size
    q8, dense = O.synth_weights(ocfg, seed=11)
    lens, offs = [5, 0, 37], [0, 3, 100]
    model = gpu_model(pkg, ocfg, q8, max_batch=3, max_ctx=40)
    noises, ths = zip(*[O.synth_inputs(ocfg, 1, c, B, seed=20 + i) for i, c in enumerate(lens)])
    noise = torch.cat(noises)
    packed = torch.cat([t[0] for t in ths])
    hid, toks, _, _ = model.draft_step(noise.cuda(), packed.cuda(), ctx_lens=lens, rope_offsets=offs,
                                       hidden_fp32=True)
    torch.cuda.synchronize()
    for i in range(3):
        ref = O.draft_forward(ocfg, dense, noises[i], ths[i], cache=_oracle_cache(ocfg, 0, 0, offs[i]))
        check_hidden(hid[i:i + 1], ref)
        check_tokens(toks[i:i + 1], O.draft_logits(dense, ref, B), MARGIN)
    model.close()


def test_ragged_cached_batch(pkg):
    """Sequences with different new-context counts per step sharing one cache
    (each its own offset and ring), against one oracle cache per sequence."""
    ocfg = tiny_cfg()
    B = ocfg.block_size
    q8, dense = O.synth_weights(ocfg, seed=12)
    model = gpu_model(pkg, ocfg, q8, max_batch=2, max_ctx=50)
    cache = model.make_cache(sink_size=4, window_size=24)
    oc = [_oracle_cache(ocfg, 4, 24) for _ in range(2)]
    steps = [[50, 9], [2, 7], [8, 1], [3, 3], [0, 5]]
    for t, lens in enumerate(steps):
        ins = [O.synth_inputs(ocfg, 1, c, B, seed=300 + 10 * t + i) for i, c in enumerate(lens)]
        noise = torch.cat([n for n, _ in ins])
        packed = torch.cat([th[0] for _, th in ins])
        hid, toks, _, _ = model.draft_step(noise.cuda(), packed.cuda(), ctx_lens=lens, cache=cache,
                                           hidden_fp32=True)
        torch.cuda.synchronize()
        for i in range(2):
            ref = O.draft_forward(ocfg, dense, ins[i][0], ins[i][1], cache=oc[i])
            check_hidden(hid[i:i + 1], ref)
            check_tokens(toks[i:i + 1], O.draft_logits(dense, ref, B), MARGIN)
            for c in oc[i]:
                c.trim(B)
        for c in cache:
            c.trim(B)
        offs = [cache.store.state(0, s)[0] for s in range(2)]
        assert offs == [oc[0][0].offset, oc[1][0].offset]
    model.close()
