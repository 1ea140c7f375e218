"""Loading a HuggingFace-style checkpoint onto the device (loader.py:20-58):
the projections are quantised by the CUDA quantiser bit-exactly as the
reference rule does (ane_model.py:265-279), the loaded model matches the
oracle run on the same stored values, and a saved int8 checkpoint loads back
to identical tensors and identical outputs."""
import importlib

import numpy as np
import pytest
import torch

from oracle import dflash_oracle as O
from helpers import check_hidden, check_tokens, tiny_cfg
from loader_util import PROJ_NAMES, make_checkpoint, oracle_weights

pytestmark = pytest.mark.gpu

MARGIN = 0.05


@pytest.fixture(scope="module")
def L(pkg):
    return importlib.import_module("mirror-sd_b200.loader")


def test_load_quantise_and_forward(L, pkg, tmp_path):
    ocfg = tiny_cfg()
    stored = make_checkpoint(tmp_path, ocfg, seed=3, layout="sharded", prefix="model.")
    lm = (torch.randn(ocfg.vocab_size, ocfg.hidden_size, generator=torch.Generator().manual_seed(4)) * 0.02
          ).to(torch.bfloat16)
    model, cfg = L.load_dflash_model(tmp_path, lm.cuda(), max_batch=2, max_ctx=24)
    # the CUDA quantiser gives the reference's int8 bytes and fp16 scales
    for i, layer in enumerate(model._weights.layers):
        for k, path in PROJ_NAMES.items():
            q, s = O.quantize_q8(stored[f"layers.{i}.{path}.weight"].numpy())
            assert np.array_equal(layer.q[k].cpu().numpy(), q), (i, k)
            assert np.array_equal(layer.s[k].cpu().numpy().view(np.uint16), s.view(np.uint16)), (i, k)
    dense = oracle_weights(ocfg, stored, lm)
    noise, th = O.synth_inputs(ocfg, 2, 24, ocfg.block_size, seed=5)
    hid, toks, _, _ = model.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    torch.cuda.synchronize()
    ref = O.draft_forward(ocfg, dense, noise, th)
    check_hidden(hid, ref)
    check_tokens(toks, O.draft_logits(dense, ref, ocfg.block_size), MARGIN)
    model.close()


def test_q8_checkpoint_round_trip(L, pkg, tmp_path):
    ocfg = tiny_cfg()
    make_checkpoint(tmp_path / "hf", ocfg, seed=6)
    w, cfg = L.load_dflash_weights(tmp_path / "hf")
    L.save_q8_checkpoint(w, cfg, tmp_path / "q8")
    w2, cfg2 = L.load_dflash_weights(tmp_path / "q8")
    assert cfg2 == cfg
    for a, b in zip(w.layers, w2.layers):
        for k in a.q:
            assert torch.equal(a.q[k], b.q[k]) and torch.equal(a.s[k], b.s[k])
        assert torch.equal(a.q_norm, b.q_norm) and torch.equal(a.input_layernorm, b.input_layernorm)
    assert torch.equal(w.fc, w2.fc)
    lm = (torch.randn(ocfg.vocab_size, ocfg.hidden_size, generator=torch.Generator().manual_seed(7)) * 0.02
          ).to(torch.bfloat16).cuda()
    m1 = pkg.DFlashDraftModel(cfg, w, lm, max_batch=1, max_ctx=16)
    m2 = pkg.DFlashDraftModel(cfg2, w2, lm, max_batch=1, max_ctx=16)
    noise, th = O.synth_inputs(ocfg, 1, 16, ocfg.block_size, seed=8)
    h1, t1, _, _ = m1.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    h2, t2, _, _ = m2.draft_step(noise.cuda(), th.cuda(), hidden_fp32=True)
    torch.cuda.synchronize()
    assert torch.equal(h1, h2) and torch.equal(t1, t2)
    m1.close()
    m2.close()
