"""The decode loop around the device draft (generate.py:591-789): greedy
speculative output must equal the target's own greedy decode, token for
token, whatever the draft proposes; acceptance lengths stay within the
block."""
import importlib

import pytest
import torch

from oracle import dflash_oracle as O
from helpers import gpu_model, tiny_cfg
from toy_target import ToyTarget

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("sink,window,soft,layered", [(64, 1024, False, False), (4, 16, False, False),
                                                      (64, 1024, True, False), (64, 1024, True, True)])
def test_spec_generate_equals_greedy(pkg, sink, window, soft, layered):
    G = importlib.import_module("mirror-sd_b200.generate")
    ocfg = tiny_cfg(mask_token_id=999)   # the mask id is a token of the target's vocabulary
    target = ToyTarget(ocfg.vocab_size, ocfg.hidden_size, seed=11, layered=layered)
    q8, _ = O.synth_weights(ocfg, seed=12)
    q8["lm_head"] = target.E.float().cpu()           # the draft's lm_head is the target's embedding
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=32)
    prompt = torch.randint(0, ocfg.vocab_size, (20,), generator=torch.Generator().manual_seed(13)).tolist()
    out, stats = G.spec_generate(target, model, prompt, 40, sink_size=sink, window_size=window,
                                 soft_anchor=soft)
    want = target.greedy(prompt, 40)
    assert out == want
    assert stats.total_tokens == 40
    assert all(1 <= a <= ocfg.block_size for a in stats.acceptance_lengths)
    assert stats.draft_steps == len(stats.acceptance_lengths) >= 40 // ocfg.block_size
    model.close()


def test_spec_generate_rejects_mask_outside_vocab(pkg):
    G = importlib.import_module("mirror-sd_b200.generate")
    ocfg = tiny_cfg()                     # default mask id 151669 > vocab 1000
    target = ToyTarget(ocfg.vocab_size, ocfg.hidden_size, seed=31)
    q8, _ = O.synth_weights(ocfg, seed=32)
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=32)
    with pytest.raises(ValueError, match="mask_token_id"):
        G.spec_generate(target, model, [1, 2, 3], 4)
    model.close()


def test_spec_generate_stop_token(pkg):
    G = importlib.import_module("mirror-sd_b200.generate")
    ocfg = tiny_cfg(mask_token_id=999)
    target = ToyTarget(ocfg.vocab_size, ocfg.hidden_size, seed=21)
    q8, _ = O.synth_weights(ocfg, seed=22)
    q8["lm_head"] = target.E.float().cpu()
    model = gpu_model(pkg, ocfg, q8, max_batch=1, max_ctx=32)
    prompt = [5, 6, 7, 8]
    want = target.greedy(prompt, 30)
    stop_tok = want[len(prompt) + 7]                  # the 8th generated token
    out, _ = G.spec_generate(target, model, prompt, 30, stop_token_ids=[stop_tok])
    first = want.index(stop_tok, len(prompt))
    assert out == want[:first + 1]
    model.close()
