"""Greedy speculative decoding around the device draft model (the block-draft
loop of mirror_sd/generate.py:591-789).

Per step:
1. build the block [anchor, mask x (B-1)] and embed it with the target's
   embedding (generate.py:594-597);
2. run one cached draft step with lm_head + greedy argmax fused on the device
   (:599-606), then trim the draft cache by B (:608-609);
3. verify [anchor, drafts] with the target (:615-700);
4. accept the longest matching prefix on the device (:722-728);
5. roll the target cache back over the rejected positions (:750-767);
6. the target features of the acc+1 kept positions become the next step's
   context rows (:773).

With greedy sampling the output equals the target's own greedy decode,
whatever the draft proposes; the draft only changes how many target calls
that takes.

The target is any object with
    embed(ids [1, n] int64) -> [1, n, H] bf16 on the draft's device
    forward(ids [1, n], cache) -> (logits [1, n, V], features [1, n, F*H] bf16,
        or the F selected layers as a list of [1, n, H] tensors, which the
        draft's fc GEMM reads in place), appending the n positions to ``cache``
    make_cache() -> an object with trim(n)
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import torch

from .dflash import DFlashDraftModel, accept


@dataclass
class SpecDecodeStats:
    """Counters of one generation (generate.py:239-268)."""
    total_tokens: int = 0
    accepted_tokens: int = 0
    draft_steps: int = 0
    total_time: float = 0.0
    prefill_time: float = 0.0
    acceptance_lengths: List[int] = field(default_factory=list)
    spec_lengths: List[int] = field(default_factory=list)
    total_draft_time: float = 0.0
    total_verify_time: float = 0.0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted_tokens / max(self.draft_steps, 1)

    @property
    def avg_acceptance_length(self) -> float:
        return sum(self.acceptance_lengths) / len(self.acceptance_lengths) if self.acceptance_lengths else 0.0

    @property
    def avg_spec_length(self) -> float:
        return sum(self.spec_lengths) / len(self.spec_lengths) if self.spec_lengths else 0.0


@torch.no_grad()
def spec_generate(target, draft: DFlashDraftModel, input_ids: Sequence[int], max_new_tokens: int,
                  stop_token_ids: Optional[Sequence[int]] = None,
                  sink_size: int = 64, window_size: int = 1024,
                  soft_anchor: bool = False, anchor_top_k: int = 8) -> Tuple[List[int], SpecDecodeStats]:
    """Greedy speculative generation.  Returns (prompt + generated ids, stats).

    ``soft_anchor``: from the second step on, the draft embeds block row 0 as
    the softmax-weighted sum of the top ``anchor_top_k`` tokens under the
    previous verify logits at the correction position (generate.py:1422-1436,
    :1639), on the device.  The verify pass still scores the hard anchor, so
    the output is unchanged; only the drafts (and the acceptance) differ."""
    if not 0 <= draft.mask_token_id < draft.config.vocab_size:
        raise ValueError(f"mask_token_id {draft.mask_token_id} is not a token of the "
                         f"{draft.config.vocab_size}-entry vocabulary")
    stats = SpecDecodeStats()
    dev = draft.device
    stop = set(stop_token_ids or [])
    out = [int(t) for t in input_ids]
    n_prompt = len(out)
    t0 = time.perf_counter()

    # prefill: the prompt's logits give the first token, its features the first context
    tcache = target.make_cache()
    logits, feats = target.forward(torch.tensor([out], device=dev), tcache)
    out.append(int(torch.argmax(logits[0, -1]).item()))
    target_hidden = feats
    stats.prefill_time = time.perf_counter() - t0

    dcache = draft.make_cache(sink_size=sink_size, window_size=window_size)
    B = draft.block_size
    prev_logits = None                    # [1, V] verify logits at the last correction position
    while len(out) - n_prompt < max_new_tokens and out[-1] not in stop:
        t1 = time.perf_counter()
        anchor = out[-1]
        block = torch.tensor([[anchor] + [draft.mask_token_id] * (B - 1)], device=dev)
        noise = target.embed(block)
        drafts = draft.draft_tokens(noise, target_hidden, cache=dcache,   # [1, B-1] int32
                                    anchor_logits=prev_logits, anchor_top_k=anchor_top_k)
        for c in dcache:
            c.trim(B)
        t2 = time.perf_counter()
        verify_ids = torch.cat([torch.tensor([[anchor]], device=dev, dtype=torch.int64),
                                drafts.to(torch.int64)], dim=1)
        logits, feats = target.forward(verify_ids, tcache)
        posterior = torch.argmax(logits, dim=-1).to(torch.int32)         # [1, B]
        acc, corr = accept(drafts, posterior)
        a = int(acc[0].item())                                            # one host sync per step
        new = drafts[0, :a].tolist() + [int(corr[0].item())]
        tcache.trim(B - (a + 1))                                          # rejected positions
        target_hidden = ([f[:, :a + 1, :] for f in feats] if isinstance(feats, (list, tuple))
                         else feats[:, :a + 1, :])
        if soft_anchor:
            prev_logits = logits[:, a, :]
        stats.total_verify_time += time.perf_counter() - t2
        stats.total_draft_time += t2 - t1
        for tok in new:
            if len(out) - n_prompt >= max_new_tokens:
                break
            out.append(int(tok))
            if tok in stop:
                break
        stats.acceptance_lengths.append(a + 1)
        stats.spec_lengths.append(B - 1)
        stats.accepted_tokens += a
        stats.draft_steps += 1
    stats.total_tokens = len(out) - n_prompt
    stats.total_time = time.perf_counter() - t0
    return out, stats
