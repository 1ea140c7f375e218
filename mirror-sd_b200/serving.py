"""Continuous-batching front end of the device draft: one draft KV cache
holding many independent sequences, driven one step at a time.

The reference drafts one request at a time (mirror_sd/generate.py:591-789);
its server runs that loop per request.  Here each step covers any subset of
the cache's sequences (``cache_seqs`` of the C ABI), so a server can prefill
new requests in context-row budgets while the others decode, and every
decode step of all active requests is one device forward.  Per request the
semantics are the reference loop's:
- the block is [anchor, mask x (B-1)] (generate.py:594-597);
- the step appends the request's new context rows (the target features of
  its last accepted tokens, generate.py:773) and its block rows to the cache;
- after drafting, the block rows are trimmed again (generate.py:608-609);
- acceptance is the longest matching prefix against the verifier's ids
  (generate.py:722-728), on the device.

Above 64 block rows per step the forward runs its projections and lm_head as
dense tensor-core GEMMs; below, on the W8A16 kernels.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .dflash import DFlashDraftModel


class DraftServer:
    """Slots 0..max_seqs-1 of one draft cache; a request owns one slot from
    ``prefill`` until ``release``."""

    def __init__(self, model: DFlashDraftModel, max_seqs: Optional[int] = None, sink_size: int = 64,
                 window_size: int = 1024, max_len: Optional[int] = None):
        self.model = model
        self.max_seqs = int(max_seqs or model.max_batch)
        self.cache = model.make_cache(sink_size=sink_size, window_size=window_size, max_len=max_len,
                                      max_batch=self.max_seqs)
        self.block = model.block_size
        self.active = set()

    def _check(self, seqs: Sequence[int]):
        if len(set(seqs)) != len(seqs) or any(not 0 <= s < self.max_seqs for s in seqs):
            raise ValueError(f"sequence slots must be distinct and in [0, {self.max_seqs})")

    def prefill(self, seqs: Sequence[int], noise, target_hidden, ctx_lens: Sequence[int]):
        """First draft step of new requests: their whole prompt features
        (packed rows, or a list of the F selected target layers) enter the
        cache.  Returns the draft ids [len(seqs), B-1]."""
        seqs = [int(s) for s in seqs]
        self._check(seqs)
        if any(s in self.active for s in seqs):
            raise ValueError("prefill of a slot that is still active (release it first)")
        self.cache.reset_seqs(seqs)                       # start from an empty slot
        self.active.update(seqs)
        toks = self.step(seqs, noise, target_hidden, ctx_lens)[0]
        return toks

    def step(self, seqs: Sequence[int], noise, target_hidden, ctx_lens: Sequence[int],
             target_tokens=None, anchor_logits=None, out_tokens=None, acc_len=None, correction=None):
        """One draft step of active requests ``seqs``: new context rows
        ``ctx_lens[i]`` for request i (packed in ``target_hidden``), block
        embeddings ``noise`` [len(seqs), B, H].  With ``target_tokens``
        [len(seqs), B] also the accepted lengths and correction ids.
        The block rows are trimmed from the cache afterwards."""
        seqs = [int(s) for s in seqs]
        self._check(seqs)
        if any(s not in self.active for s in seqs):
            raise ValueError("step of a slot that was not prefilled")
        _, toks, acc, cor = self.model.draft_step(
            noise, target_hidden, ctx_lens=ctx_lens, cache=self.cache, cache_seqs=seqs,
            target_tokens=target_tokens, anchor_logits=anchor_logits, want_hidden=False,
            out_tokens=out_tokens, acc_len=acc_len, correction=correction)
        self.cache.trim_seqs(seqs, [noise.shape[1]] * len(seqs))
        return toks, acc, cor

    def rollback(self, seqs: Sequence[int], counts: Sequence[int]):
        """Drop the last counts[i] cache rows of request seqs[i]."""
        self._check([int(s) for s in seqs])
        self.cache.trim_seqs(seqs, counts)

    def release(self, seqs: Sequence[int]):
        seqs = [int(s) for s in seqs]
        self._check(seqs)
        self.cache.reset_seqs(seqs)
        self.active.difference_update(seqs)

    def state(self, seq: int):
        """(RoPE offset, cached rows) of one slot."""
        return self.cache.store.state(0, int(seq))

    def close(self):
        self.cache.store.close()


def geometric_accepts(n: int, steps: int, p: float, cap: int, seed: int) -> List[List[int]]:
    """Synthetic verifier outcome of the batched serving config: per step and
    request, the accepted draft length, P(accept >= k) = p^k, capped at the
    block's cap drafts."""
    g = torch.Generator().manual_seed(seed)
    u = torch.rand(steps, n, cap, generator=g) < p
    runs = torch.cumprod(u.to(torch.int32), dim=2).sum(dim=2)
    return runs.tolist()


def targets_for(toks: torch.Tensor, accepts: torch.Tensor, vocab: int) -> torch.Tensor:
    """Verifier ids that agree with the drafts for exactly accepts[i] tokens:
    [n, B] with position accepts[i] changed (the bonus position otherwise)."""
    n, nd = toks.shape
    t = torch.cat([toks, torch.zeros(n, 1, dtype=toks.dtype, device=toks.device)], dim=1)
    pos = torch.arange(nd + 1, device=toks.device)[None, :]
    wrong = pos == accepts[:, None]
    return torch.where(wrong & (pos < nd), (t + 1) % vocab, t)
