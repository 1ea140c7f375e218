"""Host logic of the batched serving front end (no GPU): the synthetic
verifier's geometric acceptance and the verifier ids it implies, checked
with the oracle's longest-prefix acceptance (generate.py:722-728)."""
import importlib

import torch

from oracle import dflash_oracle as O


def _serving():
    return importlib.import_module("mirror-sd_b200.serving")


def test_geometric_accepts_distribution():
    S = _serving()
    a = torch.tensor(S.geometric_accepts(4000, 3, 0.85, 15, seed=1))
    assert a.min() >= 0 and a.max() <= 15
    # P(accept >= k) = 0.85^k, capped at 15
    for k in (1, 3, 6):
        frac = (a >= k).float().mean().item()
        assert abs(frac - 0.85 ** k) < 0.02, (k, frac)
    assert S.geometric_accepts(5, 2, 0.85, 15, seed=3) == S.geometric_accepts(5, 2, 0.85, 15, seed=3)


def test_targets_for_gives_the_planned_acceptance():
    S = _serving()
    g = torch.Generator().manual_seed(2)
    toks = torch.randint(0, 1000, (64, 15), generator=g, dtype=torch.int32)
    acc = torch.tensor(S.geometric_accepts(64, 1, 0.85, 15, seed=4)[0], dtype=torch.int32)
    tgt = S.targets_for(toks, acc, 1000)
    assert tgt.shape == (64, 16)
    for d, t, a in zip(toks.tolist(), tgt.tolist(), acc.tolist()):
        got, cor = O.accept(d, t)
        assert got == a and cor == t[a]
