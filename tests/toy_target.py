"""A small causal target model for the decode-loop tests.

Each position is computed on its own, in float64, from its token and the
running mean of all earlier embeddings, so its logits are bitwise identical
whether it is fed alone or inside a verify block.  That makes speculative
output comparable with plain greedy decoding token for token."""
import torch


class ToyCache:
    def __init__(self):
        self.sums = []

    def trim(self, n: int):
        if n > 0:
            del self.sums[-n:]


class ToyTarget:
    def __init__(self, vocab: int, hidden: int, n_feat: int = 5, seed: int = 0, device="cuda",
                 layered: bool = False):
        """``layered``: forward returns the features as a list of n_feat
        [1, n, hidden] layers instead of one [1, n, n_feat * hidden] concat."""
        self.layered = layered
        g = torch.Generator().manual_seed(seed)
        self.dev = torch.device(device)
        self.E = (torch.randn(vocab, hidden, generator=g) * 0.02).to(torch.bfloat16).to(self.dev)
        self.E64 = self.E.double()
        s = hidden ** -0.5
        self.W1 = (torch.randn(hidden, hidden, generator=g, dtype=torch.float64) * 30 * s).to(self.dev)
        self.W2 = (torch.randn(hidden, hidden, generator=g, dtype=torch.float64) * 30 * s).to(self.dev)
        self.A = [(torch.randn(hidden, hidden, generator=g, dtype=torch.float64) * s).to(self.dev)
                  for _ in range(n_feat)]

    def make_cache(self):
        return ToyCache()

    def embed(self, ids):
        if int(ids.min()) < 0 or int(ids.max()) >= self.E.shape[0]:  # host-side check
            raise ValueError("token id outside the vocabulary")
        return self.E[ids.to(self.dev)]

    def forward(self, ids, cache):
        logits, feats = [], []
        for tok in ids[0].tolist():
            e = self.E64[tok]
            s = e if not cache.sums else cache.sums[-1] + e
            cache.sums.append(s)
            m = s / len(cache.sums)
            h = torch.tanh(self.W1 @ e + self.W2 @ m)
            logits.append(self.E64 @ h)
            feats.append(torch.cat([torch.tanh(a @ h) for a in self.A]))
        cat = torch.stack(feats)[None].to(torch.bfloat16)
        if self.layered:
            return torch.stack(logits)[None], list(cat.chunk(len(self.A), dim=-1))
        return torch.stack(logits)[None], cat

    def greedy(self, prompt, n_new):
        cache = self.make_cache()
        out = list(prompt)
        logits, _ = self.forward(torch.tensor([out]), cache)
        out.append(int(torch.argmax(logits[0, -1])))
        while len(out) - len(prompt) < n_new:
            logits, _ = self.forward(torch.tensor([[out[-1]]]), cache)
            out.append(int(torch.argmax(logits[0, -1])))
        return out
