"""Kernel-level parity on the GPU, each through its C-ABI entry point.

References: the CPU oracle (oracle/dflash_oracle.py) for the quantiser, the
QK-norm/RoPE/attention composition and argmax/acceptance; a plain fp32
product of the same (exactly representable) operands for the GEMMs.
"""
import os

import numpy as np
import pytest
import torch

from oracle import dflash_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K(pkg):
    import importlib
    return importlib.import_module("mirror-sd_b200.kernels")


def test_quantizer_bit_exact_vs_reference(pkg, golden_dir):
    z = np.load(os.path.join(golden_dir, "quantizer_q8.npz"))
    q, s = pkg.quantize_q8(torch.from_numpy(z["w"]).cuda())
    assert np.array_equal(q.cpu().numpy(), z["q"])
    assert np.array_equal(s.cpu().numpy().view(np.uint16), z["s"].view(np.uint16))


def test_quantizer_bit_exact_random(pkg):
    g = torch.Generator().manual_seed(3)
    w = torch.randn(333, 1000, generator=g) * 0.02
    w[7] = 0
    w[9, :5] = torch.tensor([0.5, -0.5, 1.5, -2.5, 127.0]) * (1.0 / 127.0)
    q, s = pkg.quantize_q8(w.cuda())
    qr, sr = O.quantize_q8(w.numpy())
    assert np.array_equal(q.cpu().numpy(), qr)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), sr.view(np.uint16))


@pytest.mark.parametrize("M,N,Kd", [(1, 256, 128), (8, 384, 640), (16, 1024, 4096), (32, 768, 5120),
                                    (31, 256, 17408), (64, 512, 1024),
                                    # at least one tile per SM on a poorly filled last
                                    # round: stream-K with short K (8B and 4B gate|up)
                                    (16, 24576, 4096), (32, 19456, 2560)])
def test_w8_linear_vs_fp32(K, M, N, Kd):
    g = torch.Generator().manual_seed(M * 7 + N)
    w = torch.randn(N, Kd, generator=g) * 0.02
    q, s = O.quantize_q8(w.numpy())
    x = (torch.randn(M, Kd, generator=g)).to(torch.float16)
    y = K.w8_linear(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), x.cuda()).float().cpu()
    ref = x.float() @ torch.from_numpy(O.dequantize_q8(q, s)).T
    err = (y - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2e-3 * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("M,N,Kd,bf16", [(128, 256, 64, True), (200, 512, 1024, True),
                                         (64, 256, 256, False), (300, 768, 512, False),
                                         (1000, 256, 25600, True),
                                         # more tiles than SMs: the partial last round is split
                                         # along K (12 tiles x 8 parts; 4 tiles x 16 parts)
                                         (1280, 4096, 2048, True), (1000, 4864, 4096, False),
                                         # 96 tiles (fewer than SMs) in 3 K-parts: two parts per CTA
                                         (384, 8192, 2048, True)])
def test_tc_gemm_vs_fp32(K, M, N, Kd, bf16):
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(M + N + Kd)
    a = torch.randn(M, Kd, generator=g).to(dt)
    b = torch.randint(-127, 128, (N, Kd), generator=g).to(dt) if not bf16 else \
        (torch.randn(N, Kd, generator=g) * 0.05).to(dt)
    d = K.tc_gemm(a.cuda(), b.cuda()).cpu()
    ref = a.double() @ b.double().T
    err = (d.double() - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item() + 1e-3, err


def _attn_ref(q, k, v, G):
    # q [b, NQ, B, D], k/v [b, NKV, L, D] -> [b, B, NQ*D]
    kk = torch.repeat_interleave(k, G, dim=1)
    vv = torch.repeat_interleave(v, G, dim=1)
    o = O.sdpa(q, kk, vv, 128 ** -0.5)
    b, nq, B, D = q.shape
    return o.transpose(1, 2).reshape(b, B, nq * D)


@pytest.mark.parametrize("b,nq,nkv,B,L", [(1, 40, 8, 32, 96), (1, 32, 8, 16, 2064), (2, 4, 2, 8, 20),
                                          (1, 40, 8, 32, 4128), (3, 8, 1, 16, 700),
                                          # many (sequence, head) CTAs: two per SM, column halves
                                          (80, 32, 8, 16, 300), (40, 16, 8, 8, 1111),
                                          # 64 < query rows <= 128 with many CTAs
                                          (60, 40, 8, 16, 257)])
def test_attention_vs_fp32(K, b, nq, nkv, B, L):
    g = torch.Generator().manual_seed(b * 1000 + L)
    q = torch.randn(b, nq, B, 128, generator=g).to(torch.float16)
    k = torch.randn(b, nkv, L, 128, generator=g).to(torch.float16)
    v = torch.randn(b, nkv, L, 128, generator=g).to(torch.float16)
    # q, k already "normed" (unit rms) as in the draft forward
    out = K.attention(q.cuda(), k.cuda(), v.cuda()).float().cpu()
    ref = _attn_ref(q.float(), k.float(), v.float(), nq // nkv)
    err = (out - ref).abs().max().item()
    assert err < 1e-2, err


@pytest.mark.parametrize("b,nq,nkv,B,C", [(1, 40, 8, 32, 64), (2, 32, 8, 16, 300)])
def test_attention_fused_qknorm_rope(K, b, nq, nkv, B, C):
    """Raw Q/K: RMSNorm per head + neox RoPE (q at C+j, k at i) + attention,
    against the oracle's composition (dflash.py:291-317)."""
    g = torch.Generator().manual_seed(C)
    L = C + B
    q = torch.randn(b, nq, B, 128, generator=g).to(torch.float16)
    k = torch.randn(b, nkv, L, 128, generator=g).to(torch.float16)
    v = torch.randn(b, nkv, L, 128, generator=g).to(torch.float16)
    qn = 1 + 0.1 * torch.randn(128, generator=g)
    kn = 1 + 0.1 * torch.randn(128, generator=g)
    out = K.attention(q.cuda(), k.cuda(), v.cuda(), normrope=True, q_norm=qn.cuda(), k_norm=kn.cuda(),
                      rope_theta=1e6, q_pos0=C, k_pos0=0).float().cpu()
    qr = O.rope_neox(O.rms_norm(q.float(), qn, 1e-6), torch.arange(B) + C, 1e6)
    kr = O.rope_neox(O.rms_norm(k.float(), kn, 1e-6), torch.arange(L), 1e6)
    ref = _attn_ref(qr, kr, v.float(), nq // nkv)
    err = (out - ref).abs().max().item()
    assert err < 2e-2, err


@pytest.mark.parametrize("b,B,H,V", [(1, 32, 5120, 151936), (2, 16, 256, 1000), (1, 8, 4096, 33)])
def test_lm_head_argmax_bit_exact(K, b, B, H, V):
    """Given the same bf16 hidden rows, the fused lm_head argmax equals the
    fp64 argmax of the same products wherever the top-2 margin exceeds 1e-4."""
    g = torch.Generator().manual_seed(V)
    hn = torch.randn(b, B, H, generator=g).to(torch.bfloat16)
    E = (torch.randn(V, H, generator=g) * 0.02).to(torch.bfloat16)
    if V > 100:
        E[100] = E[57]          # exact duplicate row -> exact tie, first index must win
    toks = K.lm_head_argmax(hn.cuda(), E.cuda()).cpu()
    logits = hn[:, 1:].double() @ E.double().T
    ref = torch.argmax(logits, dim=-1)
    top = torch.topk(logits, 2, dim=-1).values
    clear = (top[..., 0] - top[..., 1]) > 1e-4
    assert torch.equal(toks[clear].long(), ref[clear]), "argmax mismatch on a clear maximum"


def test_lm_head_tie_first_index(K):
    H, V = 256, 300
    E = torch.zeros(V, H, dtype=torch.bfloat16)
    E[:, 0] = 1.0
    hn = torch.zeros(1, 4, H, dtype=torch.bfloat16)
    hn[0, :, 0] = 1.0
    E[250, 0] = 2.0
    E[260, 0] = 2.0           # tie between 250 and 260 -> 250
    toks = K.lm_head_argmax(hn.cuda(), E.cuda()).cpu()
    assert toks.tolist() == [[250, 250, 250]]


def test_accept_device(pkg):
    draft = torch.tensor([[5, 6, 7], [5, 6, 7], [1, 2, 3], [9, 9, 9]], dtype=torch.int32)
    target = torch.tensor([[5, 6, 7, 8], [5, 9, 7, 8], [4, 2, 3, 0], [9, 9, 9, 1]], dtype=torch.int32)
    acc, cor = pkg.accept(draft.cuda(), target.cuda())
    want = [O.accept(d.tolist(), t.tolist()) for d, t in zip(draft, target)]
    assert acc.cpu().tolist() == [w[0] for w in want]
    assert cor.cpu().tolist() == [w[1] for w in want]


def test_lm_head_accept_fused(K):
    g = torch.Generator().manual_seed(11)
    b, B, H, V = 3, 8, 256, 500
    hn = torch.randn(b, B, H, generator=g).to(torch.bfloat16)
    E = (torch.randn(V, H, generator=g) * 0.02).to(torch.bfloat16)
    toks = K.lm_head_argmax(hn.cuda(), E.cuda()).cpu()
    target = torch.cat([toks, torch.zeros(b, 1, dtype=torch.int32)], dim=1)
    target[1, 3] = (target[1, 3] + 1) % V
    target[2, 0] = (target[2, 0] + 1) % V
    t2, acc, cor = K.lm_head_argmax(hn.cuda(), E.cuda(), target=target.cuda())
    want = [O.accept(d.tolist(), t.tolist()) for d, t in zip(toks, target)]
    assert acc.cpu().tolist() == [w[0] for w in want] == [B - 1, 3, 0]
    assert cor.cpu().tolist() == [w[1] for w in want]


def _bf16_ulps(got_bf16, want_f32):
    """max |got - bf16(want)| in units of the bf16 spacing at bf16(want)."""
    w = torch.as_tensor(want_f32, dtype=torch.float32)
    wb = w.to(torch.bfloat16).float()
    g = got_bf16.float().cpu()
    _, e = torch.frexp(torch.where(wb == 0, torch.full_like(wb, 2.0 ** -126), wb))
    spacing = torch.ldexp(torch.ones_like(wb), (e - 8).to(torch.int32))
    return (torch.abs(g - wb) / spacing).max().item()


def test_soft_anchor_vs_reference_fixture(K, golden_dir):
    """The device soft anchor against the reference's ``_make_soft_anchor``:
    within one bf16 rounding step of the reference's fp32 sum (the device
    sums in the same order; expf may differ from numpy's exp by an ulp)."""
    z = np.load(os.path.join(golden_dir, "soft_anchor.npz"))
    for c in "abcd":
        E = torch.from_numpy(z[f"{c}.E"].astype(np.int16)).view(torch.bfloat16)
        logits = torch.from_numpy(z[f"{c}.logits"])
        if int(z[f"{c}.bf16_logits"]):
            logits = logits.to(torch.bfloat16)          # exact: the values are bf16
        out = K.soft_anchor(logits.cuda(), E.cuda(), int(z[f"{c}.k"]))
        assert _bf16_ulps(out, z[f"{c}.anchor"]) <= 1.0, c


@pytest.mark.parametrize("rows,V,H,k,bf16", [(1, 151936, 5120, 8, False), (4, 151936, 4096, 8, True),
                                             (3, 32000, 256, 16, False), (2, 5, 64, 1, False),
                                             (32, 151936, 1024, 8, False)])
def test_soft_anchor_vs_oracle(K, rows, V, H, k, bf16):
    g = torch.Generator().manual_seed(V + rows)
    E = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16)
    logits = torch.randn(rows, V, generator=g) * 4.0
    if bf16:
        logits = logits.to(torch.bfloat16)
    if V > 17:   # a duplicated top value: the lower index must come first
        logits[0, 17] = logits[0, 9] = logits[0].max() + 1
    out = K.soft_anchor(logits.cuda(), E.cuda(), k).cpu()
    Ef = E.float().numpy()
    for r in range(rows):
        ids, w, anchor = O.soft_anchor(logits[r].float().numpy(), Ef, k)
        if r == 0 and V > 17 and k > 1:
            assert list(ids[:2]) == [9, 17]
        assert _bf16_ulps(out[r], anchor) <= 1.0, r


def test_soft_anchor_strided_rows(K):
    """Rows of a [b, B, V] verify output at the correction position, passed
    as a strided view (ld = B * V)."""
    g = torch.Generator().manual_seed(5)
    V, H, B = 3000, 128, 4
    E = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16)
    full = torch.randn(2, B, V, generator=g)
    view = full.cuda()[:, 2, :]
    out = K.soft_anchor(view, E.cuda(), 8).cpu()
    for r in range(2):
        _, _, anchor = O.soft_anchor(full[r, 2].numpy(), E.float().numpy(), 8)
        assert _bf16_ulps(out[r], anchor) <= 1.0
