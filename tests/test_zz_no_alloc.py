"""dflash_attention_noalloc: attention whose scratch is a static device array.

It is for callers that cannot allocate device memory.  Its output must match
dflash_attention, the entry point with a caller workspace, on consecutive calls
of different shapes.  The shared array keeps the previous call's contents, so
these checks also cover stale scratch.  This file is collected last, so it runs
both after the other tests and, run by itself, in a fresh process.
"""
import ctypes

import pytest
import torch


def _noalloc(pkg, q, k, v, normrope=False, q_norm=None, k_norm=None, rope_theta=1e6,
             q_pos0=0, k_pos0=0, eps=1e-6):
    N = pkg._native
    lib = N.load()
    b, nq, blk, _ = q.shape
    nkv, L = k.shape[1], k.shape[2]
    out = torch.empty((b, blk, nq * 128), dtype=torch.float16, device=q.device)
    st = torch.cuda.current_stream(q.device).cuda_stream
    N.check(lib.dflash_attention_noalloc(N.ptr(q), N.ptr(k), N.ptr(v), b, nq, nkv, blk, L,
                                         int(normrope), N.ptr(q_norm), N.ptr(k_norm),
                                         float(rope_theta), int(q_pos0), int(k_pos0), float(eps),
                                         N.ptr(out), st), "dflash_attention_noalloc")
    return out


def _inputs(seed, b, nq, nkv, B, L):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, nq, B, 128, generator=g).to(torch.float16).cuda()
    k = torch.randn(b, nkv, L, 128, generator=g).to(torch.float16).cuda()
    v = torch.randn(b, nkv, L, 128, generator=g).to(torch.float16).cuda()
    qn = (1 + 0.1 * torch.randn(128, generator=g)).cuda()
    kn = (1 + 0.1 * torch.randn(128, generator=g)).cuda()
    return q, k, v, qn, kn


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_on_consecutive_calls(pkg):
    import importlib
    K = importlib.import_module("mirror-sd_b200.kernels")
    # call 1: 32 query / 8 kv heads, block 32, ctx 4096, raw Q/K with
    # the fused per-head RMSNorm + RoPE; call 2: a smaller ragged shape, plain Q/K
    q1, k1, v1, qn1, kn1 = _inputs(1, 1, 32, 8, 32, 4096 + 32)
    q2, k2, v2, _, _ = _inputs(2, 2, 8, 2, 16, 300)
    out1 = _noalloc(pkg, q1, k1, v1, normrope=True, q_norm=qn1, k_norm=kn1, q_pos0=4096, k_pos0=0)
    out2 = _noalloc(pkg, q2, k2, v2)
    ref1 = K.attention(q1, k1, v1, normrope=True, q_norm=qn1, k_norm=kn1, rope_theta=1e6,
                       q_pos0=4096, k_pos0=0)
    ref2 = K.attention(q2, k2, v2)
    torch.cuda.synchronize()
    for out, ref in ((out1, ref1), (out2, ref2)):
        assert torch.isfinite(out.float()).all()
        err = (out.float() - ref.float()).abs().max().item()
        assert err < 2e-2, err
    # both calls also against an fp32 restatement on the CPU (per-head RMSNorm
    # and neox RoPE for the first, GQA attention for both), so a fault shared
    # by the two entry points' kernels cannot pass unseen
    from oracle import dflash_oracle as O
    qr = O.rope_neox(O.rms_norm(q1.float().cpu(), qn1.cpu(), 1e-6), torch.arange(32) + 4096, 1e6)
    kr = O.rope_neox(O.rms_norm(k1.float().cpu(), kn1.cpu(), 1e-6), torch.arange(4096 + 32), 1e6)
    want1 = _attn_fp32(qr, kr, v1.float().cpu())
    want2 = _attn_fp32(q2.float().cpu(), k2.float().cpu(), v2.float().cpu())
    for out, want in ((out1, want1), (out2, want2)):
        err = (out.float().cpu() - want).abs().max().item()
        assert err < 2e-2, err


def _attn_fp32(q, k, v):
    """fp32 non-causal GQA attention: q [b, NQ, B, 128], k/v [b, NKV, L, 128]
    -> [b, B, NQ*128] (the reference's mx.repeat + SDPA, dflash.py:310-317)."""
    G = q.shape[1] // k.shape[1]
    kk = torch.repeat_interleave(k, G, dim=1)
    vv = torch.repeat_interleave(v, G, dim=1)
    p = torch.softmax(torch.matmul(q, kk.transpose(-1, -2)) * 128 ** -0.5, dim=-1)
    o = torch.matmul(p, vv)
    b, nq, B, D = q.shape
    return o.transpose(1, 2).reshape(b, B, nq * D)


def test_noalloc_rejects_shapes_beyond_the_static_array(pkg):
    """Size validation runs on the host before any CUDA work (no GPU needed)."""
    lib = pkg._native.load()
    fake = ctypes.c_void_p(256)  # never dereferenced: the call fails before any launch
    st = lib.dflash_attention_noalloc(fake, fake, fake, 8, 32, 8, 24, 65536, 0, None, None,
                                      1e6, 0, 0, 1e-6, fake, None)
    assert st == pkg._native.DFLASH_ERR_INVALID
    assert "static array" in pkg._native.last_error()
