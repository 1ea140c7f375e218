"""Thin torch wrappers over the kernel-level C entry points (one hot-path
kernel each), used by the parity tests and the attention-only benchmark."""
import ctypes

import torch

from . import _native as N


def _st(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def w8_linear(q: torch.Tensor, s: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """y = x . (q * s)^T with the W8A16 skinny kernel; x [M, K] f16 (M <= 64)."""
    lib = N.load()
    Nn, K = q.shape
    x = x.to(torch.float16).contiguous()
    M = x.shape[0]
    y = torch.empty((M, Nn), dtype=torch.float16, device=x.device)
    N.check(lib.dflash_w8_linear(N.ptr(q.contiguous()), N.ptr(s.to(torch.float16).contiguous()), Nn, K,
                                 N.ptr(x), M, N.ptr(y), _st(x.device)), "dflash_w8_linear")
    return y


def tc_gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """D = a . b^T (fp32) on the tcgen05 kernel; a [M, K], b [N, K] both bf16 or both f16."""
    lib = N.load()
    if a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("a and b must both be bf16 or both f16")
    a, b = a.contiguous(), b.contiguous()
    M, K = a.shape
    Nn = b.shape[0]
    d = torch.empty((M, Nn), dtype=torch.float32, device=a.device)
    N.check(lib.dflash_tc_gemm(N.ptr(a), N.ptr(b), M, Nn, K, int(a.dtype == torch.bfloat16),
                               N.ptr(d), _st(a.device)), "dflash_tc_gemm")
    return d


def attention(q, k, v, normrope=False, q_norm=None, k_norm=None, rope_theta=1e6,
              q_pos0=0, k_pos0=0, eps=1e-6, workspace=None):
    """Non-causal GQA attention (optionally with fused QK RMSNorm + RoPE).
    q [b, NQ, B, 128], k/v [b, NKV, L, 128] f16 -> out [b, B, NQ*128] f16."""
    lib = N.load()
    b, nq, blk, _ = q.shape
    nkv, L = k.shape[1], k.shape[2]
    q, k, v = (t.to(torch.float16).contiguous() for t in (q, k, v))
    out = torch.empty((b, blk, nq * 128), dtype=torch.float16, device=q.device)
    need = lib.dflash_attention_workspace_size(b, nq, nkv, blk, L)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty((need,), dtype=torch.uint8, device=q.device)
    qn = q_norm.to(torch.float32).contiguous() if q_norm is not None else None
    kn = k_norm.to(torch.float32).contiguous() if k_norm is not None else None
    N.check(lib.dflash_attention(N.ptr(q), N.ptr(k), N.ptr(v), b, nq, nkv, blk, L, int(normrope),
                                 N.ptr(qn), N.ptr(kn), float(rope_theta), int(q_pos0), int(k_pos0),
                                 float(eps), N.ptr(out), N.ptr(workspace), workspace.numel(),
                                 _st(q.device)), "dflash_attention")
    return out


def lm_head_argmax(hn, E, target=None, workspace=None):
    """Greedy ids for rows 1..B-1 of hn [b, B, H] (bf16) against E [V, H] (bf16);
    with target [b, B] also (acc_len, correction)."""
    lib = N.load()
    b, blk, H = hn.shape
    V = E.shape[0]
    hn, E = hn.to(torch.bfloat16).contiguous(), E.to(torch.bfloat16).contiguous()
    toks = torch.empty((b, blk - 1), dtype=torch.int32, device=hn.device)
    need = lib.dflash_lm_head_workspace_size(b, blk, V, H)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty((need,), dtype=torch.uint8, device=hn.device)
    acc = cor = tt = None
    if target is not None:
        tt = target.to(torch.int32).contiguous()
        acc = torch.empty((b,), dtype=torch.int32, device=hn.device)
        cor = torch.empty((b,), dtype=torch.int32, device=hn.device)
    N.check(lib.dflash_lm_head_argmax(N.ptr(hn), N.ptr(E), b, blk, H, V, N.ptr(toks), N.ptr(tt),
                                      N.ptr(acc), N.ptr(cor), N.ptr(workspace), workspace.numel(),
                                      _st(hn.device)), "dflash_lm_head_argmax")
    return toks if target is None else (toks, acc, cor)


def soft_anchor(logits, E, top_k=8, workspace=None):
    """Soft anchor rows (generate.py:1422-1436): logits [b, V] (fp32 or bf16,
    rows may be strided) and E [V, H] bf16 -> [b, H] bf16, the softmax-weighted
    sum of the top_k rows of E under each row of logits."""
    lib = N.load()
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    if logits.dtype not in (torch.float32, torch.bfloat16):
        logits = logits.to(torch.float32)
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    b, V = logits.shape
    E = E.to(torch.bfloat16).contiguous()
    if E.shape[0] != V:
        raise ValueError(f"E has {E.shape[0]} rows, logits {V} columns")
    H = E.shape[1]
    out = torch.empty((b, H), dtype=torch.bfloat16, device=logits.device)
    need = lib.dflash_soft_anchor_workspace_size(b)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty((need,), dtype=torch.uint8, device=logits.device)
    N.check(lib.dflash_soft_anchor(N.ptr(logits), int(logits.dtype == torch.bfloat16), b, V,
                                   logits.stride(0), int(top_k), N.ptr(E), H, N.ptr(out),
                                   N.ptr(workspace), workspace.numel(), _st(logits.device)),
            "dflash_soft_anchor")
    return out
