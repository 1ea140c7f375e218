"""Run one hot-path kernel of the draft step on a named case, for timing and
for ncu captures that stay small (each case holds < 2 GB on the device and
streams more than the 126 MB L2 per launch).

    python mirror-sd_b200/profile_kernels.py <case> [--iters N] [--warmup W]

Cases (27B-class draft dims, 32 block rows):
  w8_gu    gate|up W8A16 projection   N=34816 K=5120   (178 MB int8)
  w8_down  down W8A16 projection      N=5120  K=17408  (89 MB)
  w8_qkv   fused q|k|v projection     N=7168  K=5120   (37 MB)
  w8_o     o projection               N=5120  K=5120   (21 MB)
  w8:N:K   any W8A16 shape (N, K multiples of 128)
  lm_head  tied lm_head + argmax      V=151936 H=5120  (1.56 GB bf16)
  attn     block attention            40/8 heads, 32 queries, kv 4128
  attn16   the same at batch 16, kv 32800 (2.1 GB of K/V)
  attn_c5  the batched serving shape: 256 sequences, 32 q / 8 kv heads, 16
           queries, kv 1104 (a sink 64 / window 1024 cache plus the block)
  fc       context fc GEMM            4096 x 25600 x 5120 (bf16)
  attn_sweep  block attention, 40/8 heads, 32 queries, ctx 1K..32K, batch 1 and 16
              (prints a markdown table: time, bandwidth, fraction of measured HBM)
  step1    one draft step at the bench's 27B dims (block 32, ctx 4096, batch 1) with
           one decoder layer, so the fc and context K|V GEMMs run exactly as in
           the bench with about 4 GB on the device
  serve    one stateless draft step of --seqs sequences (default 64) of block 16,
           ctx 64 each, 8B-class dims: the dense block path (tcgen05 projections
           and lm_head over f16 weight copies); about 6 GB on the device
Prints the mean launch time measured with CUDA events and the achieved
bandwidth (or TFLOP/s for fc).
"""
import argparse
import importlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def attn_sweep(K, dev, iters):
    """c4: block attention (40 query / 8 kv heads, 32 queries, head 128) over
    ctx 1K..32K at batch 1 and 16; algorithmic bytes = Q + O + K + V (f16)."""
    peaks = os.path.join(os.path.dirname(HERE), "MEASURED_PEAKS.json")
    hbm = 6650.0
    if os.path.exists(peaks):
        import json
        with open(peaks) as f:
            hbm = float(json.load(f).get("hbm_gbs", hbm))
    print("| batch | ctx | kv rows | MB | us | GB/s | of HBM | TFLOP/s |")
    print("|---|---|---|---|---|---|---|---|")
    g = torch.Generator(device=dev).manual_seed(0)
    ws = None
    for b in (1, 16):
        for C in (1024, 4096, 8192, 16384, 32768):
            L = C + 32
            q = torch.randn(b, 40, 32, 128, generator=g, device=dev).to(torch.float16)
            k = torch.randn(b, 8, L, 128, generator=g, device=dev).to(torch.float16)
            v = torch.randn(b, 8, L, 128, generator=g, device=dev).to(torch.float16)
            need = K.N.load().dflash_attention_workspace_size(b, 40, 8, 32, L)
            if ws is None or ws.numel() < need:
                ws = torch.empty(need, dtype=torch.uint8, device=dev)
            for _ in range(3):
                K.attention(q, k, v, workspace=ws)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                K.attention(q, k, v, workspace=ws)
            e1.record()
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) / iters * 1e3
            nbytes = 2 * b * 40 * 32 * 128 * 2 + 2 * b * 8 * L * 128 * 2
            flops = 4.0 * b * 40 * 32 * L * 128
            print(f"| {b} | {C} | {L} | {nbytes / 1e6:.1f} | {us:.1f} | {nbytes / us / 1e3:.0f} | "
                  f"{nbytes / us / 1e3 / hbm:.2f} | {flops / us / 1e6:.0f} |")
            del q, k, v


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--seqs", type=int, default=64)
    a = ap.parse_args()
    importlib.import_module("mirror-sd_b200")
    K = importlib.import_module("mirror-sd_b200.kernels")
    dev = torch.device("cuda", 0)
    if a.case == "attn_sweep":
        K.N = importlib.import_module("mirror-sd_b200._native")
        attn_sweep(K, dev, a.iters)
        return
    g = torch.Generator(device=dev).manual_seed(0)
    M = 32
    if a.case.startswith("w8_") or a.case.startswith("w8:"):
        if a.case.startswith("w8:"):  # w8:N:K
            N, Kd = (int(v) for v in a.case.split(":")[1:3])
        else:
            N, Kd = {"w8_gu": (34816, 5120), "w8_down": (5120, 17408), "w8_qkv": (7168, 5120),
                     "w8_o": (5120, 5120)}[a.case]
        q = torch.randint(-127, 128, (N, Kd), generator=g, device=dev, dtype=torch.int8)
        s = (torch.rand(N, generator=g, device=dev) * 1e-3).to(torch.float16)
        x = torch.randn(M, Kd, generator=g, device=dev).to(torch.float16)
        fn = lambda: K.w8_linear(q, s, x)
        nbytes, flops = N * Kd, 2 * M * N * Kd
    elif a.case == "lm_head":
        V, H = 151936, 5120
        E = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        hn = torch.randn(1, M, H, generator=g, device=dev).to(torch.bfloat16)
        ws = torch.empty(1 << 20, dtype=torch.uint8, device=dev)
        fn = lambda: K.lm_head_argmax(hn, E, workspace=ws)
        nbytes, flops = V * H * 2, 2 * (M - 1) * V * H
    elif a.case in ("attn", "attn16", "attn_c5"):
        bsz, L, nq, Mq = {"attn": (1, 4128, 40, M), "attn16": (16, 32800, 40, M),
                          "attn_c5": (256, 1104, 32, 16)}[a.case]
        qq = torch.randn(bsz, nq, Mq, 128, generator=g, device=dev).to(torch.float16)
        kk = torch.randn(bsz, 8, L, 128, generator=g, device=dev).to(torch.float16)
        vv = torch.randn(bsz, 8, L, 128, generator=g, device=dev).to(torch.float16)
        ws = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        fn = lambda: K.attention(qq, kk, vv, workspace=ws)
        nbytes, flops = bsz * 2 * 8 * L * 128 * 2, bsz * 4 * nq * Mq * L * 128
    elif a.case == "step1":
        pkg = importlib.import_module("mirror-sd_b200")
        cfg = pkg.DFlashConfig(hidden_size=5120, num_hidden_layers=1, intermediate_size=17408,
                               num_attention_heads=40, num_key_value_heads=8, head_dim=128,
                               vocab_size=151936, block_size=32)
        cfg.target_layer_ids = list(range(5))
        w, lm = pkg.synth_weights_q8(cfg, seed=0, device=dev)
        C, B, H = 4096, 32, 5120
        model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=1, max_ctx=C, max_block=B, device=dev)
        noise = (torch.randn(1, B, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        th = torch.randn(1, C, 5 * H, generator=g, device=dev).to(torch.bfloat16)
        toks = torch.empty((1, B - 1), dtype=torch.int32, device=dev)
        fn = lambda: model.draft_step(noise, th, want_hidden=False, out_tokens=toks)
        nbytes = C * 5 * H * 2 + H * 5 * H * 2
        flops = 2 * C * 5 * H * H + 2 * C * H * 2 * 8 * 128
    elif a.case == "serve":
        pkg = importlib.import_module("mirror-sd_b200")
        cfg = pkg.DFlashConfig(hidden_size=4096, num_hidden_layers=5, intermediate_size=12288,
                               num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                               vocab_size=151936, block_size=16)
        cfg.target_layer_ids = list(range(5))
        w, lm = pkg.synth_weights_q8(cfg, seed=0, device=dev)
        n, C, B, H = a.seqs, 64, 16, 4096
        model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=n, max_ctx=C, max_block=B, device=dev)
        noise = (torch.randn(n, B, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        th = torch.randn(n, C, 5 * H, generator=g, device=dev).to(torch.bfloat16)
        toks = torch.empty((n, B - 1), dtype=torch.int32, device=dev)
        fn = lambda: model.draft_step(noise, th, want_hidden=False, out_tokens=toks)
        Mb = n * B
        params = 5 * ((32 + 16) * 128 * H + H * 32 * 128 + 3 * 12288 * H)
        nbytes = params * 2 + 151936 * H * 2
        flops = 2 * Mb * (params + 151936 * H) + 2 * n * C * (5 * H * H + H * 5 * 2 * 8 * 128)
    elif a.case == "fc":
        Mr, Kd, N = 4096, 25600, 5120
        A = torch.randn(Mr, Kd, generator=g, device=dev).to(torch.bfloat16)
        B = (torch.randn(N, Kd, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        fn = lambda: K.tc_gemm(A, B)
        nbytes, flops = (Mr + N) * Kd * 2, 2 * Mr * N * Kd
    else:
        raise SystemExit(f"unknown case {a.case}")
    for _ in range(a.warmup):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / a.iters
    print(f"{a.case}: {ms * 1e3:.1f} us/call  {nbytes / ms / 1e6:.0f} GB/s  {flops / ms / 1e9:.1f} TFLOP/s")


if __name__ == "__main__":
    main()
