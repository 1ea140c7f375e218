#!/usr/bin/env python
"""Benchmark of the B200 DFlash draft step (one JSON line on rank 0).

Workload (BASELINE.json metric): Qwen3.5-27B-class DFlash draft -- hidden
5120, 40 q / 8 kv heads, head_dim 128, SwiGLU 17408, 5 layers, vocab 151936 --
W8A16 (int8 per-output-channel weights, fp16 scales), block 32, context 4096,
batch 1 per GPU.  A step is one stateless draft forward: fc + hidden_norm over
the 4096 context rows, 5 decoder layers, final norm, tied lm_head + greedy
argmax over the vocabulary and acceptance against synthetic target tokens
that keep each drafted token with probability 0.9.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU, each rank drafting its own
sequence (requests shard by batch with no collective on the hot path);
value = sum over ranks of drafted tokens / max over ranks of the step time.
`--impl reference` times the reference algorithm on the host CPU (the fp32
CPU restatement in oracle/, MLX being unavailable) on rank 0 only.
"""
import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "draft tok/s & µs/draft-step (27B-class, block 32, ctx 4K); % HBM roofline"
CFG_27B = dict(hidden_size=5120, num_hidden_layers=5, intermediate_size=17408, num_attention_heads=40,
               num_key_value_heads=8, head_dim=128, vocab_size=151936, block_size=32)
CFG_8B = dict(hidden_size=4096, num_hidden_layers=5, intermediate_size=12288, num_attention_heads=32,
              num_key_value_heads=8, head_dim=128, vocab_size=151936, block_size=16)
F = 5


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def step_bytes(c, ctx, batch):
    """Algorithmic HBM bytes of one draft step: int8 projection weights + fp32
    scales, bf16 fc and lm_head, bf16 target_hidden and noise rows."""
    H, I, nq, nkv, L, V = (c["hidden_size"], c["intermediate_size"], c["num_attention_heads"],
                           c["num_key_value_heads"], c["num_hidden_layers"], c["vocab_size"])
    per_layer = (nq * 128 * H) + 2 * (nkv * 128 * H) + H * nq * 128 + 3 * I * H
    scales = (nq * 128 + 2 * nkv * 128 + H + 2 * I + H) * 2
    return (L * (per_layer + scales) + H * F * H * 2 + V * H * 2
            + batch * ctx * F * H * 2 + batch * c["block_size"] * H * 2)


def step_flops(c, ctx, batch):
    H, I, nq, nkv, L, V, B = (c["hidden_size"], c["intermediate_size"], c["num_attention_heads"],
                              c["num_key_value_heads"], c["num_hidden_layers"], c["vocab_size"],
                              c["block_size"])
    rows_kv = ctx + B
    fc = 2 * ctx * F * H * H
    per_layer = 2 * B * H * nq * 128 + 2 * rows_kv * H * 2 * nkv * 128 + 2 * B * nq * 128 * H \
        + 2 * B * H * 2 * I + 2 * B * I * H + 4 * B * nq * rows_kv * 128
    return batch * (fc + L * per_layer + 2 * (B - 1) * V * H)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.rows, self.proc, self.marks = [], None, []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(gpu_id)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = [r for t, r in self.rows if t0 - 0.25 <= t <= t1 + 0.25] or [r for _, r in self.rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()), default=None)}


def build_model(pkg, cfgd, ctx, batch, device, seed=0):
    import torch
    cfg = pkg.DFlashConfig(**cfgd)
    cfg.target_layer_ids = list(range(F))
    w, lm = pkg.synth_weights_q8(cfg, seed=seed, device=device)
    model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=batch, max_ctx=ctx, max_block=cfg.block_size,
                                 device=device)
    return cfg, w, lm, model


def synth_inputs(cfgd, ctx, batch, device, seed):
    import torch
    g = torch.Generator(device=device).manual_seed(1000 + seed)
    H, B = cfgd["hidden_size"], cfgd["block_size"]
    noise = (torch.randn(batch, B, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    th = torch.randn(batch, ctx, F * H, generator=g, device=device).to(torch.bfloat16)
    return noise, th


def synth_targets(toks, vocab, p_keep, seed):
    """Target posterior that keeps each drafted id with probability p_keep."""
    import torch
    g = torch.Generator(device=toks.device).manual_seed(77 + seed)
    b, n = toks.shape
    keep = torch.rand(b, n, generator=g, device=toks.device) < p_keep
    other = (toks + 1 + torch.randint(0, vocab - 1, (b, n), generator=g, device=toks.device)) % vocab
    t = torch.where(keep, toks, other)
    bonus = torch.randint(0, vocab, (b, 1), generator=g, device=toks.device, dtype=torch.int32)
    return torch.cat([t.to(torch.int32), bonus], dim=1)


# ---------------------------------------------------------------- CPU (oracle) leg
def cpu_oracle_weights(w, lm):
    import torch
    from oracle import dflash_oracle as O
    deq = lambda l, k: (l.q[k].float() * l.s[k].float()[:, None]).cpu()
    layers = [O.OracleLayer(**{k: deq(l, k) for k in ["wq", "wk", "wv", "wo", "wg", "wu", "wd"]},
                            in_norm=l.input_layernorm.float().cpu(),
                            post_norm=l.post_attention_layernorm.float().cpu(),
                            q_norm=l.q_norm.float().cpu(), k_norm=l.k_norm.float().cpu()) for l in w.layers]
    return O.OracleWeights(w.fc.float().cpu(), w.hidden_norm.float().cpu(), w.norm.float().cpu(),
                           lm.float().cpu(), layers)


def cpu_step_time(cfgd, dense, noise, th, steps, warmup=0, budget_s=None):
    """Time full fp32 draft steps of the CPU oracle (forward + lm_head +
    argmax): `warmup` untimed steps, then `steps` timed ones (or fewer when
    `budget_s` seconds of timed steps run out).  Returns the timed durations."""
    import torch
    from oracle import dflash_oracle as O
    torch.set_num_threads(os.cpu_count())
    ocfg = O.OracleConfig(**cfgd)
    nz, tt = noise.float().cpu(), th.float().cpu()
    times = []
    with torch.no_grad():
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            hid = O.draft_forward(ocfg, dense, nz, tt)
            O.greedy(O.draft_logits(dense, hid, cfgd["block_size"]))
            if i >= warmup:
                times.append(time.perf_counter() - t0)
            if budget_s is not None and sum(times) > budget_s:
                break
    return times


def run_reference_arm(args, cfgd, rank, world):
    """The reference algorithm on the host CPU: the fp32 oracle restatement of
    mirror_sd/dflash.py (MLX cannot run here), on weights and inputs built on
    the CPU by the oracle itself (nothing of the CUDA library is loaded), with
    exactly --warmup untimed and --steps timed draft steps."""
    import torch
    from oracle import dflash_oracle as O
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count())
    ocfg = O.OracleConfig(**cfgd)
    ocfg.num_target_features = F
    t0 = time.perf_counter()
    _, dense = O.synth_weights(ocfg, seed=0, random_norms=False)
    noise, th = O.synth_inputs(ocfg, args.batch, args.ctx, cfgd["block_size"], seed=1)
    build_s = time.perf_counter() - t0
    times = cpu_step_time(cfgd, dense, noise, th, steps=args.steps, warmup=args.warmup)
    t = statistics.mean(times)
    toks = args.batch * (cfgd["block_size"] - 1)
    val = toks / t
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "draft tok/s",
            "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup, "ms_per_step": t * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, cfgd),
            "cpu_baseline": {"value": val, "unit": "draft tok/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": f"{len(times)} timed full draft steps (after {args.warmup} untimed) "
                                       f"of the fp32 CPU restatement (oracle/dflash_oracle.py; MLX "
                                       f"unavailable) on the same config, weights built on the CPU by the "
                                       f"oracle ({build_s:.0f} s, untimed), torch CPU with "
                                       f"{os.cpu_count()} threads"},
            "e2e": {"value": val, "unit": "draft tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(args, cfgd):
    return {"workload": f"{args.config}: DFlash draft step, W8A16, hidden {cfgd['hidden_size']}, "
                        f"{cfgd['num_attention_heads']}/{cfgd['num_key_value_heads']} heads, FFN "
                        f"{cfgd['intermediate_size']}, {cfgd['num_hidden_layers']} layers, vocab "
                        f"{cfgd['vocab_size']}, block {cfgd['block_size']}, ctx {args.ctx}, batch "
                        f"{args.batch} per GPU",
            "ctx": args.ctx, "block": cfgd["block_size"], "batch_per_gpu": args.batch,
            "accept_p": 0.9, "l2": "no flush: every step streams ~3.7 GB of weights/inputs (> 126 MB L2)",
            "parallelism": f"batch-sharded x{args.gpus}, no collectives"}


CFG_4B = dict(hidden_size=2560, num_hidden_layers=5, intermediate_size=9728, num_attention_heads=32,
              num_key_value_heads=8, head_dim=128, vocab_size=151936, block_size=16)


def run_fp32(args, pkg, rank, world, dev):
    """--config c1: the CPU plumbing config in fp32-accumulate mode on the GPU:
    4B-class dims, every weight fp32 N(0, 0.02), block 16, ctx 64, batch 1
    per GPU, block ids uniform with position 0 the mask id (embedded by the
    tied lm_head), target_hidden N(0, 1).  A step is the fp32 draft forward
    + lm_head argmax + acceptance on the CUDA cores, replayed from a CUDA
    graph.  Returns the JSON line on rank 0."""
    import torch
    shard = importlib.import_module("mirror-sd_b200.shard")
    cfgd = dict(CFG_4B)
    cfg = pkg.DFlashConfig(**cfgd)
    cfg.target_layer_ids = list(range(F))
    w, lm = pkg.synth_weights_f32(cfg, seed=0, device=dev)
    B, H, V, C = cfgd["block_size"], cfgd["hidden_size"], cfgd["vocab_size"], args.ctx
    model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=args.batch, max_ctx=C, max_block=B, device=dev)
    g = torch.Generator(device=dev).manual_seed(rank)
    ids = torch.randint(0, V, (args.batch, B), generator=g, device=dev)
    ids[:, 0] = cfg.mask_token_id
    noise = lm[ids]
    th = torch.randn(args.batch, C, F * H, generator=g, device=dev)
    out_t = torch.empty((args.batch, B - 1), dtype=torch.int32, device=dev)
    _, toks, _, _ = model.draft_step(noise, th, want_hidden=False)
    target = synth_targets(toks, V, 0.9, rank)
    acc = torch.empty((args.batch,), dtype=torch.int32, device=dev)
    cor = torch.empty((args.batch,), dtype=torch.int32, device=dev)

    def step():
        model.draft_step(noise, th, target_tokens=target, want_hidden=False, out_tokens=out_t, acc_len=acc,
                         correction=cor)

    for _ in range(args.warmup):
        step()
    launches = model._lib.dflash_last_launch_count(model._handle)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(dev).wait_stream(side)
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        step()
    for _ in range(3):
        graph.replay()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local_gpu_id(dev)) if rank == 0 else None
    time.sleep(0.6 if sampler else 0)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    s0.record()
    for _ in range(args.steps):
        graph.replay()
    s1.record()
    torch.cuda.synchronize(dev)
    t1 = time.time()
    if sampler:
        sampler.stop()
    ms = shard.max_over_ranks(s0.elapsed_time(s1) / args.steps)
    del graph
    model.close()
    if rank != 0:
        return None
    hbm = peaks()[0]
    I, NQ, NKV, L = cfgd["intermediate_size"], cfgd["num_attention_heads"], cfgd["num_key_value_heads"], \
        cfgd["num_hidden_layers"]
    params = L * ((NQ + 2 * NKV) * 128 * H + H * NQ * 128 + 3 * I * H) + F * H * H + V * H
    nbytes = 4 * (params + args.batch * (C * F * H + B * H))
    return {"metric": "draft tok/s, fp32-accumulate mode (c1: 4B-class, fp32 weights, block 16, ctx 64)",
            "value": shard.job_throughput([args.batch * (B - 1)] * world, ms), "unit": "draft tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32: fp32 weights, activations and accumulation (CUDA cores)", "data": "synthetic",
            "config": {"workload": f"c1: 4B-class fp32 draft, block {B}, ctx {C}, batch {args.batch} per GPU",
                       "parallelism": f"batch-sharded x{world}, no collectives"},
            "roofline": {"bound": "hbm", "bytes_per_step": nbytes, "achieved": nbytes / (ms / 1e3) / 1e9,
                         "peak": hbm, "unit": "GB/s", "frac": nbytes / (ms / 1e3) / 1e9 / hbm},
            "launches_per_step": launches,
            "clocks": sampler.summary(t0, t1) if sampler else None}


def run_serving(args, pkg, rank, world, dev):
    """--config c5: batched serving on the 8B-class draft.  256 requests with
    contexts uniform in [512, 8192] and block 16 are sharded over the ranks
    (longest first, no collective); each rank prefills its requests into one
    sink 64 / window 1024 draft cache in 16K-row chunks, then times decode
    steps of all its requests together.  A synthetic verifier accepts a
    geometric number of drafts per request (P(accept >= k) = 0.85^k); the
    next step brings accept + 1 context rows per request.  One step = the
    draft forward of every request (dense tcgen05 projections and lm_head at
    these row counts), the verifier emulation (two small torch ops), device
    acceptance, the accepted lengths read back, and the block-row trim.
    Returns the JSON line on rank 0 (None elsewhere)."""
    import torch
    shard = importlib.import_module("mirror-sd_b200.shard")
    serving = importlib.import_module("mirror-sd_b200.serving")
    cfgd = dict(CFG_8B)
    B, H, V = cfgd["block_size"], cfgd["hidden_size"], cfgd["vocab_size"]
    g = torch.Generator().manual_seed(5)
    ctx_all = torch.randint(512, 8193, (args.seqs,), generator=g).tolist()
    mine = shard.shard_requests(ctx_all, world, rank, B)
    n = len(mine)
    ctx = [ctx_all[i] for i in mine]
    chunk_rows = 16384
    cfg = pkg.DFlashConfig(**cfgd)
    cfg.target_layer_ids = list(range(F))
    w, lm = pkg.synth_weights_q8(cfg, seed=0, device=dev)
    model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=n, max_ctx=8192, max_block=B, device=dev,
                                 max_ctx_rows=chunk_rows)
    server = serving.DraftServer(model, n, sink_size=64, window_size=1024)
    gd = torch.Generator(device=dev).manual_seed(17 + rank)
    pool = torch.randn(chunk_rows, F * H, generator=gd, device=dev).to(torch.bfloat16)
    noise = (torch.randn(n, B, H, generator=gd, device=dev) * 0.02).to(torch.bfloat16)
    # prefill (timed separately): chunks of whole requests within the row budget
    torch.cuda.synchronize(dev)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    i = 0
    while i < n:
        j, rows = i, 0
        while j < n and rows + ctx[j] <= chunk_rows:
            rows += ctx[j]
            j += 1
        server.prefill(list(range(i, j)), noise[i:j], pool[:rows], ctx[i:j])
        i = j
    p1.record()
    torch.cuda.synchronize(dev)
    prefill_ms = p0.elapsed_time(p1)
    steps = args.warmup + args.steps
    plan = torch.tensor(serving.geometric_accepts(n, steps + 1, 0.85, B - 1, seed=100 + rank),
                        dtype=torch.int32, device=dev)
    seqs = list(range(n))
    out_t = torch.empty((n, B - 1), dtype=torch.int32, device=dev)
    lens = [int(a) + 1 for a in plan[0].tolist()]      # the prefill step's verify outcome

    def dstep(t, lens):
        server.step(seqs, noise, pool[:sum(lens)], lens, out_tokens=out_t)
        tgt = serving.targets_for(out_t, plan[t + 1], V)
        a, _ = pkg.accept(out_t, tgt)
        return [int(x) + 1 for x in a.cpu().tolist()]

    for t in range(args.warmup):
        lens = dstep(t, lens)
    launches = model._lib.dflash_last_launch_count(model._handle)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local_gpu_id(dev)) if rank == 0 else None
    time.sleep(0.6 if sampler else 0)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    s.record()
    accepted, ctx_rows = 0, 0
    for t in range(args.warmup, steps):
        ctx_rows += sum(lens)
        lens = dstep(t, lens)
        accepted += sum(x - 1 for x in lens)
    e.record()
    torch.cuda.synchronize(dev)
    t_wall1 = time.time()
    if world > 1:
        dist.barrier()
    ms = s.elapsed_time(e) / args.steps
    ms_max = shard.max_over_ranks(ms)
    per_rank = shard.gather_to_rank0({"n": n, "accepted": accepted, "ctx_rows": ctx_rows,
                                      "prefill_ms": prefill_ms, "prefill_rows": sum(ctx)})
    if sampler:
        sampler.stop()
    line = None
    if rank == 0:
        hbm, tf_burst, tf_sust, src = peaks()
        # burst peak for a sub-second timed region, the sustained one beyond
        tf_peak, peak_name = (tf_burst, "bf16_tflops") if ms * args.steps < 1e3 else \
            (tf_sust, "bf16_tflops_sustained")
        n_all = sum(r["n"] for r in per_rank)
        acc_all = sum(r["accepted"] for r in per_rank)
        M = n * B
        L, NQ, NKV, I = cfgd["num_hidden_layers"], cfgd["num_attention_heads"], cfgd["num_key_value_heads"], \
            cfgd["intermediate_size"]
        params = (NQ + 2 * NKV) * 128 * H + H * NQ * 128 + 3 * I * H
        cr = ctx_rows / args.steps
        flops = 2.0 * M * (L * params + V * H) + 2.0 * cr * (F * H * H + H * L * 2 * NKV * 128)
        line = {
            "metric": "batched serving draft tok/s (8B-class, 256 requests, ctx U[512, 8192], block 16)",
            "value": shard.job_throughput([r["n"] * (B - 1) for r in per_rank], ms_max),
            "unit": "draft tok/s", "accepted_tok_s": acc_all / args.steps / (ms_max / 1e3),
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "w8a16: int8 weights (exact f16 copies on the dense path), bf16/f16 activations, "
                     "fp32 accumulate", "data": "synthetic",
            "config": {"workload": "c5 batched serving", "requests": args.seqs, "requests_this_rank0": n,
                       "block": B, "ctx": "U[512, 8192] prefilled", "cache": "sink 64 / window 1024",
                       "accept": "geometric p=0.85", "parallelism": f"requests sharded over {world} GPU(s)"},
            "tensor_roofline": {"flops_per_step_rank0": flops, "achieved_tflops": flops / (ms / 1e3) / 1e12,
                                "peak": tf_peak, "frac": flops / (ms / 1e3) / 1e12 / tf_peak,
                                "frac_of_sustained": flops / (ms / 1e3) / 1e12 / tf_sust,
                                "peak_source": f"{src} {peak_name} (timed region {ms * args.steps:.0f} ms)"},
            "prefill": {"rows": sum(r["prefill_rows"] for r in per_rank),
                        "ms_max": max(r["prefill_ms"] for r in per_rank)},
            "mean_accept": acc_all / (args.steps * n_all),
            "gpu_launches_per_step": launches + 2,
            "clocks": sampler.summary(t_wall0, t_wall1) if sampler else None,
        }
    server.close()
    model.close()
    return line


# ---------------------------------------------------------------- kernel cases
KERNEL_CASES = """\
Kernel cases (--kernel CASE), each one hot-path kernel through its C entry
point on the 27B-class dims (32 block rows), small enough for an ncu capture
(< 2 GB on the device, more than the 126 MB L2 streamed per launch):
  w8_gu    gate|up W8A16 projection   N=34816 K=5120   (178 MB int8)
  w8_down  down W8A16 projection      N=5120  K=17408  (89 MB)
  w8_qkv   fused q|k|v projection     N=7168  K=5120   (37 MB)
  w8_o     o projection               N=5120  K=5120   (26 MB)
  w8:N:K   any W8A16 shape (N, K multiples of 128)
  lm_head  tied lm_head + argmax      V=151936 H=5120  (1.56 GB bf16)
  attn     block attention            40/8 heads, 32 queries, kv 4128
  attn16   the same at batch 16, kv 32800 (2.1 GB of K/V)
  attn_c5  the batched serving shape: 256 sequences, 32 q / 8 kv heads, 16
           queries, kv 1104 (a sink 64 / window 1024 cache plus the block)
  fc       context fc GEMM            4096 x 25600 x 5120 (bf16)
  step1    one draft step at the bench's 27B dims (block 32, ctx 4096, batch 1)
           with one decoder layer: the fc and context K|V GEMMs exactly as in
           the bench with about 4 GB on the device
  serve    one stateless draft step of --seqs sequences (64 by default) of
           block 16, ctx 64 each, 8B-class dims: the dense block path
"""


def run_kernel_case(case, iters, warmup, seqs):
    """Time one kernel case with CUDA events (mean of `iters` launches after
    `warmup`) and print one JSON line: time, algorithmic bytes and flops."""
    import torch
    pkg = _pkg()
    K = importlib.import_module("mirror-sd_b200.kernels")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    M = 32
    if case.startswith("w8_") or case.startswith("w8:"):
        if case.startswith("w8:"):
            N, Kd = (int(v) for v in case.split(":")[1:3])
        else:
            N, Kd = {"w8_gu": (34816, 5120), "w8_down": (5120, 17408), "w8_qkv": (7168, 5120),
                     "w8_o": (5120, 5120)}[case]
        q = torch.randint(-127, 128, (N, Kd), generator=g, device=dev, dtype=torch.int8)
        s = (torch.rand(N, generator=g, device=dev) * 1e-3).to(torch.float16)
        x = torch.randn(M, Kd, generator=g, device=dev).to(torch.float16)
        fn = lambda: K.w8_linear(q, s, x)
        nbytes, flops = N * Kd, 2 * M * N * Kd
    elif case == "lm_head":
        V, H = 151936, 5120
        E = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        hn = torch.randn(1, M, H, generator=g, device=dev).to(torch.bfloat16)
        ws = torch.empty(pkg._native.load().dflash_lm_head_workspace_size(1, M, V, H), dtype=torch.uint8,
                         device=dev)
        fn = lambda: K.lm_head_argmax(hn, E, workspace=ws)
        nbytes, flops = V * H * 2, 2 * (M - 1) * V * H
    elif case in ("attn", "attn16", "attn_c5"):
        bsz, L, nq, Mq = {"attn": (1, 4128, 40, M), "attn16": (16, 32800, 40, M),
                          "attn_c5": (256, 1104, 32, 16)}[case]
        qq = torch.randn(bsz, nq, Mq, 128, generator=g, device=dev).to(torch.float16)
        kk = torch.randn(bsz, 8, L, 128, generator=g, device=dev).to(torch.float16)
        vv = torch.randn(bsz, 8, L, 128, generator=g, device=dev).to(torch.float16)
        ws = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        fn = lambda: K.attention(qq, kk, vv, workspace=ws)
        nbytes, flops = bsz * 2 * 8 * L * 128 * 2, bsz * 4 * nq * Mq * L * 128
    elif case == "step1":
        cfg = pkg.DFlashConfig(**dict(CFG_27B, num_hidden_layers=1))
        cfg.target_layer_ids = list(range(F))
        w, lm = pkg.synth_weights_q8(cfg, seed=0, device=dev)
        C, B, H = 4096, 32, 5120
        model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=1, max_ctx=C, max_block=B, device=dev)
        noise = (torch.randn(1, B, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        th = torch.randn(1, C, F * H, generator=g, device=dev).to(torch.bfloat16)
        toks = torch.empty((1, B - 1), dtype=torch.int32, device=dev)
        fn = lambda: model.draft_step(noise, th, want_hidden=False, out_tokens=toks)
        nbytes = C * F * H * 2 + H * F * H * 2
        flops = 2 * C * F * H * H + 2 * C * H * 2 * 8 * 128
    elif case == "serve":
        cfg = pkg.DFlashConfig(**CFG_8B)
        cfg.target_layer_ids = list(range(F))
        w, lm = pkg.synth_weights_q8(cfg, seed=0, device=dev)
        n, C, B, H = seqs, 64, 16, 4096
        model = pkg.DFlashDraftModel(cfg, w, lm, max_batch=n, max_ctx=C, max_block=B, device=dev)
        noise = (torch.randn(n, B, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        th = torch.randn(n, C, F * H, generator=g, device=dev).to(torch.bfloat16)
        toks = torch.empty((n, B - 1), dtype=torch.int32, device=dev)
        fn = lambda: model.draft_step(noise, th, want_hidden=False, out_tokens=toks)
        params = 5 * ((32 + 16) * 128 * H + H * 32 * 128 + 3 * 12288 * H)
        nbytes = params * 2 + 151936 * H * 2
        flops = 2 * n * B * (params + 151936 * H) + 2 * n * C * (F * H * H + H * 5 * 2 * 8 * 128)
    elif case == "fc":
        Mr, Kd, N = 4096, 25600, 5120
        A = torch.randn(Mr, Kd, generator=g, device=dev).to(torch.bfloat16)
        Bm = (torch.randn(N, Kd, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        fn = lambda: K.tc_gemm(A, Bm)
        nbytes, flops = (Mr + N) * Kd * 2, 2 * Mr * N * Kd
    else:
        raise SystemExit(f"unknown kernel case {case}\n{KERNEL_CASES}")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / iters
    print(json.dumps({"kernel_case": case, "us_per_call": ms * 1e3, "bytes": nbytes, "flops": flops,
                      "gb_s": nbytes / ms / 1e6, "tflop_s": flops / ms / 1e9, "iters": iters,
                      "warmup": warmup}), flush=True)


def run_attention_sweep(iters):
    """c4: block attention (40 query / 8 kv heads, 32 queries, head 128) over
    ctx 1K..32K at batch 1 and 16, one JSON line per point; algorithmic bytes =
    Q + O + K + V (f16), fraction of the measured HBM copy peak."""
    import torch
    _pkg()
    K = importlib.import_module("mirror-sd_b200.kernels")
    lib = importlib.import_module("mirror-sd_b200._native").load()
    hbm = peaks()[0]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    ws = None
    for b in (1, 16):
        for C in (1024, 4096, 8192, 16384, 32768):
            L = C + 32
            q = torch.randn(b, 40, 32, 128, generator=g, device=dev).to(torch.float16)
            k = torch.randn(b, 8, L, 128, generator=g, device=dev).to(torch.float16)
            v = torch.randn(b, 8, L, 128, generator=g, device=dev).to(torch.float16)
            need = lib.dflash_attention_workspace_size(b, 40, 8, 32, L)
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
            print(json.dumps({"config": "c4 attention sweep", "batch": b, "ctx": C, "kv_rows": L,
                              "bytes": nbytes, "us": us, "gb_s": nbytes / us / 1e3,
                              "hbm_frac": nbytes / us / 1e3 / hbm, "tflop_s": flops / us / 1e6}), flush=True)
            del q, k, v


def _cpulist(txt):
    cpus = set()
    for part in txt.split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_numa(dev):
    """(NUMA node, set of local CPUs) of the GPU's PCI device from sysfs,
    restricted to the CPUs this process may use; (None, None) when unknown."""
    import torch
    p = torch.cuda.get_device_properties(dev)
    path = f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    try:
        with open(os.path.join(path, "numa_node")) as f:
            node = int(f.read().strip())
        with open(os.path.join(path, "local_cpulist")) as f:
            cpus = _cpulist(f.read()) & os.sched_getaffinity(0)
    except (OSError, ValueError):
        return None, None
    return node, (cpus or None)


def local_gpu_id(dev):
    import torch
    props = torch.cuda.get_device_properties(dev)
    uid = getattr(props, "uuid", None)
    return f"GPU-{uid}" if uid is not None else dev.index


def _pkg():
    import importlib
    pkg = importlib.import_module("mirror-sd_b200")
    sys.modules.setdefault("mirror_sd_b200", pkg)
    return pkg


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c3", "c2", "c5", "c4", "c1"], default="c3",
                    help="c3 headline; c2 8B step; c5 batched serving; c4 attention sweep; "
                         "c1 fp32-accumulate mode")
    ap.add_argument("--kernel", default=None, help="time one kernel case instead (list: --kernel help)")
    ap.add_argument("--iters", type=int, default=20, help="--kernel / c4: timed launches")
    ap.add_argument("--seqs", type=int, default=256, help="c5: requests over all GPUs")
    ap.add_argument("--ctx", type=int, default=None)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-serving", action="store_true",
                    help="skip the batched c5 serving run that the c3 line carries under 'serving'")
    ap.add_argument("--serving-steps", type=int, default=10)
    args = ap.parse_args()
    if args.kernel is not None:
        if args.kernel == "help":
            print(KERNEL_CASES)
            return
        run_kernel_case(args.kernel, args.iters, args.warmup, args.seqs)
        return
    if args.config == "c4":
        run_attention_sweep(args.iters)
        return
    cfgd = dict(CFG_27B if args.config == "c3" else CFG_8B)
    if args.ctx is None:
        args.ctx = {"c3": 4096, "c1": 64}.get(args.config, 2048)
    if args.warmup < 3:
        args.warmup = 3

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # CPU only: rank 0 runs it, the other ranks exit at once (no process
        # group, no CUDA context)
        run_reference_arm(args, cfgd, rank, world)
        return
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    pkg = _pkg()
    shard = importlib.import_module("mirror-sd_b200.shard")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.config in ("c5", "c1"):
        if args.steps == 200:
            args.steps = 20
        line = (run_serving if args.config == "c5" else run_fp32)(args, pkg, rank, world, dev)
        if line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    cfg, w, lm, model = build_model(pkg, cfgd, args.ctx, args.batch, dev, seed=0)
    B = cfgd["block_size"]
    # world * batch independent requests; this rank drafts its share (no collective on the data path)
    mine = shard.shard_requests([args.ctx] * (world * args.batch), world, rank, B)
    noise, th = synth_inputs(cfgd, args.ctx, len(mine), dev, mine[0])
    out_h = torch.empty((args.batch, B, cfgd["hidden_size"]), dtype=torch.bfloat16, device=dev)
    out_t = torch.empty((args.batch, B - 1), dtype=torch.int32, device=dev)
    acc = torch.empty((args.batch,), dtype=torch.int32, device=dev)
    cor = torch.empty((args.batch,), dtype=torch.int32, device=dev)
    _, toks, _, _ = model.draft_step(noise, th, want_hidden=False)
    target = synth_targets(toks, cfgd["vocab_size"], 0.9, rank)

    def step(events=None):
        model.draft_step(noise, th, target_tokens=target, out_hidden=out_h, out_tokens=out_t,
                         acc_len=acc, correction=cor, phase_events=events)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    launches_per_step = model._lib.dflash_last_launch_count(model._handle)

    # per-step phase events (recorded by the library on the launch stream)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(8)] for _ in range(args.steps)]
    for es in ev:
        for e in es:
            e.record()
    torch.cuda.synchronize(dev)
    props = torch.cuda.get_device_properties(dev)
    gpu_id = getattr(props, "uuid", None)
    sampler = ClockSampler(f"GPU-{gpu_id}" if gpu_id is not None else local) if rank == 0 else None
    time.sleep(0.6 if sampler else 0)
    for _ in range(3):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    start.record()
    for i in range(args.steps):
        step(ev[i])
    end.record()
    torch.cuda.synchronize(dev)
    t_wall1 = time.time()
    if world > 1:
        dist.barrier()
    ms_eager = start.elapsed_time(end) / args.steps

    # the same step captured once in a CUDA graph and replayed: the headline
    # step time (launch overhead off the host; every kernel still runs)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(dev).wait_stream(side)
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        step()
    for _ in range(3):
        graph.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gs.record()
    for _ in range(args.steps):
        graph.replay()
    ge.record()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = gs.elapsed_time(ge) / args.steps
    del graph
    phases = {}
    names = pkg._native.PHASE_NAMES
    for k in range(1, 8):
        phases[names[k]] = statistics.mean(ev[i][k - 1].elapsed_time(ev[i][k]) for i in range(args.steps))
    ms_max = shard.max_over_ranks(ms)
    ms_eager_max = shard.max_over_ranks(ms_eager)
    accs = shard.gather_to_rank0(acc.cpu().tolist())
    acc_mean = statistics.mean(a for r in accs for a in r) if accs else None

    # end-to-end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # pinned host buffers on the GPU's own NUMA node: allocate them from
        # the CPUs local to the GPU's PCI device, then restore the affinity
        node, local_cpus = gpu_numa(dev)
        saved_aff = os.sched_getaffinity(0)
        if local_cpus:
            try:
                os.sched_setaffinity(0, local_cpus)
            except OSError:   # the placement is an optimisation, never a requirement
                local_cpus = None
        noise_h = noise.cpu().pin_memory()
        th_h = th.cpu().pin_memory()
        tgt_h = target.cpu().pin_memory()
        tok_h = torch.empty((args.batch, B - 1), dtype=torch.int32).pin_memory()
        acc_h = torch.empty((args.batch,), dtype=torch.int32).pin_memory()
        cor_h = torch.empty((args.batch,), dtype=torch.int32).pin_memory()
        try:
            os.sched_setaffinity(0, saved_aff)
        except OSError:
            pass
        # this rank's host->device rate alone (one copy of target_hidden)
        th_probe = torch.empty_like(th)
        torch.cuda.synchronize(dev)
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record()
        th_probe.copy_(th_h, non_blocking=True)
        h1.record()
        torch.cuda.synchronize(dev)
        h2d_alone = th.numel() * 2 / (h0.elapsed_time(h1) / 1e3) / 1e9
        del th_probe
        # two input buffer sets: step i+1's host->device copies run on a copy
        # stream while step i computes; every step's copies are in the timed region
        bufs = [(torch.empty_like(noise), torch.empty_like(th), torch.empty_like(target)) for _ in range(2)]
        copy_st = torch.cuda.Stream(dev)
        comp_st = torch.cuda.current_stream(dev)
        copied = [torch.cuda.Event() for _ in range(2)]
        used = [torch.cuda.Event() for _ in range(2)]
        for e in used:
            e.record(comp_st)
        k2 = max(5, min(args.steps, 50))

        def issue_copy(i):
            nd, td, tg = bufs[i % 2]
            with torch.cuda.stream(copy_st):
                copy_st.wait_event(used[i % 2])  # step i-2 has finished with this set
                nd.copy_(noise_h, non_blocking=True)
                td.copy_(th_h, non_blocking=True)
                tg.copy_(tgt_h, non_blocking=True)
                copied[i % 2].record(copy_st)

        def e2e_run(n):
            copy_st.wait_stream(comp_st)  # the first copy starts after the start event
            issue_copy(0)
            for i in range(n):
                if i + 1 < n:
                    issue_copy(i + 1)
                nd, td, tg = bufs[i % 2]
                comp_st.wait_event(copied[i % 2])
                model.draft_step(nd, td, target_tokens=tg, want_hidden=False, out_tokens=out_t,
                                 acc_len=acc, correction=cor)
                used[i % 2].record(comp_st)
                tok_h.copy_(out_t, non_blocking=True)
                acc_h.copy_(acc, non_blocking=True)
                cor_h.copy_(cor, non_blocking=True)

        e2e_run(3)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(comp_st)
        e2e_run(k2)
        e2.record(comp_st)
        torch.cuda.synchronize(dev)
        ms_e2e = shard.max_over_ranks(s2.elapsed_time(e2) / k2)
        h2d = noise.numel() * 2 + th.numel() * 2 + target.numel() * 4
        d2h = out_t.numel() * 4 + acc.numel() * 4 + cor.numel() * 4
        ranks_h2d = shard.gather_to_rank0({"gpu_numa_node": node, "local_cpus": len(local_cpus or []),
                                           "h2d_gbs_alone": h2d_alone,
                                           "h2d_gbs_in_e2e": h2d / (ms_e2e / 1e3) / 1e9})
        e2e = {"value": shard.job_throughput([args.batch * (B - 1)] * world, ms_e2e), "unit": "draft tok/s",
               "ms_per_step": ms_e2e, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "steps": k2, "api": "DFlashDraftModel.draft_step on pinned host tensors; the next step's "
               "host->device copies overlap the current step (copy stream, two buffer sets)",
               "host_buffers": "pinned, allocated from the CPUs local to the GPU's PCI device (NUMA node "
                               "of the GPU) when sysfs names them",
               "per_rank": ranks_h2d}

    if sampler:
        sampler.stop()
    cpu_base = None
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        dense = cpu_oracle_weights(w, lm)
        times = cpu_step_time(cfgd, dense, noise, th, steps=2, warmup=0, budget_s=30)
        t = min(times)
        cpu_base = {"value": args.batch * (B - 1) / t, "unit": "draft tok/s",
                    "cores": os.cpu_count(), "kind": "port",
                    "sample": f"{len(times)} full fp32 draft step(s) (oracle/dflash_oracle.py, "
                              f"the reference's MLX being unavailable), best of them"}
        del dense
    model.close()
    del model, w, lm
    torch.cuda.empty_cache()
    # the batched config (c5) on the same GPUs, reported under "serving"
    serving = None
    if not args.no_serving:
        sargs = argparse.Namespace(**vars(args))
        sargs.steps, sargs.warmup = args.serving_steps, 3
        serving = run_serving(sargs, pkg, rank, world, dev)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    hbm, tf_burst, tf_sust, src = peaks()
    nbytes = step_bytes(cfgd, args.ctx, args.batch)
    nflops = step_flops(cfgd, args.ctx, args.batch)
    fc_flops = 2.0 * args.batch * args.ctx * F * cfgd["hidden_size"] * cfgd["hidden_size"]
    t_fc = phases["fc_gemm"] / 1e3
    fc_tfs = fc_flops / t_fc / 1e12 if t_fc > 0 else None
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get(f"fc_gemm_{args.config}_ctx{args.ctx}")
    t_step = ms_max / 1e3
    # The timed region of the headline is K graph replays of a ~2 ms step: a
    # burst, well under the seconds-long loop (at ~1350 MHz under the power
    # cap) the sustained peak was measured over, so the burst peak is the
    # denominator; the sustained fraction is reported beside it.
    timed_s = ms * args.steps / 1e3
    if timed_s < 1.0:
        tf_peak, peak_name = tf_burst, "bf16_tflops"
        peak_why = f"burst peak, the timed region is {timed_s * 1e3:.0f} ms"
    else:
        tf_peak, peak_name = tf_sust, "bf16_tflops_sustained"
        peak_why = f"sustained peak, the timed region is {timed_s:.1f} s"
    line = {
        "metric": METRIC, "value": shard.job_throughput([args.batch * (B - 1)] * world, ms_max),
        "unit": "draft tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "us_per_step": ms_max * 1e3, "timing": "CUDA graph of one step, replayed K times; events on the "
        "replay stream", "ms_per_step_eager": ms_eager_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "w8a16: int8 weights, bf16/f16 activations, fp32 accumulate", "data": "synthetic",
        "config": workload_config(args, cfgd),
        "roofline": {"bound": "tensor", "kernel": "fc GEMM (tcgen05, bf16)", "achieved": fc_tfs,
                     "peak": tf_peak, "unit": "TFLOP/s", "frac": (fc_tfs / tf_peak) if fc_tfs else None,
                     "frac_of_sustained": (fc_tfs / tf_sust) if fc_tfs else None,
                     "peak_source": f"{src} {peak_name}: {peak_why}", "traffic": traffic,
                     "flops_per_launch": fc_flops, "launch_ms": phases["fc_gemm"]},
        "step_roofline": {"bytes": nbytes, "flops": nflops,
                          "hbm_floor_ms": nbytes / (hbm * 1e9) * 1e3,
                          "tensor_floor_ms": nflops / (tf_peak * 1e12) * 1e3,
                          "frac_of_max_floor": max(nbytes / (hbm * 1e9), nflops / (tf_peak * 1e12)) / t_step,
                          "frac_of_max_floor_sustained": max(nbytes / (hbm * 1e9),
                                                             nflops / (tf_sust * 1e12)) / t_step,
                          "hbm_frac": nbytes / t_step / (hbm * 1e9)},
        "phases_ms": phases, "accept_len_mean": acc_mean,
        "gpu_launches": launches_per_step * args.steps, "launches_per_step": launches_per_step,
        "clocks": sampler.summary(t_wall0, t_wall1) if sampler else None,
        "e2e": e2e,
    }
    if cpu_base is not None:
        line["cpu_baseline"] = cpu_base
    if serving is not None:
        line["serving"] = serving
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
