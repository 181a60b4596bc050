"""Benchmark of the teenygrad hot path on B200.

Default workload (BASELINE metric "tokens/s (1B decoder)"): the Llama-style
1B decoder (16 layers, d 2048, 32/8 heads x 64, SwiGLU 8192, vocab 32000,
bf16, N(0, 0.02) random init), batch 16 prompts of 1024 uniform-random ids
per GPU, prefill + 128 greedy tokens.  One step = that whole generation.
Multi-GPU: one process per GPU, weak scaling (16 sequences per GPU), the
generated ids all-gathered over NCCL at the end of every step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c4|c5|c3]

--impl reference times the CPU oracle port of the same workload (the
reference has no runnable CPU or GPU implementation) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C4 = dict(n_layers=16, d_model=2048, n_heads=32, n_kv_heads=8, head_dim=64, ffn_hidden=8192, vocab=32000,
          batch=16, prompt=1024, gen=128)
C5 = dict(n_layers=16, d_model=2048, n_heads=32, n_kv_heads=8, head_dim=64, ffn_hidden=8192, vocab=32000,
          batch=64, ctx=2048)
C3 = dict(B=8, H=32, S=4096, D=128)
C2 = dict(B=32, C=64, H=56, W=56, layers=4)
C1 = dict(B=1, S=128, d=256, heads=4, ffn=1024)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm=d["hbm_gbs"], tc=d["bf16_tflops"], tc_sus=d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                    src="measured")
    return dict(hbm=6650.0, tc=1590.0, tc_sus=1400.0, src="fallback")


# ------------------------------------------------------------------ clocks --
class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""

    def __init__(self, index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.seek(0)
        rows = [l.split(",") for l in self.f.read().strip().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- helpers ----
def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    if n_gpus > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        from datetime import timedelta
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        return dist.get_rank(), dist.get_world_size(), local
    torch.cuda.set_device(0)
    return 0, 1, 0


def barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_loop(fn, iters, stream=None):
    """Average ms per call, CUDA events on the launching (current) stream."""
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(iters):
        fn()
    e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def graph_time(fn, iters=10):
    """ms per replay of a CUDA graph that captures fn() once (kernel time
    without host launch overhead)."""
    import torch
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
        fn()
    g.replay()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(iters):
        g.replay()
    e1.record(cur)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def graph_time_flushed(fn, iters=10):
    """ms per replay of a CUDA graph of fn(), with L2 (126 MB) flushed by a
    256 MB write before every replay; only the replays are timed."""
    import torch
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
        fn()
    g.replay()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    cur = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for e0, e1 in evs:
        flush.fill_(1)
        e0.record(cur)
        g.replay()
        e1.record(cur)
    torch.cuda.synchronize()
    return sum(e0.elapsed_time(e1) for e0, e1 in evs) / iters


# ------------------------------------------------------------ CPU baseline --
def cpu_baseline_c4(budget_s=25.0):
    """Oracle port on host cores: 1 of 16 layers for 1 of 16 sequences,
    prefill of the 1024-token prompt plus decode steps, extrapolated to the
    whole workload (16 layers x 16 sequences x (prefill + 128 tokens))."""
    import numpy as np
    import oracle
    from oracle.decoder import OracleDecoder
    c = C4

    class Cfg:
        n_layers = 1
        d_model = c["d_model"]
        n_heads = c["n_heads"]
        n_kv_heads = c["n_kv_heads"]
        head_dim = c["head_dim"]
        ffn_hidden = c["ffn_hidden"]
        vocab = 512          # the LM head / embedding are timed separately below
        rope_theta = 10000.0
        norm_eps = 1e-5

    r = np.random.default_rng(0)
    d, F = Cfg.d_model, Cfg.ffn_hidden
    qd, kd = Cfg.n_heads * Cfg.head_dim, Cfg.n_kv_heads * Cfg.head_dim

    def w(*s):
        return oracle.round_bf16((r.standard_normal(s, dtype=np.float32) * 0.02))

    layer = dict(attn_norm=np.ones(d, np.float32), wq=w(qd, d), wk=w(kd, d), wv=w(kd, d), wo=w(d, qd),
                 mlp_norm=np.ones(d, np.float32), w_gate=w(F, d), w_up=w(F, d), w_down=w(d, F))
    params = dict(embed=oracle.round_bf16(r.standard_normal((Cfg.vocab, d), dtype=np.float32)),
                  lm_head=w(Cfg.vocab, d), final_norm=np.ones(d, np.float32), layers=[layer])
    dec = OracleDecoder(Cfg, params)
    ids = r.integers(0, Cfg.vocab, (1, c["prompt"]))
    t0 = time.perf_counter()
    dec.forward(ids)
    t_prefill = time.perf_counter() - t0
    n_dec, t1 = 0, time.perf_counter()
    while n_dec < 3 and time.perf_counter() - t1 < budget_s * 0.3:
        dec.forward(r.integers(0, Cfg.vocab, (1, 1)))
        n_dec += 1
    t_dec = (time.perf_counter() - t1) / max(n_dec, 1)
    # LM head per token (32000 x 2048), measured once on a 4000-row slice
    xs = oracle.round_bf16(r.standard_normal((1, d), dtype=np.float32))
    wl = w(4000, d)
    t2 = time.perf_counter()
    oracle.linear(xs, wl)
    t_lm = (time.perf_counter() - t2) * (c["vocab"] / 4000)
    per_seq = c["n_layers"] * (t_prefill + c["gen"] * t_dec) + (c["gen"] + 1) * t_lm
    total = c["batch"] * per_seq
    tokens = c["batch"] * (c["prompt"] + c["gen"])
    return {"value": tokens / total, "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": (f"oracle C port, 1 of {c['n_layers']} layers x 1 of {c['batch']} sequences: prefill "
                       f"{c['prompt']} tokens ({t_prefill:.2f}s) + {n_dec} decode steps ({t_dec*1e3:.0f} ms each) "
                       f"+ LM head ({t_lm*1e3:.0f} ms/token), extrapolated to the full workload ({total:.0f}s)")}


def cpu_baseline_c5(budget_s=20.0):
    """Oracle int8 decode step, 1 of 16 layers x 1 of 64 sequences, bytes/s."""
    import numpy as np
    import oracle
    c = C5
    r = np.random.default_rng(0)
    d, F = c["d_model"], c["ffn_hidden"]
    qkv = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    shapes = [(qkv, d), (d, c["n_heads"] * c["head_dim"]), (2 * F, d), (d, F)]
    qs = [oracle.quantize_int8(r.standard_normal(s, dtype=np.float32) * 0.02) for s in shapes]
    t0 = time.perf_counter()
    for (q, s), (n, k) in zip(qs, shapes):
        oracle.int8_linear(oracle.round_bf16(r.standard_normal((1, k), dtype=np.float32)), q, s)
    kq = oracle.round_bf16(r.standard_normal((1, c["n_heads"], 1, c["head_dim"]), dtype=np.float32))
    kk = oracle.round_bf16(r.standard_normal((1, c["n_kv_heads"], c["ctx"], c["head_dim"]), dtype=np.float32))
    oracle.attention(kq, kk, kk, 0.125, True)
    t = time.perf_counter() - t0
    bytes_layer = sum(n * k + 4 * n for n, k in shapes) + 2 * c["n_kv_heads"] * c["ctx"] * c["head_dim"] * 2
    return {"value": bytes_layer / t / 1e9, "unit": "GB/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"oracle C port: one decoder layer's int8 GEMVs + decode attention for 1 of 64 sequences ({t:.2f}s)"}


# ----------------------------------------------------------------- C4 -------
def c4_bytes_flops():
    c = C4
    d, F, V = c["d_model"], c["ffn_hidden"], c["vocab"]
    qkv = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    shapes = {"qkv": (qkv, d), "o": (d, c["n_heads"] * c["head_dim"]), "gate_up": (2 * F, d), "down": (d, F)}
    layer_params = sum(n * k for n, k in shapes.values())
    return shapes, layer_params


def run_c4(args, rank, world, local):
    import numpy as np
    import torch
    from teenygrad_b200.decoder import Decoder, DecoderConfig
    from teenygrad_b200 import ops
    c = C4
    B, S, G = c["batch"], c["prompt"], c["gen"]
    cfg = DecoderConfig(n_layers=c["n_layers"], d_model=c["d_model"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                        head_dim=c["head_dim"], ffn_hidden=c["ffn_hidden"], vocab=c["vocab"], max_batch=B,
                        max_seq=S + G, max_prefill_tokens=B * S)
    dec = Decoder(cfg, device=local)
    dec.init_random(seed=1234, std=0.02)
    gen = torch.Generator(device="cpu").manual_seed(42 + rank)
    prompt_host = torch.randint(0, c["vocab"], (B, S), generator=gen, dtype=torch.int32).pin_memory()
    prompt = prompt_host.cuda()
    out = torch.empty(B, G, device="cuda", dtype=torch.int32)
    gathered = torch.empty(world * B, G, device="cuda", dtype=torch.int32)
    comm = None
    if world > 1:
        from teenygrad_b200.dist import Comm
        comm = Comm(rank, world, timeout_ms=60000, device=local)

    def step():
        dec.generate(prompt, G, out=out)
        if comm is not None:
            comm.all_gather(out, gathered)

    for _ in range(args.warmup):
        step()
    barrier(world)
    clk = Clocks(local) if rank == 0 else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    barrier(world)
    clocks = clk.stop() if clk else None
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    tokens = world * B * (S + G)
    value = tokens / (ms / 1e3)

    # ---- end to end through the public API with host buffers
    out_host = torch.empty(B, G, dtype=torch.int32).pin_memory()
    gathered_host = torch.empty(world * B, G, dtype=torch.int32).pin_memory()

    def e2e_step():
        p = prompt_host.cuda(non_blocking=True)
        o = dec.generate(p, G)
        if comm is not None:
            comm.all_gather(o, gathered)
            gathered_host.copy_(gathered, non_blocking=True)
        else:
            out_host.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step()
    barrier(world)
    t0 = time.perf_counter()
    ev0.record()
    for _ in range(args.steps):
        e2e_step()
    ev1.record()
    barrier(world)
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)

    # ---- phase split: prefill vs decode (CUDA events)
    ms_prefill = time_loop(lambda: dec.prefill(prompt), 2)
    dec.prefill(prompt)
    ms_decode = time_loop(lambda: dec.decode_step(), G - 1)

    # ---- dominant kernels, timed live on this stream:
    # decode GEMV: the 4 linear layers x 16 layers with distinct weights (1.9 GB,
    # larger than L2), replayed as one CUDA graph of 64 back-to-back launches;
    # prefill GEMM: the gate/up layer at 16384 tokens, CUDA events around launches.
    pk = peaks()
    shapes, layer_params = c4_bytes_flops()
    nl = c["n_layers"]
    wts = [{k: (torch.randn(n, kk, device="cuda") * 0.02).bfloat16() for k, (n, kk) in shapes.items()} for _ in range(nl)]
    xs = {k: torch.randn(B, kk, device="cuda").bfloat16() for k, (n, kk) in shapes.items()}

    def gemv_all():
        for L in wts:
            for k in shapes:
                ops.linear(xs[k], L[k], swiglu=(k == "gate_up"))

    gemv_ms = graph_time(gemv_all, iters=10)
    gemv_bytes = nl * sum(2 * n * kk + 2 * B * kk + 2 * B * (n // 2 if k == "gate_up" else n)
                          for k, (n, kk) in shapes.items())
    gemv_gbs = gemv_bytes / (gemv_ms / 1e3) / 1e9
    xp = torch.randn(B * S, c["d_model"], device="cuda").bfloat16()
    n_gu = shapes["gate_up"][0]
    ops.linear(xp, wts[0]["gate_up"], swiglu=True)
    gemm_ms = time_loop(lambda: ops.linear(xp, wts[0]["gate_up"], swiglu=True), 10)
    gemm_tflops = 2 * B * S * n_gu * c["d_model"] / (gemm_ms / 1e3) / 1e12
    del wts
    dom_decode = ms_decode * (G - 1) >= ms_prefill
    if dom_decode:
        # DRAM traffic per launch: the ncu capture of the gate/up GEMV (profiles/gemv_tc_decode_gate_up.md:
        # 68.01 MB read + written for 67.4 MB of algorithmic bytes) scaled to the average launch of the step
        traffic = round(gemv_bytes / (4 * nl) * (68.01 / 67.4))
        roof = {"kernel": "gemv_tc_kernel (decode linear layers, bf16 weights, 16 tokens)", "bound": "hbm",
                "achieved": round(gemv_gbs, 1), "peak": pk["hbm"], "unit": "GB/s",
                "frac": round(gemv_gbs / pk["hbm"], 3), "traffic": traffic,
                "traffic_note": "bytes per average launch: ncu dram bytes / algorithmic bytes of the gate/up GEMV capture, times the average algorithmic bytes",
                "peak_source": pk["src"]}
    else:
        roof = {"kernel": "gemm_tc_kernel (prefill gate/up, 16384x16384x2048)", "bound": "tensor",
                "achieved": round(gemm_tflops, 1), "peak": pk["tc"], "unit": "TFLOP/s",
                "frac": round(gemm_tflops / pk["tc"], 3), "traffic": None, "peak_source": pk["src"]}
    secondary = {"prefill_gemm_gate_up_tflops": round(gemm_tflops, 1),
                 "prefill_gemm_frac_of_peak": round(gemm_tflops / pk["tc"], 3),
                 "decode_gemv_gbs": round(gemv_gbs, 1), "decode_gemv_frac_of_hbm": round(gemv_gbs / pk["hbm"], 3),
                 "decode_gemv_ms_per_step": round(gemv_ms, 4)}
    if comm is not None:
        comm.close()
    # prefill: set_state, embedding, per layer (rmsnorm, QKV GEMM, rope_kv, attention,
    # O GEMM, rmsnorm, gate/up GEMM, down GEMM), LM-head GEMV (norm fused), argmax, advance.
    # decode: embedding, per layer (QKV GEMV with norm + RoPE + KV-cache write fused,
    # attention, O GEMV, gate/up GEMV with norm fused, down GEMV), LM head, argmax, advance.
    launches_prefill = 2 + 8 * c["n_layers"] + 3
    launches_decode = 1 + 5 * c["n_layers"] + 3
    launches = launches_prefill + (G - 1) * launches_decode
    res = {
        "metric": "tokens/s (1B decoder)", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform-random ids, N(0,0.02) random-init weights)",
        "config": {"workload": "C4: Llama-style 1B decoder, batch 16 x 1024-token prompts + 128 greedy tokens per GPU",
                   "model": "llama-1b (16L, d2048, 32q/8kv x 64, SwiGLU 8192, vocab 32000)", "global_batch": world * B,
                   "seq_len": S, "gen_tokens": G, "parallelism": f"dp{world} (batch-sharded; generated ids all-gathered with the library's NCCL communicator)",
                   "tokens_counted": "prompt + generated tokens of all sequences",
                   "l2": "inputs larger than L2 (2.2 GB of weights streamed per step)",
                   "prefill_ms": round(ms_prefill, 3), "decode_ms_per_token": round(ms_decode, 4),
                   "prefill_tokens_per_s": round(B * S / (ms_prefill / 1e3), 1),
                   "decode_tokens_per_s": round(B / (ms_decode / 1e3), 1), **secondary},
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": B * S * 4,
                "d2h_bytes_per_step": (world * B if world > 1 else B) * G * 4},
        "gpu_launches": launches * args.steps,
        "roofline": roof,
        "clocks": clocks,
    }
    return res


def run_c5(args, rank, world, local):
    import torch
    from teenygrad_b200.decoder import Decoder, DecoderConfig
    c = C5
    B = c["batch"]
    cfg = DecoderConfig(n_layers=c["n_layers"], d_model=c["d_model"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                        head_dim=c["head_dim"], ffn_hidden=c["ffn_hidden"], vocab=c["vocab"], max_batch=B,
                        max_seq=c["ctx"] + 64, max_prefill_tokens=B, weights_int8=True)
    dec = Decoder(cfg, device=local)
    dec.init_random(seed=7)
    ids = torch.randint(0, c["vocab"], (B,), dtype=torch.int32, device="cuda")
    steps = min(args.steps * 8, 60)
    dec.fill_kv_random(ids, c["ctx"], seed=5)
    for _ in range(args.warmup):
        dec.decode_step()
    dec.fill_kv_random(ids, c["ctx"], seed=5)
    barrier(world)
    clk = Clocks(local) if rank == 0 else None
    ms = time_loop(lambda: dec.decode_step(), steps)
    clocks = clk.stop() if clk else None
    ms = max_over_ranks(ms, world)
    d, F, V = c["d_model"], c["ffn_hidden"], c["vocab"]
    qkv = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    w_bytes = c["n_layers"] * (qkv * d + d * c["n_heads"] * c["head_dim"] + 2 * F * d + d * F) + V * d
    s_bytes = 4 * (c["n_layers"] * (qkv + d + 2 * F + d) + V)
    ctx_mean = c["ctx"] + steps / 2
    kv_bytes = c["n_layers"] * B * c["n_kv_heads"] * ctx_mean * c["head_dim"] * 2 * 2
    step_bytes = w_bytes + s_bytes + kv_bytes
    pk = peaks()
    gbs = world * step_bytes / (ms / 1e3) / 1e9
    return {"metric": "HBM GB/s (int8 weight-only decode, 1B decoder)", "value": round(gbs, 1), "unit": "GB/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x bf16",
            "data": "synthetic", "config": {"workload": "C5: int8 weight-only decode, batch 64, KV 2048 pre-filled N(0,1)",
                                            "tokens_per_s": round(world * B / (ms / 1e3), 1),
                                            "bytes_per_step": int(step_bytes)},
            "roofline": {"bound": "hbm", "achieved": round(gbs / world, 1), "peak": pk["hbm"], "unit": "GB/s",
                         "frac": round(gbs / world / pk["hbm"], 3), "traffic": None, "peak_source": pk["src"]},
            "clocks": clocks}


def run_c3(args, rank, world, local):
    import torch
    from teenygrad_b200 import ops
    c = C3
    B, H, S, D = c["B"], c["H"], c["S"], c["D"]
    q = torch.randn(B, H, S, D, device="cuda").bfloat16()
    k = torch.randn(B, H, S, D, device="cuda").bfloat16()
    v = torch.randn(B, H, S, D, device="cuda").bfloat16()
    for _ in range(args.warmup):
        ops.attention(q, k, v, causal=True, return_lse=True)
    barrier(world)
    clk = Clocks(local) if rank == 0 else None
    ms = time_loop(lambda: ops.attention(q, k, v, causal=True, return_lse=True), args.steps)
    clocks = clk.stop() if clk else None
    ms = max_over_ranks(ms, world)
    flops = 4 * B * H * D * S * (S + 1) / 2
    tf = flops / (ms / 1e3) / 1e12
    pk = peaks()
    return {"metric": "TFLOP/s (causal flash-attention prefill bf16)", "value": round(world * tf, 1), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C3: B8 H32 S4096 D128 causal, O + LSE"},
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": pk["tc"], "unit": "TFLOP/s",
                         "frac": round(tf / pk["tc"], 3), "traffic": None, "peak_source": pk["src"]},
            "clocks": clocks}


def run_c2(args, rank, world, local):
    """4 x (3x3 conv 64->64, pad 1 + bias + folded BN + ReLU), NCHW, batch 32, 56x56."""
    import torch
    from teenygrad_b200 import ops
    c = C2
    B, C, H, W = c["B"], c["C"], c["H"], c["W"]
    g = torch.Generator(device="cpu").manual_seed(0)
    res = {}
    pk = peaks()
    flops_conv = 2 * B * C * H * W * C * 9
    for dt in (torch.bfloat16, torch.float32):
        x = torch.randn(B, C, H, W, generator=g).to("cuda", dt)
        layers = []
        for _ in range(c["layers"]):
            w = (torch.randn(C, C, 3, 3, generator=g) * math.sqrt(2.0 / (C * 9))).to("cuda", dt)
            bias = (torch.randn(C, generator=g) * 0.1).cuda()
            gam, bet = (torch.rand(C, generator=g) + 0.5).cuda(), (torch.randn(C, generator=g) * 0.1).cuda()
            mu, var = (torch.randn(C, generator=g) * 0.1).cuda(), (torch.rand(C, generator=g) + 0.5).cuda()
            sc, sh = ops.bn_fold(gam, bet, mu, var, 1e-5, bias)
            layers.append((w, sc, sh))

        def stage():
            y = x
            for w, sc, sh in layers:
                y = ops.conv2d(y, w, scale=sc, shift=sh, pad=1, act="relu")
            return y

        for _ in range(args.warmup):
            stage()
        # CUDA-graph replays of the stage (and of one conv) with L2 flushed before each
        ms = graph_time_flushed(stage, max(args.steps, 3))
        ms_conv = graph_time_flushed(
            lambda: ops.conv2d(x, layers[0][0], scale=layers[0][1], shift=layers[0][2], pad=1, act="relu"), 5)
        res[str(dt).split(".")[1]] = (ms, ms_conv)
    ms_bf16, conv_bf16 = res["bfloat16"]
    ms_f32, conv_f32 = res["float32"]
    tf = flops_conv / (conv_bf16 / 1e3) / 1e12
    return {"metric": "images/s (ResNet-style conv stage, 4 x conv3x3 + bias + BN + ReLU)", "value": round(world * B / (ms_bf16 / 1e3), 1),
            "unit": "images/s", "n_gpus": world, "steps": max(args.steps, 3), "warmup": args.warmup, "ms_per_step": round(ms_bf16, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C2: 4 x 3x3 conv 64->64 + bias + folded BN + ReLU, B32 56x56 NCHW",
                       "timing": "CUDA graph replays, L2 flushed (256 MB write) before each", "l2": "flushed",
                       "fp32_ms_per_step": round(ms_f32, 3), "fp32_images_per_s": round(B / (ms_f32 / 1e3), 1),
                       "bf16_conv_ms": round(conv_bf16, 4), "fp32_conv_ms": round(conv_f32, 4),
                       "fp32_conv_tflops": round(flops_conv / (conv_f32 / 1e3) / 1e12, 1)},
            "roofline": {"kernel": "conv_tc_kernel (+ NHWC transpose), one conv", "bound": "tensor", "achieved": round(tf, 1),
                         "peak": pk["tc"], "unit": "TFLOP/s", "frac": round(tf / pk["tc"], 3), "traffic": None,
                         "peak_source": pk["src"]}}


def run_c1(args, rank, world, local):
    import torch
    from teenygrad_b200.block import block_forward, random_block_params
    c = C1
    p = random_block_params(d=c["d"], F=c["ffn"], seed=0)
    x = torch.randn(c["B"], c["S"], c["d"], device="cuda")
    for _ in range(args.warmup):
        block_forward(x, p, c["heads"])
    us = graph_time(lambda: block_forward(x, p, c["heads"]), iters=50) * 1e3
    return {"metric": "us per block (fp32 pre-norm transformer block)", "value": round(us, 2), "unit": "us",
            "n_gpus": world, "steps": 50, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C1: B1 S128 d256 4x64 heads, causal SDPA, RMSNorm 1e-6, SwiGLU 1024, fp32",
                       "timing": "CUDA graph of one block forward (latency-bound: 9 library kernels + 4 torch layout copies)"}}


def ncu_case(which):
    """Small fixed cases for ncu captures of one kernel kind (the commands in profiles/):
    gemv, gemv8, attn_dec, gemm, fa, conv, or c4 (prefill + 3 decode steps for the launch list)."""
    import torch
    from teenygrad_b200 import ops
    torch.manual_seed(0)
    if which == "gemv":          # decode gate/up GEMV (SwiGLU), 16 tokens, 3 distinct weights
        ws = [(torch.randn(16384, 2048, device="cuda") * 0.02).bfloat16() for _ in range(3)]
        x = torch.randn(16, 2048, device="cuda").bfloat16()
        for w in ws:
            ops.linear(x, w, swiglu=True)
    elif which == "gemv8":       # C5 decode gate/up GEMV: 64 tokens, int8 weights (4 distinct, 134 MB)
        qs = [ops.quantize_int8((torch.randn(16384, 2048, device="cuda") * 0.02)) for _ in range(4)]
        x = torch.randn(64, 2048, device="cuda").bfloat16()
        for q, s in qs:
            ops.int8_linear(x, q, s, swiglu=True)
    elif which == "attn_dec":    # C4 decode attention layer: 16 seqs x 8 kv heads x 1100 keys, G = 4
        q = torch.randn(16, 32, 1, 64, device="cuda").bfloat16()
        k = torch.randn(16, 8, 1100, 64, device="cuda").bfloat16()
        v = torch.randn(16, 8, 1100, 64, device="cuda").bfloat16()
        for _ in range(3):
            ops.attention(q, k, v, causal=True)
    elif which == "gemm":        # C4 prefill gate/up GEMM 16384 x 16384 x 2048 with SwiGLU
        w = (torch.randn(16384, 2048, device="cuda") * 0.02).bfloat16()
        x = torch.randn(16384, 2048, device="cuda").bfloat16()
        for _ in range(2):
            ops.linear(x, w, swiglu=True)
    elif which == "fa":          # a quarter of C3: B2 H32 S4096 D128 causal (1024 CTAs)
        q, k, v = (torch.randn(2, 32, 4096, 128, device="cuda").bfloat16() for _ in range(3))
        for _ in range(2):
            ops.attention(q, k, v, causal=True)
    elif which == "conv":        # one C2 conv: B32 64->64 56x56 3x3 + BN + ReLU
        x = torch.randn(32, 64, 56, 56, device="cuda").bfloat16()
        w = (torch.randn(64, 64, 3, 3, device="cuda") * 0.05).bfloat16()
        sc, sh = torch.ones(64, device="cuda"), torch.zeros(64, device="cuda")
        for _ in range(2):
            ops.conv2d(x, w, scale=sc, shift=sh, pad=1, act="relu")
    elif which == "c4":          # C4 decoder: prefill 16 x 1024 + 3 graph-replayed decode steps
        from teenygrad_b200.decoder import Decoder, DecoderConfig
        dec = Decoder(DecoderConfig(max_batch=16, max_seq=1024 + 128, max_prefill_tokens=16 * 1024))
        dec.init_random(1)
        dec.prefill(torch.randint(0, 32000, (16, 1024), dtype=torch.int32, device="cuda"))
        for _ in range(3):
            dec.decode_step()
    else:
        raise SystemExit(f"unknown ncu case {which}")
    torch.cuda.synchronize()
    print("ok", which)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c4", choices=["c4", "c5", "c3", "c2", "c1"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-case", default=None, help="run one small profiling case and exit")
    args = ap.parse_args()
    if args.ncu_case:
        ncu_case(args.ncu_case)
        return
    rank = int(os.environ.get("RANK", "0"))
    world_env = int(os.environ.get("WORLD_SIZE", "1"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        cb = cpu_baseline_c5() if args.workload == "c5" else cpu_baseline_c4()
        metric = {"c4": "tokens/s (1B decoder)", "c5": "HBM GB/s (int8 weight-only decode, 1B decoder)",
                  "c3": "tokens/s (1B decoder)"}[args.workload]
        print(json.dumps({"impl": "reference", "metric": metric, "value": cb["value"], "unit": cb["unit"],
                          "n_gpus": args.gpus, "steps": 1, "warmup": 0, "higher_is_better": True,
                          "config": {"workload": args.workload.upper()}, "cpu_baseline": cb,
                          "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return 0

    rank, world, local = dist_setup(max(args.gpus, world_env))
    run = {"c4": run_c4, "c5": run_c5, "c3": run_c3, "c2": run_c2, "c1": run_c1}[args.workload]
    res = run(args, rank, world, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in ("c4", "c5"):
        res["cpu_baseline"] = cpu_baseline_c5() if args.workload == "c5" else cpu_baseline_c4()
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
