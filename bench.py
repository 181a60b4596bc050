"""Benchmark of the teenygrad hot path on B200.

Default workload (BASELINE metric "tokens/s (1B decoder)"): the Llama-style
1B decoder (16 layers, d 2048, 32/8 heads x 64, SwiGLU 8192, vocab 32000,
bf16, N(0, 0.02) random init), a global batch of 16 prompts of 1024
uniform-random ids, prefill + 128 greedy tokens.  One step = that whole
generation.  Multi-GPU: one process per GPU, the 16 sequences sharded by
batch (16 / N per GPU, strong scaling, the headline), the generated ids
all-gathered over NCCL at the end of every step; the same run with 16
sequences per GPU (weak scaling) is reported beside it.  At N = 1 the line
also carries the C3 (flash attention), C5 (int8 decode) and C2 (conv stage)
figures, each with its own clock record.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c4|c5|c3|c2|c1]

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
CONV_REPS = 12   # launches per graph replay when one C2 convolution is timed
C1 = dict(B=1, S=128, d=256, heads=4, ffn=1024)
# DRAM bytes (read + written) per algorithmic byte of the decode GEMV, from an ncu
# capture of the gate/up launch (bench.py --ncu-case gemv): 68.18 MB for 67.37 MB
GEMV_TRAFFIC_RATIO = 1.012


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


def cpu_baseline_c3():
    """Oracle causal attention on 1 of the 256 (batch, head) pairs of C3, TFLOP/s."""
    import numpy as np
    import oracle
    c = C3
    r = np.random.default_rng(0)
    q, k, v = (oracle.round_bf16(r.standard_normal((1, 1, c["S"], c["D"]), dtype=np.float32)) for _ in range(3))
    t0 = time.perf_counter()
    oracle.attention(q, k, v, 1.0 / math.sqrt(c["D"]), True)
    t = time.perf_counter() - t0
    fl = 4 * c["D"] * c["S"] * (c["S"] + 1) / 2
    return {"value": fl / t / 1e12, "unit": "TFLOP/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"oracle C port: 1 of 256 (batch, head) pairs, S 4096 D 128 causal ({t:.2f}s)"}


def cpu_baseline_c2():
    """Oracle conv + folded BN + ReLU on 1 of the 32 images, one of the 4 convs; images/s."""
    import numpy as np
    import oracle
    c = C2
    r = np.random.default_rng(0)
    x = r.standard_normal((1, c["C"], c["H"], c["W"]), dtype=np.float32)
    w = (r.standard_normal((c["C"], c["C"], 3, 3), dtype=np.float32) * math.sqrt(2.0 / (c["C"] * 9))).astype(np.float32)
    sc, sh = np.ones(c["C"], np.float32), np.zeros(c["C"], np.float32)
    t0 = time.perf_counter()
    oracle.conv2d(x, w, scale=sc, shift=sh, pad=1, act="relu")
    t = (time.perf_counter() - t0) * c["layers"]
    return {"value": 1.0 / t, "unit": "images/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"oracle C port (f32): 1 image x 1 conv, times 4 convs ({t:.3f}s per image)"}


def cpu_baseline_c1():
    """Oracle fp32 pre-norm block (the whole C1 workload), us per block."""
    import numpy as np
    import oracle  # noqa: F401
    from oracle.decoder import block_forward
    c = C1
    r = np.random.default_rng(0)
    d, F = c["d"], c["ffn"]
    p = {n: (r.standard_normal(sh, dtype=np.float32) * 0.02).astype(np.float32)
         for n, sh in (("wq", (d, d)), ("wk", (d, d)), ("wv", (d, d)), ("wo", (d, d)), ("w_gate", (F, d)),
                       ("w_up", (F, d)), ("w_down", (d, F)))}
    p["attn_norm"], p["mlp_norm"] = np.ones(d, np.float32), np.ones(d, np.float32)
    x = r.standard_normal((c["B"], c["S"], d), dtype=np.float32)
    block_forward(x, p, c["heads"])
    t0 = time.perf_counter()
    n = 10
    for _ in range(n):
        block_forward(x, p, c["heads"])
    t = (time.perf_counter() - t0) / n
    return {"value": t * 1e6, "unit": "us", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"oracle C port: the whole C1 block, mean of {n}"}


# ----------------------------------------------------------------- C4 -------
def c4_bytes_flops():
    c = C4
    d, F, V = c["d_model"], c["ffn_hidden"], c["vocab"]
    qkv = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    shapes = {"qkv": (qkv, d), "o": (d, c["n_heads"] * c["head_dim"]), "gate_up": (2 * F, d), "down": (d, F)}
    layer_params = sum(n * k for n, k in shapes.values())
    return shapes, layer_params


def _c4_decoder(B, local):
    from teenygrad_b200.decoder import Decoder, DecoderConfig
    c = C4
    S, G = c["prompt"], c["gen"]
    cfg = DecoderConfig(n_layers=c["n_layers"], d_model=c["d_model"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                        head_dim=c["head_dim"], ffn_hidden=c["ffn_hidden"], vocab=c["vocab"], max_batch=B,
                        max_seq=S + G, max_prefill_tokens=B * S)
    dec = Decoder(cfg, device=local)
    dec.init_random(seed=1234, std=0.02)
    return dec


def _c4_generation(args, dec, B, rank, world, comm, seed_base):
    """Times `steps` generations of B local sequences (+ the all-gather of the
    ids): device-resident prompts, then end to end from pinned host memory.
    Returns ms per step (max over ranks), e2e ms, this rank's ms, prefill ms,
    all-gather ms and the gathered ids of the last step."""
    import torch
    c = C4
    S, G = c["prompt"], c["gen"]
    gen = torch.Generator(device="cpu").manual_seed(seed_base + rank)
    prompt_host = torch.randint(0, c["vocab"], (B, S), generator=gen, dtype=torch.int32).pin_memory()
    prompt = prompt_host.cuda()
    out = torch.empty(B, G, device="cuda", dtype=torch.int32)
    gathered = torch.empty(world * B, G, device="cuda", dtype=torch.int32)

    def step():
        dec.generate(prompt, G, out=out)
        if comm is not None:
            comm.all_gather(out, gathered)

    for _ in range(args.warmup):
        step()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    barrier(world)
    my_ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(my_ms, world)

    # end to end through the public API with host buffers
    gathered_host = torch.empty(world * B, G, dtype=torch.int32).pin_memory()

    def e2e_step():
        p = prompt_host.cuda(non_blocking=True)
        o = dec.generate(p, G)
        if comm is not None:
            comm.all_gather(o, gathered)
            gathered_host.copy_(gathered, non_blocking=True)
        else:
            gathered_host.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step()
    barrier(world)
    ev0.record()
    for _ in range(args.steps):
        e2e_step()
    ev1.record()
    barrier(world)
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)

    # phase split (CUDA events): prefill alone; the all-gather alone
    ms_prefill = max_over_ranks(time_loop(lambda: dec.prefill(prompt), 3), world)
    ms_ag = 0.0
    if comm is not None:
        barrier(world)
        ms_ag = max_over_ranks(time_loop(lambda: comm.all_gather(out, gathered), 20), world)
    return ms, e2e_ms, my_ms, ms_prefill, ms_ag, gathered, out


def run_c4(args, rank, world, local):
    import torch
    from teenygrad_b200 import ops
    from teenygrad_b200.dist import shard
    c = C4
    Bg, S, G = c["batch"], c["prompt"], c["gen"]
    # strong scaling (the config): the global batch of 16 sharded over the ranks
    start, B = shard(Bg, world, rank)
    assert Bg % world == 0, "the all-gather needs equal shards (N must divide 16)"
    comm = None
    if world > 1:
        from teenygrad_b200.dist import Comm
        comm = Comm(rank, world, timeout_ms=60000, device=local)
    dec = _c4_decoder(B, local)
    clk = Clocks(local) if rank == 0 else None
    ms, e2e_ms, my_ms, ms_prefill, ms_ag, gathered, out = _c4_generation(args, dec, B, rank, world, comm, 42)
    clocks = clk.stop() if clk else None
    per_rank = [my_ms]
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([my_ms], device="cuda", dtype=torch.float64)
        allt = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        per_rank = [round(float(x.item()), 3) for x in allt]
    per_rank = [round(x, 3) for x in per_rank]
    # the gathered ids: this rank's block is its own generation, and every rank
    # holds the same gathered array (checksum min == max over ranks)
    ids_ok = True
    if comm is not None:
        import torch.distributed as dist
        torch.cuda.synchronize()
        ids_ok = bool(torch.equal(gathered[rank * B:(rank + 1) * B], out))
        ck = (gathered.long() * torch.arange(1, gathered.numel() + 1, device="cuda").view_as(gathered)).sum()
        lo, hi = ck.clone(), ck.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        ok_t = torch.tensor([int(ids_ok and bool(lo == hi))], device="cuda")
        dist.all_reduce(ok_t, op=dist.ReduceOp.MIN)
        ids_ok = bool(ok_t.item())
    tokens = Bg * (S + G)
    value = tokens / (ms / 1e3)
    decode_ms = (ms - ms_prefill - ms_ag) / (G - 1)

    # weak scaling (16 sequences per GPU) beside it, for N > 1
    weak = None
    if world > 1:
        del dec
        torch.cuda.empty_cache()
        dec_w = _c4_decoder(Bg, local)
        wms = _c4_generation(args, dec_w, Bg, rank, world, comm, 4242)[0]
        weak = {"tokens_per_s": round(world * Bg * (S + G) / (wms / 1e3), 1), "ms_per_step": round(wms, 3),
                "sequences_per_gpu": Bg}
        del dec_w
        torch.cuda.empty_cache()
    else:
        del dec

    # ---- dominant kernels, timed live on this stream:
    # decode GEMV: the 4 linear layers x 16 layers with distinct weights (1.9 GB,
    # larger than L2), replayed as one CUDA graph of 64 back-to-back launches;
    # prefill GEMM: the gate/up layer at 16384 tokens, CUDA events around launches.
    pk = peaks()
    shapes, layer_params = c4_bytes_flops()
    nl = c["n_layers"]
    wts = [{k: (torch.randn(n, kk, device="cuda") * 0.02).bfloat16() for k, (n, kk) in shapes.items()} for _ in range(nl)]
    xs = {k: torch.randn(Bg, kk, device="cuda").bfloat16() for k, (n, kk) in shapes.items()}

    def gemv_all():
        for L in wts:
            for k in shapes:
                ops.linear(xs[k], L[k], swiglu=(k == "gate_up"))

    gemv_ms = graph_time(gemv_all, iters=10)
    gemv_bytes = nl * sum(2 * n * kk + 2 * Bg * kk + 2 * Bg * (n // 2 if k == "gate_up" else n)
                          for k, (n, kk) in shapes.items())
    gemv_gbs = gemv_bytes / (gemv_ms / 1e3) / 1e9
    xp = torch.randn(Bg * S, c["d_model"], device="cuda").bfloat16()
    n_gu = shapes["gate_up"][0]
    ops.linear(xp, wts[0]["gate_up"], swiglu=True)
    gemm_ms = time_loop(lambda: ops.linear(xp, wts[0]["gate_up"], swiglu=True), 10)
    gemm_tflops = 2 * Bg * S * n_gu * c["d_model"] / (gemm_ms / 1e3) / 1e12
    del wts, xp
    torch.cuda.empty_cache()
    # DRAM bytes per launch from ncu captures of the same kernels (dram__bytes_read.sum +
    # dram__bytes_write.sum; commands: bench.py --ncu-case gemv / gemm under
    # ncu --set full -k regex:<kernel> -s 1 -c 1): the gate/up GEMV read+wrote 1.012x its
    # algorithmic bytes, scaled here to the average launch of the 64
    traffic = round(gemv_bytes / (4 * nl) * GEMV_TRAFFIC_RATIO)
    roof = {"kernel": "gemv_tc_kernel (decode linear layers, bf16 weights, 16 tokens)", "bound": "hbm",
            "achieved": round(gemv_gbs, 1), "peak": pk["hbm"], "unit": "GB/s",
            "frac": round(gemv_gbs / pk["hbm"], 3), "traffic": traffic,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the gate/up decode GEMV "
                              "(small case), per algorithmic byte, times the average launch's algorithmic bytes",
            "peak_source": pk["src"]}
    if comm is not None:
        comm.close()
    # prefill: set_state, embedding, per layer (rmsnorm, QKV GEMM with RoPE + KV-cache write
    # fused, attention, O GEMM, rmsnorm, gate/up GEMM, down GEMM), LM-head GEMV (norm fused),
    # argmax, advance.
    # decode: embedding, per layer (QKV GEMV with norm + RoPE + KV-cache write fused,
    # attention, O GEMV, gate/up GEMV with norm fused, down GEMV), LM head, argmax, advance.
    launches_prefill = 2 + 7 * c["n_layers"] + 3
    launches_decode = 1 + 5 * c["n_layers"] + 3
    launches = launches_prefill + (G - 1) * launches_decode
    cfg = {"workload": "C4: Llama-style 1B decoder, global batch 16 x 1024-token prompts + 128 greedy tokens, "
                       "batch-sharded over the GPUs",
           "model": "llama-1b (16L, d2048, 32q/8kv x 64, SwiGLU 8192, vocab 32000)", "global_batch": Bg,
           "sequences_per_gpu": B, "seq_len": S, "gen_tokens": G,
           "parallelism": f"dp{world} (batch-sharded; generated ids all-gathered with the library's NCCL communicator)",
           "tokens_counted": "prompt + generated tokens of all sequences",
           "l2": "inputs larger than L2 (2.2 GB of weights streamed per step)",
           "prefill_ms": round(ms_prefill, 3), "decode_ms_per_token": round(decode_ms, 4),
           "decode_ms_source": "(timed step - prefill - all-gather) / 127 graph-replayed decode steps",
           "prefill_tokens_per_s": round(Bg * S / (ms_prefill / 1e3), 1),
           "decode_tokens_per_s": round(Bg / (decode_ms / 1e3), 1),
           "per_rank_ms": per_rank, "allgather_ms": round(ms_ag, 4), "allgather_ids_checked": ids_ok,
           "prefill_gemm_gate_up_tflops": round(gemm_tflops, 1),
           "prefill_gemm_frac_of_peak": round(gemm_tflops / pk["tc"], 3),
           "decode_gemv_gbs": round(gemv_gbs, 1), "decode_gemv_frac_of_hbm": round(gemv_gbs / pk["hbm"], 3),
           "decode_gemv_ms_per_step": round(gemv_ms, 4)}
    if weak is not None:
        cfg["weak_scaling"] = weak
    res = {
        "metric": "tokens/s (1B decoder)", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random ids, N(0,0.02) random-init weights)", "config": cfg,
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": B * S * 4,
                "d2h_bytes_per_step": Bg * G * 4},
        "gpu_launches": launches * args.steps,
        "roofline": roof,
        "clocks": clocks,
    }
    return res


def run_c5(args, rank, world, local):
    import torch
    from teenygrad_b200.decoder import Decoder, DecoderConfig
    from teenygrad_b200.dist import shard
    c = C5
    B = shard(c["batch"], world, rank)[1]     # the batch of 64 sharded over the ranks
    cfg = DecoderConfig(n_layers=c["n_layers"], d_model=c["d_model"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                        head_dim=c["head_dim"], ffn_hidden=c["ffn_hidden"], vocab=c["vocab"], max_batch=B,
                        max_seq=c["ctx"] + 64, max_prefill_tokens=B, weights_int8=True)
    dec = Decoder(cfg, device=local)
    dec.init_random(seed=7)
    ids = torch.randint(0, c["vocab"], (B,), dtype=torch.int32, device="cuda")
    steps = min(args.steps * 8, 60)
    clk = Clocks(local) if rank == 0 else None
    dec.fill_kv_random(ids, c["ctx"], seed=5)
    for _ in range(args.warmup):
        dec.decode_step()
    # blocks of `steps` decode steps from a freshly filled cache (it holds ctx + 64
    # positions) until >= 0.6 s were timed, so the clock record samples them
    tot, n = 0.0, 0
    while tot < 600.0 or n < 1:
        dec.fill_kv_random(ids, c["ctx"], seed=5)
        barrier(world)
        tot += time_loop(lambda: dec.decode_step(), steps) * steps
        n += steps
    clocks = clk.stop() if clk else None
    ms = max_over_ranks(tot / n, world)
    d, F, V = c["d_model"], c["ffn_hidden"], c["vocab"]
    qkv = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    w_bytes = c["n_layers"] * (qkv * d + d * c["n_heads"] * c["head_dim"] + 2 * F * d + d * F) + V * d
    s_bytes = 4 * (c["n_layers"] * (qkv + d + 2 * F + d) + V)
    ctx_mean = c["ctx"] + steps / 2
    kv_bytes = c["n_layers"] * B * c["n_kv_heads"] * ctx_mean * c["head_dim"] * 2 * 2
    step_bytes = w_bytes + s_bytes + kv_bytes          # this rank's bytes per decode step
    pk = peaks()
    gbs = world * step_bytes / (ms / 1e3) / 1e9
    return {"metric": "HBM GB/s (int8 weight-only decode, 1B decoder)", "value": round(gbs, 1), "unit": "GB/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8 x bf16",
            "data": "synthetic", "config": {"workload": "C5: int8 weight-only decode, batch 64 (sharded over the GPUs), "
                                                        "KV 2048 pre-filled N(0,1)",
                                            "sequences_per_gpu": B,
                                            "tokens_per_s": round(c["batch"] / (ms / 1e3), 1),
                                            "bytes_per_step_per_gpu": int(step_bytes),
                                            "l2": "inputs larger than L2 (1.04 GB of int8 weights + 4.3 GB KV per step)"},
            "roofline": {"kernel": "decode step (int8 GEMVs + decode attention), bytes per step / step time",
                         "bound": "hbm", "achieved": round(gbs / world, 1), "peak": pk["hbm"], "unit": "GB/s",
                         "frac": round(gbs / world / pk["hbm"], 3), "traffic": None, "peak_source": pk["src"]},
            "clocks": clocks}


def run_c3(args, rank, world, local):
    import torch
    from teenygrad_b200 import ops
    from teenygrad_b200.dist import shard
    c = C3
    Bg, H, S, D = c["B"], c["H"], c["S"], c["D"]
    # the 256 (batch, head) pairs sharded over the ranks (heads are independent: no GQA in C3)
    npairs = shard(Bg * H, world, rank)[1]
    B = 1
    q = torch.randn(1, npairs, S, D, device="cuda").bfloat16()
    k = torch.randn(1, npairs, S, D, device="cuda").bfloat16()
    v = torch.randn(1, npairs, S, D, device="cuda").bfloat16()
    H = npairs
    clk = Clocks(local) if rank == 0 else None
    for _ in range(args.warmup):
        ops.attention(q, k, v, causal=True, return_lse=True)
    est = time_loop(lambda: ops.attention(q, k, v, causal=True, return_lse=True), 2)
    steps = max(args.steps, int(math.ceil(600.0 / max(est, 1e-3))))   # >= 0.6 s, so the clock record samples it
    barrier(world)
    ms = time_loop(lambda: ops.attention(q, k, v, causal=True, return_lse=True), steps)
    clocks = clk.stop() if clk else None
    ms = max_over_ranks(ms, world)
    flops = 4 * B * H * D * S * (S + 1) / 2            # this rank's share
    tf = flops / (ms / 1e3) / 1e12
    pk = peaks()
    return {"metric": "TFLOP/s (causal flash-attention prefill bf16)", "value": round(4 * Bg * c["H"] * D * S * (S + 1) / 2 / (ms / 1e3) / 1e12, 1),
            "unit": "TFLOP/s", "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C3: B8 H32 S4096 D128 causal, O + LSE; the 256 (batch, head) pairs sharded over the GPUs",
                       "pairs_per_gpu": H, "l2": "inputs larger than L2 (Q, K, V, O: 1.07 GB per GPU at N = 1)"},
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": pk["tc"], "unit": "TFLOP/s",
                         "frac": round(tf / pk["tc"], 3), "traffic": None, "peak_source": pk["src"]},
            "clocks": clocks}


def run_c2(args, rank, world, local):
    """4 x (3x3 conv 64->64, pad 1 + bias + folded BN + ReLU), NCHW, batch 32, 56x56."""
    import torch
    from teenygrad_b200 import ops
    from teenygrad_b200.dist import shard
    c = C2
    B, C, H, W = shard(c["B"], world, rank)[1], c["C"], c["H"], c["W"]   # the 32 images sharded over the ranks
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
            # bf16: weights packed once (as an executor does at load time)
            layers.append((ops.conv2d_pack_weights(w) if dt == torch.bfloat16 else w, sc, sh))

        def stage():
            # bf16: NCHW in and out, NHWC between the convolutions (no per-conv
            # transpose launch); f32: the CUDA-core NCHW path
            y = x
            n = len(layers)
            for i, (w, sc, sh) in enumerate(layers):
                if dt == torch.bfloat16:
                    y = ops.conv2d(y, w, scale=sc, shift=sh, pad=1, act="relu", x_nhwc=i > 0, y_nhwc=i < n - 1,
                                   w_packed=True)
                else:
                    y = ops.conv2d(y, w, scale=sc, shift=sh, pad=1, act="relu")
            return y

        clk = Clocks(local) if (rank == 0 and dt == torch.bfloat16) else None
        for _ in range(args.warmup):
            stage()
        # CUDA-graph replays of the stage (and of one conv) with L2 flushed before each;
        # the bf16 stage is replayed for >= 0.6 s so that the clock record samples it
        est = graph_time_flushed(stage, 3)
        iters = max(args.steps, 3) if dt != torch.bfloat16 else max(args.steps, int(math.ceil(600.0 / max(est + 0.1, 1e-3))))
        ms = graph_time_flushed(stage, iters)
        if clk:
            res["clocks"] = clk.stop()
        if dt == torch.bfloat16:
            # one inner convolution (NHWC in and out, packed weights): CONV_REPS launches
            # on distinct inputs and outputs (more bytes than L2 holds, so each launch
            # reads its input from HBM) in one graph; ms per launch = replay / CONV_REPS,
            # so the graph's own launch latency is not counted as one kernel's time
            xhs = [torch.randn(B, H, W, C, generator=g).to("cuda", dt) for _ in range(CONV_REPS)]
            ms_conv = graph_time_flushed(
                lambda: [ops.conv2d(xh, layers[1][0], scale=layers[1][1], shift=layers[1][2], pad=1, act="relu",
                                    x_nhwc=True, y_nhwc=True, w_packed=True) for xh in xhs], 5) / CONV_REPS
            del xhs
        else:
            ms_conv = graph_time_flushed(
                lambda: ops.conv2d(x, layers[0][0], scale=layers[0][1], shift=layers[0][2], pad=1, act="relu"), 5)
        res[str(dt).split(".")[1]] = (ms, ms_conv)
    ms_bf16, conv_bf16 = res["bfloat16"]
    ms_f32, conv_f32 = res["float32"]
    clocks = res.get("clocks")
    tf = flops_conv / (conv_bf16 / 1e3) / 1e12
    ms_bf16 = max_over_ranks(ms_bf16, world)
    return {"metric": "images/s (ResNet-style conv stage, 4 x conv3x3 + bias + BN + ReLU)", "value": round(c["B"] / (ms_bf16 / 1e3), 1),
            "unit": "images/s", "n_gpus": world, "steps": max(args.steps, 3), "warmup": args.warmup, "ms_per_step": round(ms_bf16, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C2: 4 x 3x3 conv 64->64 + bias + folded BN + ReLU, B32 56x56 NCHW (images sharded over the GPUs)",
                       "layout": "bf16: NCHW stage input and output, NHWC between the convolutions, weights packed once "
                                 "before timing; f32: NCHW throughout",
                       "images_per_gpu": B,
                       "timing": "CUDA graph replays, L2 flushed (256 MB write) before each", "l2": "flushed",
                       "fp32_ms_per_step": round(ms_f32, 3), "fp32_images_per_s": round(B / (ms_f32 / 1e3), 1),
                       "bf16_conv_ms": round(conv_bf16, 4), "fp32_conv_ms": round(conv_f32, 4),
                       "bf16_conv_timing": f"{CONV_REPS} launches on distinct NHWC inputs (more than L2) per graph "
                                           "replay, L2 flushed before each replay; ms per launch",
                       "fp32_conv_tflops": round(flops_conv / (conv_f32 / 1e3) / 1e12, 1)},
            "roofline": {"kernel": f"conv_pm_kernel, one inner conv (NHWC in and out), mean of {CONV_REPS} launches", "bound": "tensor", "achieved": round(tf, 1),
                         "peak": pk["tc"], "unit": "TFLOP/s", "frac": round(tf / pk["tc"], 3), "traffic": None,
                         "peak_source": pk["src"]},
            "clocks": clocks}


def run_c1(args, rank, world, local):
    import torch
    from teenygrad_b200.block import block_graph, random_block_params
    c = C1
    p = random_block_params(d=c["d"], F=c["ffn"], seed=0)
    x = torch.randn(c["B"], c["S"], c["d"], device="cuda")
    g = block_graph(p, c["B"], c["S"], c["heads"], 1e-6, capture=True)
    g.run(x)
    for _ in range(args.warmup):
        g.launch()
    us = time_loop(g.launch, 200) * 1e3
    return {"metric": "us per block (fp32 pre-norm transformer block)", "value": round(us, 2), "unit": "us",
            "n_gpus": world, "steps": 200, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C1: B1 S128 d256 4x64 heads, causal SDPA, RMSNorm 1e-6, SwiGLU 1024, fp32",
                       "timing": "the block compiled onto the library's graph executor (planned buffers, one CUDA "
                                 "graph of its native kernels), replays timed with CUDA events; latency-bound"}}


def ncu_case(which):
    """Small fixed cases for ncu captures of one kernel kind (the commands in profiles/):
    gemv, gemv8, attn_dec, gemm, fa, conv, conv32, c1, c4 (prefill + 3 decode steps for the launch list) or c5
    (the int8 decoder: KV fill + 2 decode steps)."""
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
    elif which == "conv":        # C2 convs: B32 64->64 56x56 3x3 + BN + ReLU; NCHW, then NHWC in and out
        x = torch.randn(32, 64, 56, 56, device="cuda").bfloat16()
        w = (torch.randn(64, 64, 3, 3, device="cuda") * 0.05).bfloat16()
        sc, sh = torch.ones(64, device="cuda"), torch.zeros(64, device="cuda")
        for _ in range(2):
            ops.conv2d(x, w, scale=sc, shift=sh, pad=1, act="relu")
        xh, wp = x.permute(0, 2, 3, 1).contiguous(), ops.conv2d_pack_weights(w)
        for _ in range(2):
            ops.conv2d(xh, wp, scale=sc, shift=sh, pad=1, act="relu", x_nhwc=True, y_nhwc=True, w_packed=True)
    elif which == "conv32":      # C2 fp32 conv: B32 64->64 56x56 3x3 + BN + ReLU, NCHW (conv3x3_f32_kernel)
        x = torch.randn(32, 64, 56, 56, device="cuda")
        w = torch.randn(64, 64, 3, 3, device="cuda") * 0.05
        sc, sh = torch.ones(64, device="cuda"), torch.zeros(64, device="cuda")
        for _ in range(2):
            ops.conv2d(x, w, scale=sc, shift=sh, pad=1, act="relu")
    elif which == "c1":          # C1 fp32 block on the graph executor: 3 replays
        from teenygrad_b200.block import block_graph, random_block_params
        c = C1
        g = block_graph(random_block_params(d=c["d"], F=c["ffn"], seed=0), c["B"], c["S"], c["heads"], 1e-6, capture=True)
        g.run(torch.randn(c["B"], c["S"], c["d"], device="cuda"))
        for _ in range(3):
            g.launch()
    elif which == "c5":          # C5 int8 decoder: batch 64 over a 2048-position cache, 2 decode steps
        from teenygrad_b200.decoder import Decoder, DecoderConfig
        c = C5
        dec = Decoder(DecoderConfig(max_batch=c["batch"], max_seq=c["ctx"] + 64, max_prefill_tokens=c["batch"],
                                    weights_int8=True))
        dec.init_random(7)
        dec.fill_kv_random(torch.randint(0, c["vocab"], (c["batch"],), dtype=torch.int32, device="cuda"), c["ctx"], seed=5)
        for _ in range(2):
            dec.decode_step()
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


def secondary_n1(args, local):
    """C3, C5 and C2 at N = 1, each timed with its own clock record, for the
    default (C4) line."""
    import torch
    a = argparse.Namespace(steps=max(3, min(args.steps, 10)), warmup=3)
    out = {}
    for name, fn in (("c3", run_c3), ("c5", run_c5), ("c2", run_c2)):
        r = fn(a, 0, 1, local)
        out[name] = {"metric": r["metric"], "value": r["value"], "unit": r["unit"], "ms_per_step": r["ms_per_step"],
                     "workload": r["config"]["workload"], "roofline": r["roofline"], "clocks": r.get("clocks")}
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c4", choices=["c4", "c5", "c3", "c2", "c1"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="C4 at N = 1: skip the C3 / C5 / C2 fields")
    ap.add_argument("--ncu-case", default=None, help="run one small profiling case and exit")
    args = ap.parse_args()
    if args.ncu_case:
        ncu_case(args.ncu_case)
        return
    rank = int(os.environ.get("RANK", "0"))
    world_env = int(os.environ.get("WORLD_SIZE", "1"))

    baselines = {"c4": cpu_baseline_c4, "c5": cpu_baseline_c5, "c3": cpu_baseline_c3, "c2": cpu_baseline_c2,
                 "c1": cpu_baseline_c1}
    if args.impl == "reference":
        if rank != 0:
            return 0
        import oracle
        oracle.set_num_threads(len(os.sched_getaffinity(0)))   # every host core this process may use
        cb = baselines[args.workload]()
        metric = {"c4": "tokens/s (1B decoder)", "c5": "HBM GB/s (int8 weight-only decode, 1B decoder)",
                  "c3": "TFLOP/s (causal flash-attention prefill bf16)",
                  "c2": "images/s (ResNet-style conv stage, 4 x conv3x3 + bias + BN + ReLU)",
                  "c1": "us per block (fp32 pre-norm transformer block)"}[args.workload]
        print(json.dumps({"impl": "reference", "metric": metric, "value": cb["value"], "unit": cb["unit"],
                          "n_gpus": args.gpus, "steps": 1, "warmup": 0, "higher_is_better": args.workload != "c1",
                          "config": {"workload": args.workload.upper()}, "cpu_baseline": cb,
                          "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return 0

    rank, world, local = dist_setup(max(args.gpus, world_env))
    run = {"c4": run_c4, "c5": run_c5, "c3": run_c3, "c2": run_c2, "c1": run_c1}[args.workload]
    res = run(args, rank, world, local)
    if world == 1 and args.workload == "c4" and not args.no_secondary:
        res["secondary_workloads"] = secondary_n1(args, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        oracle.set_num_threads(len(os.sched_getaffinity(0)))
        res["cpu_baseline"] = baselines[args.workload]()
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
