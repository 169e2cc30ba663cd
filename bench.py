"""Benchmark: GPT-OSS-20B-shaped MXFP4 greedy decode (bs1) on B200, one JSON line on stdout.

Workload: 24-layer GPT-OSS-20B-shaped random-init model (MXFP4 experts,
Q8_0 attention, f16 embedding / LM head, seeded synthetic weights), a 2048-token prompt of
uniform random ids, then greedy decode.  One step = one decode token through all 24 layers
and the LM head.  Every step streams ~3.1 GB of weights (> 126 MB L2), so no L2 flush is
needed between steps.

  value     device-resident greedy decode (token fed back on the device), CUDA events
  e2e       the same decode through the public C ABI with host buffers per step
            (ms_model_decode_step: 4-byte token H2D, 8-byte argmax D2H)
  roofline  the fused MXFP4 expert FFN (gate/up + down) at the config-0 shape, events
  cpu_baseline  C++ restatement of the reference CPU path (oracle/), bounded sample

--impl reference times that CPU restatement alone (the Rust reference does not build here).
Under torchrun (N > 1) the default --mode ep splits the experts evenly over the ranks and all
ranks decode one sequence together (NCCL all-reduce of each layer's MoE output, "strong"
scaling); --mode replicas runs one independent sequence per rank ("weak" scaling, value summed).
Times are the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (bs1, bs32) + expert-matvec HBM GB/s vs peak at 1/2/4/8 B200"
PROMPT = 2048
# config 0 algorithmic bytes per token-layer: 4 experts x (3 x 4,406,400 B MXFP4 + 3 x 11,520 B f32 bias)
MOE_BYTES = 4 * (3 * 4_406_400 + 3 * 11_520)


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # the sampler is running (its first line written) before the timed region starts
        self._wait_lines(1, 5.0)
        return self

    def _lines(self):
        try:
            with open(self.path) as f:
                return sum(1 for _ in f)
        except OSError:
            return 0

    def _wait_lines(self, n, limit_s):
        t0 = time.time()
        while self.proc and self.proc.poll() is None and self._lines() < n and time.time() - t0 < limit_s:
            time.sleep(0.005)

    def __exit__(self, *exc):
        if self.proc:
            # at least one sample taken after the region's start (short regions end within 20 ms)
            self._wait_lines(self._lines() + 1, 1.0)
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------------------
def cpu_sample(steps: int, warmup: int, threads: int):
    """Oracle (C++ restatement of the reference CPU path) on a bounded sample of the workload:
    a 2-layer model with GPT-OSS-20B layer shapes and the full 201,088 x 2880 f16 LM head,
    8-token prompt, then `steps` timed decode tokens.  Per-token time for 24 layers is
    extrapolated as head + 24 x (per-layer time), the per-layer time taken from the 2-layer
    run minus a separately timed LM-head GEMV of the same model."""
    from dataclasses import replace

    from moe_stream_b200 import synth
    from oracle import oracle

    spec = replace(synth.GPT_OSS_20B, layers=2)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "sample.gguf")
        synth.write_model(path, spec, seed=0)
        m = oracle.Model(path, max_seq_len=64, threads=threads)
        prompt = synth.prompt_ids(spec, 8, seed=0)
        m.forward(prompt)
        tok = int(prompt[-1])
        for _ in range(warmup):
            tok = int(np.argmax(m.forward([tok])))
        t0 = time.perf_counter()
        for _ in range(steps):
            tok = int(np.argmax(m.forward([tok])))
        t2 = (time.perf_counter() - t0) / steps
        hid = m.last_hidden()
        m.lm_head(hid)
        t0 = time.perf_counter()
        m.lm_head(hid)
        th = time.perf_counter() - t0
        m.close()
    per_layer = max(t2 - th, 1e-6) / 2
    t24 = th + 24 * per_layer
    return {"tok_s": 1.0 / t24, "s_per_token_24L": t24, "s_per_token_2L": t2, "head_s": th,
            "sample": f"oracle decode of a 2-layer GPT-OSS-20B-shaped model with the full LM head "
                      f"({steps} timed tokens after an 8-token prompt, f32 KV), extrapolated to 24 layers"}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    r = cpu_sample(max(1, args.steps_ref), max(0, min(args.warmup, 1)), threads)
    line = {"metric": METRIC, "value": round(r["tok_s"], 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps_ref, "warmup": min(args.warmup, 1), "ms_per_step": round(1000 * r["s_per_token_24L"], 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic (seeded random-init GGUF)",
            "config": {"workload": "GPT-OSS-20B-shaped MXFP4 greedy decode, bs1", "prompt": PROMPT,
                       "note": "reference Rust binary unavailable (no cargo/crates offline); "
                               "C++ restatement of its default CPU path, all host threads"},
            "cpu_baseline": {"value": round(r["tok_s"], 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": r["sample"]},
            "e2e": {"value": round(r["tok_s"], 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------
def moe_roofline(torch, ctx, iters: int = 20):
    """Time the expert FFN at the config-0 shape on the tensor-core path (x terms + gate_up + down +
    combine through ms_moe_mxfp4_decode_packed), cycling over 4 layers of packed experts
    (1.7 GB > L2) with fresh routing per call; CUDA events on its stream."""
    from moe_stream_b200.engine import Context
    H = I = 2880
    E, K = 32, 4
    rb = H // 32 * 17
    n_layers = 4
    g = torch.Generator(device="cuda").manual_seed(0)
    gb, db = Context.mxfp4_packed_bytes(H, I, E)

    def mx(n_rows):
        b = torch.randint(0, 256, (E * n_rows * rb,), dtype=torch.uint8, device="cuda", generator=g)
        b.view(-1, 17)[:, 0] = torch.randint(119, 124, (E * n_rows * rb // 17,), dtype=torch.uint8, device="cuda",
                                             generator=g)
        return b

    stream = torch.cuda.current_stream()
    ctx.set_stream(stream)
    layers = []
    for _ in range(n_layers):
        gu = torch.empty(gb, dtype=torch.uint8, device="cuda")
        dn = torch.empty(db, dtype=torch.uint8, device="cuda")
        ctx.mxfp4_pack_experts(mx(I), mx(I), mx(H), H, I, E, gu, dn)
        torch.cuda.synchronize()
        layers.append((gu, dn, torch.randn(E * I, device="cuda", generator=g) * 0.01,
                       torch.randn(E * I, device="cuda", generator=g) * 0.01,
                       torch.randn(E * H, device="cuda", generator=g) * 0.01))
    x = torch.randn(H, device="cuda", generator=g)
    h = torch.zeros(H, device="cuda")
    idx = torch.stack([torch.randperm(E, device="cuda", generator=g)[:K] for _ in range(iters + 8)]).int()
    wts = torch.softmax(torch.randn(iters + 8, K, device="cuda", generator=g), -1)

    def call(i):
        L = layers[i % n_layers]
        ctx.moe_mxfp4_decode_packed(L[0], L[1], L[2], L[3], L[4], H, I, E, K, 0, x, idx[i], wts[i], h)

    for i in range(5):
        call(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(iters):
        call(i)
    e.record(stream)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    ctx.sync()
    del layers
    return ms, 4 * iters


def read_traffic(name="moe_tc_mxfp4_c0.md"):
    """dram bytes (read + write) of one expert-FFN call from a committed ncu summary, or None"""
    tp = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(tp):
        return None
    for line in open(tp):
        if line.startswith("traffic_bytes_per_call:"):
            return int(line.split(":")[1])
    return None


def run_ours(args):
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from moe_stream_b200 import synth
    from moe_stream_b200.engine import Context, Engine

    spec = synth.GPT_OSS_20B
    if args.layers:
        from dataclasses import replace
        spec = replace(spec, layers=args.layers)   # profiling cases only: fewer layers, same shapes
    prompt_len = args.prompt
    max_seq = prompt_len + 2 * args.warmup + 3 * args.steps + 64   # device, end-to-end and f32 legs
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    t0 = time.time()
    ctx = Context(local)
    ctx.set_stream(stream)
    ep = ws > 1 and args.mode == "ep"
    eng = Engine.from_spec(spec, seed=0, max_seq_len=max_seq, ctx=ctx,
                           ep_rank=rank if ep else 0, ep_size=ws if ep else 1)
    if ep and args.exchange == "nccl":
        uid = [Engine.nccl_unique_id(ctx) if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        eng.init_ep(uid[0])
    elif ep:
        eng.init_ep_p2p()   # MoE exchange by direct stores into the peers' mailboxes (NVLink)
    log(f"[rank {rank}] model generated + uploaded in {time.time() - t0:.1f}s")
    prompt = synth.prompt_ids(spec, prompt_len, seed=0)
    t0 = time.time()
    # the prompt runs through the order-independent decode step (one token at a time), so the decoded
    # tokens are the same bits at every GPU count and can be checked against the one-GPU sequence
    eng.set_prefill(0)
    eng.forward(prompt)
    log(f"[rank {rank}] prefill {prompt_len} tokens (one decode step per token) in {time.time() - t0:.1f}s")

    # ---- device-resident decode: warmup, then K timed steps ----
    eng.decode_steps_device(args.warmup)
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("decode_timed")   # the launch-list profile selects this range
        s.record(stream)
        eng.decode_steps_device(args.steps)
        e.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = s.elapsed_time(e)
    if ws > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    kps = eng.kernels_per_step
    ctx.sync()
    decoded = eng.token_log()[prompt_len:prompt_len + 64]   # greedy tokens fed after the prompt
    # ---- end to end through the C ABI with host buffers ----
    e2e_s = float("nan")
    if not args.no_e2e:
        tok = eng.decode_step(int(prompt[-1]))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            tok = eng.decode_step(tok)
        e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t.item())
    # the same decode on the f32 kernels in their own summation order (ms_model_set_exact(0)):
    # per-layer parity 1e-3 but not token-exact; timed the same way, for comparison
    fast_ms = float("nan")
    if not ep and not args.no_fast:
        eng.set_exact(False)
        eng.decode_steps_device(args.warmup)
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        eng.decode_steps_device(args.steps)
        e2.record(stream)
        torch.cuda.synchronize()
        fast_ms = s2.elapsed_time(e2)
        eng.set_exact(True)
    # per-class device time of one step: each kernel class's launches alone in a PDL-chained graph
    # (overwrites activations and KV cache, so it runs after the timed and end-to-end decodes)
    breakdown = None
    if not ep and not args.no_profile:
        us = eng.profile_step()
        names = {8: ["embed", "qkv_q8", "attention", "o_q8", "router", "moe_ffn", "resid_norm_q8", "lm_head"],
                 9: ["embed", "qkv_q8", "attention", "o_q8", "router", "moe_gate_up", "moe_down", "resid_norm_q8",
                     "lm_head"]}.get(len(us))
        breakdown = {names[i] if names else f"class{i}": round(v, 1) for i, v in enumerate(us)}
        breakdown["sum_us"] = round(sum(us), 1)
        log(f"[rank {rank}] per-step kernel-class us: {breakdown}")
    eng.close()

    # ---- roofline of the dominant kernel pair (MXFP4 expert FFN) ----
    # the decode's own expert kernels (order-independent gate/up + down on tcgen05): their per-layer
    # device time from the class profile above (CUDA events, each class alone in a PDL chain)
    peak, peak_kind = peaks()
    exact_us = None
    if breakdown and "moe_gate_up" in breakdown:
        exact_us = (breakdown["moe_gate_up"] + breakdown["moe_down"]) / spec.layers
    exact_ach = MOE_BYTES / (exact_us * 1e-6) / 1e9 if exact_us else float("nan")
    # and the approximate tensor-core expert FFN of the C ABI (ms_moe_mxfp4_decode_packed)
    moe_ms, moe_launches = moe_roofline(torch, ctx) if not args.no_roofline else (float("nan"), 0)
    achieved = MOE_BYTES / (moe_ms * 1e-3) / 1e9 if moe_ms == moe_ms else float("nan")
    traffic = read_traffic()
    traffic_exact = read_traffic("exact_tc_moe_c1.md")

    cpu = None
    if rank == 0 and not args.no_cpu:
        r = cpu_sample(args.steps_ref, 1, os.cpu_count() or 1)
        cpu = {"value": round(r["tok_s"], 4), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": r["sample"]}
    if rank != 0:
        return
    if args.save_tokens and rank == 0:
        np.savez(args.save_tokens, tokens=np.asarray(decoded, np.int32))
    streams = 1 if ep else ws          # expert parallel: all ranks decode one sequence together
    tokens_match = None
    ref_path = os.path.join(ROOT, "tests", "golden", "bench_tokens_c1.npz")
    if os.path.exists(ref_path) and not args.layers and prompt_len == PROMPT:
        ref = np.load(ref_path)["tokens"].tolist()
        n = min(len(ref), len(decoded))
        tokens_match = bool(n > 0 and decoded[:n] == ref[:n])
    value = streams * args.steps / (ms * 1e-3)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if ep else "weak", "vs_baseline": None, "dtype": "mxf4 x mxf4 (f32 accumulate) experts; q8_0 dp4a projections; f32 attention/KV; f16 head",
        "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
        "config": {"workload": "GPT-OSS-20B-shaped MXFP4 greedy decode, bs1, after a 2048-token prompt",
                   "model": "gpt-oss-20b-shaped", "global_batch": streams, "seq_len": prompt_len,
                   "parallelism": (f"ep{ws}" if ep else f"replicas{ws}"),
                   "ep_exchange": (args.exchange if ep else None),
                   "l2": "no flush: each step streams ~3.1 GB of weights (> 126 MB L2)"},
        "e2e": {"value": round(streams * args.steps / e2e_s, 2) if e2e_s == e2e_s else None, "unit": "tok/s", "h2d_bytes_per_step": 4 + 4,
                "d2h_bytes_per_step": 8},
        "roofline": {"kernel": "order-independent expert FFN on tcgen05 (exact_tc_kernel gate/up + down; "
                               "one token-layer of the decode above)",
                     "bound": "hbm",
                     "achieved": round(exact_ach, 1) if exact_us else None, "peak": peak, "unit": "GB/s",
                     "frac": round(exact_ach / peak, 4) if exact_us else None, "peak_kind": peak_kind,
                     "algorithmic_bytes": MOE_BYTES, "us_per_call": round(exact_us, 2) if exact_us else None,
                     "traffic": traffic_exact},
        "roofline_approx_ffn": {"kernel": "approximate expert FFN on tcgen05 (ms_moe_mxfp4_decode_packed: x terms + "
                                          "gate_up + down + combine; config-0 shape, one token-layer)",
                                "achieved": round(achieved, 1), "frac": round(achieved / peak, 4),
                                "us_per_call": round(moe_ms * 1000, 2), "traffic": traffic},
        "fast_numerics": ({"value": round(streams * args.steps / (fast_ms * 1e-3), 2), "unit": "tok/s",
                           "ms_per_step": round(fast_ms / args.steps, 4),
                           "note": "f32 kernels in their own summation order (ms_model_set_exact(0)): per-layer "
                                   "parity 1e-3, not token-exact; same model state, timed the same way"}
                          if fast_ms == fast_ms else None),
        "decoded_tokens": decoded[:16],
        "tokens_match": tokens_match,
        "gpu_launches": kps * args.steps,
        "kernels_per_step": kps,
        "kernel_us_per_step": breakdown,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


def run_case_moe(args):
    """Small profiling case: the config-0 MoE layer (gate/up + down kernels) only, ~1.7 GB."""
    import torch
    from moe_stream_b200.engine import Context
    ctx = Context(0)
    ms, _ = moe_roofline(torch, ctx, iters=max(1, args.steps))
    print(json.dumps({"case": "moe-layer", "us_per_call": round(ms * 1000, 2),
                      "achieved_gbs": round(MOE_BYTES / (ms * 1e-3) / 1e9, 1)}), flush=True)


def run_case_prefill(args):
    """Config 4's MoE step on one GPU: 8 prompts x 2048 tokens through one GPT-OSS-20B-shaped MoE
    layer (uniform random top-4 routing, seeded), tokens sorted by expert into the grouped bf16
    GEMM on tcgen05.  FLOPs = T x K x 3 x 2 x 2880^2 per layer; CUDA events on the stream."""
    import torch
    from moe_stream_b200.engine import Context
    H = I = 2880
    E, K, T = 32, 4, 8 * 2048
    rb = H // 32 * 17
    g = torch.Generator(device="cuda").manual_seed(0)
    ctx = Context(0)
    stream = torch.cuda.current_stream()
    ctx.set_stream(stream)
    gb, db = Context.mxfp4_packed_bytes(H, I, E)

    def mx(n_rows):
        b = torch.randint(0, 256, (E * n_rows * rb,), dtype=torch.uint8, device="cuda", generator=g)
        b.view(-1, 17)[:, 0] = torch.randint(119, 124, (E * n_rows * rb // 17,), dtype=torch.uint8, device="cuda",
                                             generator=g)
        return b

    gu = torch.empty(gb, dtype=torch.uint8, device="cuda")
    dn = torch.empty(db, dtype=torch.uint8, device="cuda")
    ctx.mxfp4_pack_experts(mx(I), mx(I), mx(H), H, I, E, gu, dn)
    bias = [torch.randn(E * I, device="cuda", generator=g) * 0.01, torch.randn(E * I, device="cuda", generator=g) * 0.01,
            torch.randn(E * H, device="cuda", generator=g) * 0.01]
    x = torch.randn(T, H, device="cuda", generator=g)
    x = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-5)
    idx = torch.argsort(torch.rand(T, E, device="cuda", generator=g), dim=1)[:, :K].int().contiguous()
    wts = torch.softmax(torch.randn(T, K, device="cuda", generator=g), -1).contiguous()
    out = torch.empty(T, H, device="cuda")

    def call():
        ctx.moe_mxfp4_prefill_packed(gu, dn, bias[0], bias[1], bias[2], H, I, E, K, 0, x, T, idx, wts, out)

    for _ in range(max(3, args.warmup)):
        call()
    torch.cuda.synchronize()
    n = max(1, args.steps)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        s.record(stream)
        for _ in range(n):
            call()
        e.record(stream)
        torch.cuda.synchronize()
    ms = s.elapsed_time(e) / n
    ctx.sync()
    flops = T * K * 3 * 2 * H * I
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = float(pk.get("bf16_tflops_sustained", 1400.0))
    tf = flops / (ms * 1e-3) / 1e12
    print(json.dumps({"case": "prefill", "metric": "MoE prefill TFLOP/s (config 4, one layer)", "tokens": T,
                      "ms_per_layer": round(ms, 3), "tflops": round(tf, 1), "peak_bf16_tflops": peak,
                      "peak_kind": "measured sustained" if pk else "fallback", "frac": round(tf / peak, 4),
                      "tok_s_prefill_24_layers_moe_only": round(T / (24 * ms * 1e-3), 1),
                      "clocks": clk.summary()}), flush=True)


def qwen3_step_bytes(spec, batch, ctx_len):
    """Algorithmic HBM bytes of one config-2 decode step: every weight byte once per step (experts:
    the expected unique experts of `batch` tokens under uniform routing, E(1 - (1 - k/E)^B)), the f32
    KV of every sequence at `ctx_len` positions, the f16 LM head."""
    H, L, E, k, I = spec.hidden, spec.layers, spec.experts, spec.top_k, spec.inter
    q8 = lambda rows, cols: rows * (cols // 32) * 34
    attn = q8(spec.q_dim + 2 * spec.kv_dim, H) + q8(H, spec.q_dim)
    expert = 2 * I * (H // 256) * 144 + H * (I // 256) * 210
    uniq = E * (1.0 - (1.0 - k / E) ** batch)
    router = E * H * 4
    kv = batch * ctx_len * spec.kv_heads * spec.head_dim * 4 * 2
    per_layer = attn + router + uniq * expert + kv
    return L * per_layer + spec.vocab * H * 2, uniq


def run_case_qwen3(args):
    """Config 2: Qwen3-30B-A3B-shaped Q4_K/Q6_K model, greedy decode at batch 1 and 32 with a
    4096-token KV context.  bs1 runs the single-sequence step; bs32 the lockstep batch step (one
    shared position, every weight byte streamed once per step).  Each batch prefills its prompt
    (one step per position), then K device-resident greedy steps are timed with CUDA events."""
    import torch
    from dataclasses import replace
    from moe_stream_b200 import synth
    from moe_stream_b200.engine import Context, Engine
    spec = synth.QWEN3_30B_A3B
    if args.layers:
        spec = replace(spec, layers=args.layers)
    prompt_len = args.prompt
    batches = [int(b) for b in args.batch.split(",")]
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = Context(0)
    ctx.set_stream(stream)
    t0 = time.time()
    eng = Engine.from_spec(spec, seed=0, max_seq_len=prompt_len + args.warmup + args.steps + 64, ctx=ctx)
    log(f"qwen3 model generated + uploaded in {time.time() - t0:.1f}s")
    peak, peak_kind = peaks()
    out = {"case": "qwen3-30b-a3b", "metric": "decode tok/s (bs1, bs32)", "config": {
        "workload": f"Qwen3-30B-A3B-shaped Q4_K/Q6_K greedy decode after a {prompt_len}-token prompt",
        "layers": spec.layers, "kv_context": prompt_len, "l2": "no flush: each step streams > 2 GB"},
        "steps": args.steps, "warmup": args.warmup}
    modes = ["exact", "fast"] if args.numerics == "both" else [args.numerics]
    for mode, B in [(m, b) for m in modes for b in batches]:
        # exact: the order-independent kernels (token-exact against the oracle); fast: f32 kernels
        # in their own summation order (per-layer parity 1e-3, not token-exact over long runs)
        eng.set_exact(mode == "exact")
        prompts = np.stack([synth.prompt_ids(spec, prompt_len, seed=b) for b in range(B)])
        t0 = time.time()
        if B == 1:
            eng.clear_cache()
            eng.forward(prompts[0])
            run = eng.decode_steps_device
        else:
            eng.batch_open(B)
            eng.batch_forward(prompts)
            run = eng.batch_decode_steps_device
        torch.cuda.synchronize()
        log(f"bs{B}: prefill {prompt_len} positions in {time.time() - t0:.1f}s")
        run(args.warmup)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as clk:
            s.record(stream)
            run(args.steps)
            e.record(stream)
            torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        ctx.sync()
        nbytes, uniq = qwen3_step_bytes(spec, B, prompt_len + args.warmup + args.steps // 2)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res = out.setdefault(mode, {})
        res[f"bs{B}"] = {"tok_s": round(B / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
                         "kernels_per_step": eng.kernels_per_step if B == 1 else eng.batch_kernels_per_step,
                         "algorithmic_bytes_per_step": int(nbytes), "expected_unique_experts_per_layer": round(uniq, 1),
                         "achieved_gbs": round(gbs, 1), "hbm_frac": round(gbs / peak, 4), "peak_kind": peak_kind,
                         "clocks": clk.summary()}
        if not args.no_profile:
            res[f"bs{B}"]["kernel_us_per_step"] = (eng.batch_profile_step() if B > 1 else
                                                   [round(v, 1) for v in eng.profile_step()])
        log(f"{mode} bs{B}: {res[f'bs{B}']}")
        if B > 1:
            eng.batch_close()
    eng.close()
    print(json.dumps(out), flush=True)


def qwen3next_step_bytes(spec, ctx_len):
    """Algorithmic HBM bytes of one config-3 decode step (batch 1): the Q4_K DeltaNet projections and
    the f32 recurrent state (read and written) of the DeltaNet layers, the Q8_0 gated-attention
    projections and f32 KV at ctx_len positions of the attention layers, and in every layer the f32
    router, the top-k routed Q4_K experts and the shared expert; plus the f16 LM head."""
    H, E, k, I, S = spec.hidden, spec.experts, spec.top_k, spec.inter, spec.shared_inter
    q4 = lambda rows, cols: rows * (cols // 256) * 144
    q8 = lambda rows, cols: rows * (cols // 32) * 34
    nv, hvd = spec.ssm_dt_rank, spec.ssm_inner // spec.ssm_dt_rank
    dn = (q4(spec.ssm_conv_dim, H) + q4(spec.ssm_inner, H) + q4(2 * nv, H) + q4(H, spec.ssm_inner)
          + 2 * nv * spec.ssm_state * hvd * 4 + 2 * spec.ssm_conv_dim * (spec.ssm_conv - 1) * 4)
    attn = (q8(2 * spec.q_dim + 2 * spec.kv_dim, H) + q8(H, spec.q_dim)
            + 2 * ctx_len * spec.kv_heads * spec.head_dim * 4)
    moe = E * H * 4 + k * 3 * q4(I, H) + 3 * q4(S, H)
    n_attn = sum(spec.is_attention_layer(li) for li in range(spec.layers))
    return n_attn * attn + (spec.layers - n_attn) * dn + spec.layers * moe + spec.vocab * H * 2


def run_case_qwen3next(args):
    """Config 3: Qwen3-Coder-Next-80B-shaped DeltaNet hybrid (36 Gated DeltaNet + 12 gated-attention
    layers, 512 Q4_K experts top-10 + a shared expert), greedy decode at batch 1 after a --prompt-token
    prompt (one step per position), then K device-resident greedy steps timed with CUDA events.  The
    43 GB of expert stacks are generated once and uploaded to every layer's own buffers (the routers,
    and so the routing, differ per layer)."""
    import re
    import torch
    from dataclasses import replace
    from moe_stream_b200 import synth
    from moe_stream_b200.engine import Context, Engine
    spec = synth.QWEN3_NEXT_80B
    if args.layers:
        spec = replace(spec, layers=args.layers)
    prompt_len = args.prompt
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = Context(0)
    ctx.set_stream(stream)
    t0 = time.time()
    share = lambda n: re.sub(r"^blk\.\d+\.(ffn_(gate|up|down)_exps\.weight)$", r"blk.0.\1", n) \
        if re.match(r"^blk\.\d+\.ffn_(gate|up|down)_exps\.weight$", n) else None
    eng = Engine.from_spec(spec, seed=0, max_seq_len=prompt_len + args.warmup + args.steps + 64, ctx=ctx,
                           share=share)
    log(f"qwen3-next model generated + uploaded in {time.time() - t0:.1f}s")
    peak, peak_kind = peaks()
    prompt = synth.prompt_ids(spec, prompt_len, seed=0)
    t0 = time.time()
    eng.clear_cache()
    eng.forward(prompt)
    torch.cuda.synchronize()
    log(f"prompt of {prompt_len} positions in {time.time() - t0:.1f}s")
    eng.decode_steps_device(args.warmup)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        s.record(stream)
        eng.decode_steps_device(args.steps)
        e.record(stream)
        torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    ctx.sync()
    nbytes = qwen3next_step_bytes(spec, prompt_len + args.warmup + args.steps // 2)
    gbs = nbytes / (ms * 1e-3) / 1e9
    out = {"case": "qwen3-coder-next-80b", "metric": "decode tok/s (bs1)", "value": round(1e3 / ms, 1),
           "unit": "tok/s", "ms_per_step": round(ms, 4), "steps": args.steps, "warmup": args.warmup,
           "n_gpus": 1, "dtype": "f32 (Q4_K / Q8_0 weights)", "data": "synthetic",
           "kernels_per_step": eng.kernels_per_step, "algorithmic_bytes_per_step": int(nbytes),
           "achieved_gbs": round(gbs, 1), "hbm_frac": round(gbs / peak, 4), "peak_kind": peak_kind,
           "clocks": clk.summary(),
           "config": {"workload": f"Qwen3-Coder-Next-80B-shaped DeltaNet hybrid, greedy decode after a "
                                  f"{prompt_len}-token prompt", "layers": spec.layers,
                      "attention_layers": sum(spec.is_attention_layer(li) for li in range(spec.layers)),
                      "experts": spec.experts, "top_k": spec.top_k, "kv_context": prompt_len,
                      "expert_bytes": "one generated set uploaded to every layer",
                      "l2": "no flush: each step streams > 2 GB"}}
    eng.close()
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--steps-ref", type=int, default=3, help="timed tokens of the CPU sample")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-roofline", action="store_true", help="skip the expert-FFN roofline leg")
    ap.add_argument("--no-profile", action="store_true", help="skip the per-kernel-class breakdown")
    ap.add_argument("--no-fast", action="store_true", help="skip the f32-numerics comparison leg")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt length (default 2048)")
    ap.add_argument("--layers", type=int, default=0, help="profiling only: override the layer count")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="expert-parallel MoE exchange: peer-memory stores (default) or NCCL all-reduce")
    ap.add_argument("--mode", default="ep", choices=["ep", "replicas"],
                    help="N > 1: expert parallel over one sequence (default) or N independent replicas")
    ap.add_argument("--case", default=None, choices=[None, "moe-layer", "prefill", "qwen3", "qwen3next"],
                    help="moe-layer: the decode expert FFN alone; prefill: config 4's MoE step; "
                         "qwen3: config 2 decode at the --batch sizes")
    ap.add_argument("--batch", default="1,32", help="qwen3 case: comma-separated batch sizes")
    ap.add_argument("--numerics", default="both", choices=["exact", "fast", "both"],
                    help="qwen3 case: order-independent kernels, f32 kernels, or both")
    ap.add_argument("--save-tokens", default=None, help="write the greedy tokens decoded after the prompt (npz)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case == "moe-layer":
        run_case_moe(args)
    elif args.case == "prefill":
        run_case_prefill(args)
    elif args.case == "qwen3":
        if args.prompt == PROMPT:
            args.prompt = 4096
        run_case_qwen3(args)
    elif args.case == "qwen3next":
        if args.prompt == PROMPT:
            args.prompt = 4096
        run_case_qwen3next(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
