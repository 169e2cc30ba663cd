"""Golden fixtures of the CPU oracle at the benchmarked model shapes.

Writes, from the seeded synthetic models of ``moe_stream_b200.synth`` (the weights themselves are
not stored: the GPU test regenerates them from the same seed, byte for byte):

* ``gpt_oss_20b_c1.npz`` -- configuration 1 (24-layer GPT-OSS-20B shape, MXFP4 experts): a
  32-token prompt, then 128 greedy tokens.  For every forward: the routed experts of each layer
  and the gap between each layer's k-th and (k+1)-th router logit (the tie test).  For the prompt
  forward and the last decode forward: the residual stream after every layer, every layer's
  router logits, and the final logits (top 64 and a fixed sample of 4096 ids).
* ``qwen3_30b_c2.npz`` -- configuration 2 (48-layer Qwen3-30B-A3B shape, Q4_K / Q6_K experts):
  a 16-token prompt then 32 greedy tokens at batch 1 with the same per-forward records, and 32
  sequences of 6-token prompts with 6 greedy tokens each (the bs32 lockstep batch).

Prompts are shorter than the benchmark's 2048 / 4096 tokens so the oracle (a plain C++ loop)
finishes in minutes; the decode step and its kernels are the same at every position, and the
sliding-window ring of configuration 1 (128 slots) is passed by the 160 positions.

Run: python tests/golden/make_full_golden.py [workdir for the temporary GGUF files]
"""
from __future__ import annotations

import os
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from moe_stream_b200 import synth  # noqa: E402
from oracle import oracle  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
SAMPLE_IDS = 4096


def _margins(router_logits: np.ndarray, k: int) -> np.ndarray:
    srt = -np.sort(-router_logits.astype(np.float64), axis=-1)
    return (srt[..., k - 1] - srt[..., k]).astype(np.float32)


def _decode_records(m, spec, prompt, n_new, keep_full):
    """greedy decode with per-forward routing records; full traces for forwards in keep_full"""
    L, K, E = spec.layers, spec.top_k, spec.experts
    sample = np.random.default_rng(1234).choice(spec.vocab, SAMPLE_IDS, replace=False).astype(np.int32)
    rec = {"tokens": [], "route_idx": [], "route_margin": []}
    full = {}
    tok = None
    for f in range(n_new):
        t0 = time.time()
        logits = m.forward(prompt if f == 0 else [tok])
        tok = int(np.argmax(logits))       # first maximum = lowest id on ties (engine.rs stable sort)
        idx, _ = m.last_routing(L, K)
        hid, lg = m.layer_trace(L, E)
        rec["tokens"].append(tok)
        rec["route_idx"].append(idx.astype(np.int16))
        rec["route_margin"].append(_margins(lg, K))
        if f in keep_full:
            top = np.argsort(-logits, kind="stable")[:64].astype(np.int32)
            full[f] = {"hidden": hid, "router_logits": lg, "top_ids": top, "top_vals": logits[top],
                       "sample_vals": logits[sample]}
        print(f"  forward {f}: token {tok} ({time.time() - t0:.1f}s)", flush=True)
    out = {k: np.asarray(v) for k, v in rec.items()}
    out["sample_ids"] = sample
    for f, d in full.items():
        for k, v in d.items():
            out[f"f{f}_{k}"] = v
    out["full_forwards"] = np.asarray(sorted(full), np.int32)
    return out


def gpt_oss(work: str) -> None:
    spec = synth.GPT_OSS_20B
    path = os.path.join(work, "gpt_oss_20b.gguf")
    t0 = time.time()
    synth.write_model(path, spec, seed=0)
    print(f"gpt-oss-20b GGUF written in {time.time() - t0:.0f}s", flush=True)
    m = oracle.Model(path, max_seq_len=256)
    prompt = synth.prompt_ids(spec, 32, seed=0)
    n_new = 128
    rec = _decode_records(m, spec, prompt, n_new, keep_full={0, n_new - 1})
    m.close()
    os.unlink(path)
    np.savez_compressed(os.path.join(HERE, "gpt_oss_20b_c1.npz"), prompt=prompt, seed=np.int32(0), **rec)


def qwen3(work: str) -> None:
    spec = synth.QWEN3_30B_A3B
    path = os.path.join(work, "qwen3_30b.gguf")
    t0 = time.time()
    synth.write_model(path, spec, seed=0)
    print(f"qwen3-30b GGUF written in {time.time() - t0:.0f}s", flush=True)
    m = oracle.Model(path, max_seq_len=128)
    prompt = synth.prompt_ids(spec, 16, seed=0)
    n_new = 32
    rec = _decode_records(m, spec, prompt, n_new, keep_full={0, n_new - 1})
    B, T, N = 32, 6, 6
    prompts = np.stack([synth.prompt_ids(spec, T, seed=100 + b) for b in range(B)])
    batch_tokens = np.empty((B, N), np.int32)
    for b in range(B):
        t0 = time.time()
        m.clear_cache()
        batch_tokens[b] = m.generate(prompts[b], N)
        print(f"  batch sequence {b}: {batch_tokens[b].tolist()} ({time.time() - t0:.1f}s)", flush=True)
    m.close()
    os.unlink(path)
    np.savez_compressed(os.path.join(HERE, "qwen3_30b_c2.npz"), prompt=prompt, seed=np.int32(0),
                        batch_prompts=prompts, batch_tokens=batch_tokens, **rec)


if __name__ == "__main__":
    oracle.build()
    work = sys.argv[1] if len(sys.argv) > 1 else tempfile.mkdtemp()
    which = sys.argv[2] if len(sys.argv) > 2 else "all"
    if which in ("all", "gpt-oss"):
        gpt_oss(work)
    if which in ("all", "qwen3"):
        qwen3(work)
