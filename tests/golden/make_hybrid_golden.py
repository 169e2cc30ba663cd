"""Generate ``tests/golden/tiny_qwen3_next.npz``: a seeded tiny Qwen3-Next-shaped DeltaNet hybrid
(moe_stream_b200.synth.TINY_QWEN3_NEXT: 3 Gated DeltaNet layers per gated-attention layer, head_dim
256 with rotary 0.25, 64 experts top-10, a shared expert per layer) run through the CPU oracle.

Stored: the prompt, the oracle's greedy tokens, the last-position logits after the prompt, and the
per-layer residual stream and router logits of that position.  The GPU parity test compares the
CUDA model step with these; the CPU suite re-runs the oracle against them (a pin of the oracle across
machines).

Run from the repository root:  python tests/golden/make_hybrid_golden.py
"""
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from moe_stream_b200 import synth  # noqa: E402
from oracle import oracle as orc  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tiny_qwen3_next.npz")
SEED, N_PROMPT, N_TOKENS, MAX_SEQ = 11, 8, 24, 64


def run(path: str) -> dict:
    spec = synth.TINY_QWEN3_NEXT
    prompt = synth.prompt_ids(spec, N_PROMPT, seed=SEED)
    om = orc.Model(path, max_seq_len=MAX_SEQ)
    tokens = om.generate(prompt, N_TOKENS)
    om.clear_cache()
    logits = om.forward(prompt)
    hid, lg = om.layer_trace(spec.layers, spec.experts)
    idx, w = om.last_routing(spec.layers, spec.top_k)
    om.close()
    return dict(prompt=prompt, tokens=tokens, logits=logits, layer_hidden=hid, layer_logits=lg,
                routing_idx=idx, routing_w=w)


def main() -> None:
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "tiny_qwen3_next.gguf")
        synth.write_model(path, synth.TINY_QWEN3_NEXT, seed=SEED)
        out = run(path)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, "tokens", out["tokens"].tolist())


if __name__ == "__main__":
    main()
