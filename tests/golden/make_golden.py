"""Generate the committed golden fixtures under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

1. ``dequant_kat.npz`` — block-dequant known answers.  Inputs are seeded random
   blocks plus hand-built edge blocks (every e8m0 edge 0/1/2/254/255, the -0 nibble,
   Q4_K/Q6_K scale extremes).  Expected outputs come from the ``gguf`` Python
   package (gguf 0.19.0, ``gguf.quants.dequantize``), an implementation of the GGML
   block formats independent of both the reference and this repository.  The one
   known difference, MXFP4 nibble 8, is -0.0 in moe-stream (dequant.rs:580-583) and
   +0.0 in gguf; fixtures store the moe-stream sign.
2. ``tiny_models.npz`` — seeded tiny GPT-OSS-/Qwen3-shaped models: greedy tokens,
   last hidden state and last-position logits from the CPU oracle, a regression pin
   of the oracle itself across machines.
"""
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from moe_stream_b200 import gguf as G  # noqa: E402
from moe_stream_b200 import synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def edge_mxfp4() -> np.ndarray:
    blocks = []
    for e in (0, 1, 2, 3, 127, 128, 200, 253, 254, 255):
        b = np.zeros(17, np.uint8)
        b[0] = e
        b[1:] = np.arange(16, dtype=np.uint8) | (np.arange(15, -1, -1, dtype=np.uint8) << 4)
        blocks.append(b)
    return np.concatenate(blocks)


def edge_q4k() -> np.ndarray:
    b = np.zeros((3, 144), np.uint8)
    b[0, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)       # reference test block (dequant.rs:819-837)
    b[0, 4:8] = 1
    b[1, 0:4] = np.frombuffer(np.array([0.5, 0.25], np.float16).tobytes(), np.uint8)
    b[1, 4:16] = 0xFF                                                    # all scales/mins = 63
    b[1, 16:] = 0xFF
    b[2, 0:4] = np.frombuffer(np.array([-2.0, 65504.0], np.float16).tobytes(), np.uint8)
    b[2, 4:] = np.arange(140, dtype=np.uint8)
    return b.reshape(-1)


def edge_q6k() -> np.ndarray:
    b = np.zeros((3, 210), np.uint8)                                     # zero block (dequant.rs:840-844)
    b[1, :192] = 0xFF
    b[1, 192:208] = np.array([127, 128, 1, 255] * 4, np.uint8)
    b[1, 208:210] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    b[2, :208] = np.arange(208, dtype=np.uint8)
    b[2, 208:210] = np.frombuffer(np.float16(6.1e-5).tobytes(), np.uint8)
    return b.reshape(-1)


def edge_q8_0() -> np.ndarray:
    b = np.zeros((3, 34), np.uint8)
    b[0, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    b[0, 2:] = np.array([127, 128, 129, 255, 0, 1] + list(range(26)), np.uint8)
    b[1, 0:2] = np.frombuffer(np.float16(-0.0).tobytes(), np.uint8)
    b[1, 2:] = 0x80
    b[2, 0:2] = np.array([0x01, 0x00], np.uint8)                       # smallest f16 subnormal
    b[2, 2:] = np.arange(32, dtype=np.uint8)
    return b.reshape(-1)


def gguf_dequant(qtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    import gguf
    from gguf import quants
    t = gguf.GGMLQuantizationType(qtype)
    out = quants.dequantize(raw.reshape(1, -1), t).astype(np.float32).reshape(-1)
    assert out.size == n
    if qtype == G.MXFP4:   # moe-stream keeps -0.0 for nibble 8
        nib = np.empty(n, np.uint8)
        blk = raw.reshape(-1, 17)[:, 1:]
        nib.reshape(-1, 32)[:, :16] = blk & 0x0F
        nib.reshape(-1, 32)[:, 16:] = blk >> 4
        out = np.where(nib == 8, np.float32(-0.0), out)
    return out


def make_dequant():
    rng = np.random.default_rng(1234)
    fx = {}
    cases = {
        "mxfp4": (G.MXFP4, np.concatenate([synth.rand_mxfp4(rng, 32 * 64, 0, 255), edge_mxfp4()])),
        "q4_k": (G.Q4_K, np.concatenate([synth.rand_q4_k(rng, 256 * 8), edge_q4k()])),
        "q6_k": (G.Q6_K, np.concatenate([synth.rand_q6_k(rng, 256 * 8), edge_q6k()])),
        "q8_0": (G.Q8_0, np.concatenate([synth.rand_q8_0(rng, 32 * 64), edge_q8_0()])),
        "f16": (G.F16, np.concatenate([rng.standard_normal(512).astype(np.float16).view(np.uint8),
                                       np.array([0, 0x3C, 0, 0xBC, 0x01, 0, 0xFF, 0x7B, 0, 0x7C, 0, 0xFC], np.uint8)])),
    }
    for key, (q, raw) in cases.items():
        bb, be = G.BLOCK_INFO[q]
        n = raw.size // bb * be
        fx[f"{key}_raw"] = raw
        fx[f"{key}_out"] = gguf_dequant(q, raw, n)
    np.savez_compressed(os.path.join(OUT, "dequant_kat.npz"), **fx)


def make_tiny():
    from oracle import oracle
    oracle.build()
    fx = {}
    for name, spec in (("tiny_gpt_oss", synth.TINY_GPT_OSS), ("tiny_qwen3", synth.TINY_QWEN3)):
        with tempfile.TemporaryDirectory() as d:
            p = os.path.join(d, "m.gguf")
            synth.write_model(p, spec, seed=7)
            m = oracle.Model(p, max_seq_len=256)
            prompt = synth.prompt_ids(spec, 12, seed=7)
            toks = m.generate(prompt, 16)
            m.clear_cache()
            logits = m.forward(prompt)
            fx[f"{name}_prompt"] = prompt
            fx[f"{name}_tokens"] = toks
            fx[f"{name}_logits"] = logits
            fx[f"{name}_hidden"] = m.last_hidden()
            m.close()
    np.savez_compressed(os.path.join(OUT, "tiny_models.npz"), **fx)


if __name__ == "__main__":
    make_dequant()
    make_tiny()
    print("golden fixtures written to", OUT)
