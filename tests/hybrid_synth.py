"""Seeded synthetic Gated DeltaNet layers and shared experts (Qwen3-Next / Qwen3.5 shapes) for the
oracle and GPU parity tests, plus an independent float64 numpy restatement of one DeltaNet decode
token (model/deltanet.rs:204-543) used to cross-check the C oracle."""
import numpy as np

from moe_stream_b200 import gguf as G
from moe_stream_b200 import synth


def weight(rng, qtype, rows, cols, scale):
    if qtype == G.F32:
        return (rng.standard_normal(rows * cols) * scale).astype(np.float32).view(np.uint8)
    if qtype == G.Q4_K:
        return synth.rand_q4_k(rng, rows * cols)
    if qtype == G.Q6_K:
        return synth.rand_q6_k(rng, rows * cols)
    raise ValueError(qtype)


def deltanet_layer(seed, hidden=256, nk=2, hkd=64, nv=4, hvd=128, ks=4, qtype=G.F32):
    rng = np.random.default_rng(seed)
    qt, vt = nk * hkd, nv * hvd
    conv_dim = 2 * qt + vt
    s = 1.0 / np.sqrt(hidden)
    return dict(hidden=hidden, n_k_heads=nk, head_k_dim=hkd, n_v_heads=nv, head_v_dim=hvd, conv_kernel=ks,
                eps=1e-6, qkv_q=qtype, qkv=weight(rng, qtype, conv_dim, hidden, s),
                gate_q=qtype, gate=weight(rng, qtype, vt, hidden, s),
                ba_q=qtype, ba=weight(rng, qtype, 2 * nv, hidden, s),
                out_q=qtype, out=weight(rng, qtype, hidden, vt, 1.0 / np.sqrt(vt)),
                conv1d=(rng.standard_normal((conv_dim, ks)) * 0.5).astype(np.float32),
                ssm_a=(-np.exp(rng.uniform(-1.0, 1.0, nv))).astype(np.float32),
                dt_bias=rng.uniform(-1.0, 1.0, nv).astype(np.float32),
                norm=rng.uniform(0.5, 1.5, hvd).astype(np.float32))


def dense(orc, qtype, raw, rows, cols):
    return orc.dequantize(qtype, raw, rows * cols).reshape(rows, cols).astype(np.float64)


def deltanet_step_np(orc, d, x, conv_state, rec_state):
    """float64 restatement of one decode token; returns (y, new conv_state, new rec_state)"""
    H, nk, hkd, nv, hvd, ks = (d[k] for k in ("hidden", "n_k_heads", "head_k_dim", "n_v_heads", "head_v_dim",
                                              "conv_kernel"))
    qt, vt = nk * hkd, nv * hvd
    conv_dim = 2 * qt + vt
    x = x.astype(np.float64)
    mixed = dense(orc, d["qkv_q"], d["qkv"], conv_dim, H) @ x
    z = dense(orc, d["gate_q"], d["gate"], vt, H) @ x
    ba = dense(orc, d["ba_q"], d["ba"], 2 * nv, H) @ x
    beta = 1.0 / (1.0 + np.exp(-ba[:nv]))
    alpha = d["ssm_a"].astype(np.float64) * np.log1p(np.exp(ba[nv:] + d["dt_bias"]))
    window = np.concatenate([conv_state.astype(np.float64), mixed[:, None]], axis=1)   # [C, ks]
    conv = (window * d["conv1d"].astype(np.float64)).sum(1)
    conv = conv / (1.0 + np.exp(-conv))
    new_conv = window[:, 1:].astype(np.float32)
    vpk = nv // nk
    q = np.repeat(conv[:qt].reshape(nk, hkd), vpk, axis=0)
    k = np.repeat(conv[qt:2 * qt].reshape(nk, hkd), vpk, axis=0)
    v = conv[2 * qt:].reshape(nv, hvd)
    q = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), d["eps"]) / np.sqrt(hvd)
    k = k / np.maximum(np.linalg.norm(k, axis=1, keepdims=True), d["eps"])
    S = rec_state.astype(np.float64).reshape(nv, hkd, hvd) * np.exp(alpha)[:, None, None]
    kv = np.einsum("hi,hij->hj", k, S)
    delta = (v - kv) * beta[:, None]
    S = S + k[:, :, None] * delta[:, None, :]
    o = np.einsum("hi,hij->hj", q, S)
    rms = np.sqrt((o * o).mean(1, keepdims=True) + d["eps"])
    o = o / rms * d["norm"].astype(np.float64)
    o = o.reshape(vt) * (z / (1.0 + np.exp(-z)))
    y = dense(orc, d["out_q"], d["out"], H, vt) @ o
    return y, new_conv, S.reshape(rec_state.shape).astype(np.float32)


def shared_expert(seed, hidden=256, inter=128, gu_q=G.F32, down_q=G.F32, gated=True):
    rng = np.random.default_rng(seed)
    return dict(gu_q=gu_q, gate=weight(rng, gu_q, inter, hidden, 1.0 / np.sqrt(hidden)),
                up=weight(rng, gu_q, inter, hidden, 1.0 / np.sqrt(hidden)), down_q=down_q,
                down=weight(rng, down_q, hidden, inter, 1.0 / np.sqrt(inter)),
                gate_inp=(rng.standard_normal(hidden) * 0.05).astype(np.float32) if gated else None,
                hidden=hidden, inter=inter)


def shared_expert_np(orc, e, x):
    H, I = e["hidden"], e["inter"]
    x = x.astype(np.float64)
    g = dense(orc, e["gu_q"], e["gate"], I, H) @ x
    u = dense(orc, e["gu_q"], e["up"], I, H) @ x
    o = dense(orc, e["down_q"], e["down"], H, I) @ (g / (1.0 + np.exp(-g)) * u)
    if e["gate_inp"] is not None:
        o = o / (1.0 + np.exp(-(x @ e["gate_inp"].astype(np.float64))))
    return o
