"""The oracle's decode attention half-layer (layer.rs:511-749; ops/attention.rs:9-164, 178-280)
against a float64 numpy restatement over several positions: RMSNorm, projections (exact f32 mode),
QK-norm, NeoX RoPE of the first rot_dim dims with the reference's f32 tables, GQA, attention sinks
(max(m, sink) shift and the sink term in the denominator), the sliding-window mask, the hybrid
models' gated Q ([Q_h, gate_h] per head, output x sigmoid(gate)) and the O projection."""
import numpy as np
import pytest

from .test_gpu_parity import _attn_layer


def _rms(x, w, eps):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w


def _rope_tables(rot, theta, pos):
    half = rot // 2
    inv = np.array([np.float32(1.0) / np.float32(theta ** (2.0 * i / rot)) for i in range(half)], np.float32)
    f = (np.float32(pos) * inv).astype(np.float32)
    return np.cos(f.astype(np.float64)).astype(np.float32), np.sin(f.astype(np.float64)).astype(np.float32)


def _rope(x, c, s, rot):
    half = rot // 2
    y = x.copy()
    x1, x2 = x[..., :half], x[..., half:rot]
    y[..., :half] = x1 * c - x2 * s
    y[..., half:rot] = x2 * c + x1 * s
    return y


def _attn_np(orc, d, h, K, V, pos):
    H, nh, nkv, hd, rot = d["hidden"], d["heads"], d["kv_heads"], d["head_dim"], d["rot_dim"]
    deq = lambda raw, r, c: orc.dequantize(8, raw, r * c).reshape(r, c).astype(np.float64)
    gated = bool(d.get("q_gate"))
    Dq, Dkv = nh * hd, nkv * hd
    x = _rms(h.astype(np.float64), d["attn_norm"], d["eps"])
    q = deq(d["wq"], (2 if gated else 1) * Dq, H) @ x
    k = deq(d["wk"], Dkv, H) @ x
    v = deq(d["wv"], Dkv, H) @ x
    if d.get("bq") is not None:
        q, k, v = q + d["bq"], k + d["bk"], v + d["bv"]
    gate = None
    if gated:
        qg = q.reshape(nh, 2, hd)
        q, gate = qg[:, 0, :], qg[:, 1, :]
    q, k, v = q.reshape(nh, hd), k.reshape(nkv, hd), v.reshape(nkv, hd)
    if d.get("q_norm") is not None:
        q = _rms(q, d["q_norm"], d["eps"])
        k = _rms(k, d["k_norm"], d["eps"])
    c, s = _rope_tables(rot, d["rope_theta"], pos)
    q, k = _rope(q, c, s, rot), _rope(k, c, s, rot)
    K.append(k)
    V.append(v)
    Ks, Vs = np.stack(K, 1), np.stack(V, 1)   # [nkv, pos + 1, hd]
    rep, scale = nh // nkv, 1.0 / np.sqrt(hd)
    out = np.zeros((nh, hd))
    for i in range(nh):
        sc = Ks[i // rep] @ q[i] * scale
        if d.get("window"):
            sc[: max(0, pos + 1 - d["window"])] = -np.inf
        m = sc.max()
        if d.get("sinks") is not None:
            m = max(m, float(d["sinks"][i]))
        e = np.exp(sc - m)
        den = e.sum() + (np.exp(float(d["sinks"][i]) - m) if d.get("sinks") is not None else 0.0)
        out[i] = (e / den) @ Vs[i // rep]
    if gated:
        out = out / (1.0 + np.exp(-gate))
    y = deq(d["wo"], H, Dq) @ out.reshape(-1)
    if d.get("bo") is not None:
        y = y + d["bo"]
    return h.astype(np.float64) + y


@pytest.mark.parametrize("shape", [
    dict(H=256, nh=8, nkv=2, hd=32, rot=32, window=4, sinks=True, bias=True, steps=9),     # GPT-OSS-like SWA
    dict(H=256, nh=4, nkv=2, hd=64, rot=64, qk_norm=True, theta=1e6, steps=6),            # Qwen3-like
    dict(H=256, nh=4, nkv=1, hd=256, rot=64, qk_norm=True, theta=1e7, q_gate=True, steps=6),   # hybrid gated
])
def test_oracle_attention_matches_numpy(orc, shape):
    shape = dict(shape)
    steps = shape.pop("steps")
    d = _attn_layer(3, **shape)
    st = orc.AttnState(d, attn_mode=0)
    K, V = [], []
    rng = np.random.default_rng(5)
    for pos in range(steps):
        h = rng.standard_normal(d["hidden"]).astype(np.float32)
        got = st.step(h)
        want = _attn_np(orc, d, h, K, V, pos)
        dy, wy = got.astype(np.float64) - h, want - h   # the attention output itself
        assert np.abs(dy - wy).max() / np.abs(wy).max() < 1e-5, f"position {pos}"
