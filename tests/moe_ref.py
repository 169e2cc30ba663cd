"""float64 numpy restatement of one MoE FFN layer for a GIVEN routing (layer.rs:1367-1895 for one
token: per routed slot SwiGLU (OAI clamp form, activation.rs:13-45) of the gate / up GEMVs, the down
GEMV and bias, weighted and summed in ascending expert id; repeated experts count once per slot).
Test infrastructure: used where a test supplies its own routing, which the oracle's layer cannot take."""
import numpy as np

from moe_stream_b200 import gguf as G


def moe_with_routing(orc, L, x, idx, wts):
    H, I, E = L["hidden"], L["inter"], L["n_experts"]
    gsz = G.raw_size(L["gate_q"], I * H)
    dsz = G.raw_size(L["down_q"], H * I)
    x = np.asarray(x, np.float64).reshape(H)
    out = np.zeros(H)
    deq = lambda q, raw, n: orc.dequantize(q, np.ascontiguousarray(raw), n).astype(np.float64)
    for k in np.argsort(np.asarray(idx), kind="stable"):
        e = int(idx[k])
        g = deq(L["gate_q"], L["gate"][e * gsz:(e + 1) * gsz], I * H).reshape(I, H) @ x
        u = deq(L["up_q"], L["up"][e * gsz:(e + 1) * gsz], I * H).reshape(I, H) @ x
        if L.get("gate_bias") is not None:
            g = g + L["gate_bias"].reshape(E, I)[e]
            u = u + L["up_bias"].reshape(E, I)[e]
        with np.errstate(over="ignore"):   # exp of a large negative gate: sigmoid 0, as in f32
            if L["oai_swiglu"]:
                g = np.minimum(g, 7.0)
                u = np.clip(u, -7.0, 7.0)
                a = g / (1.0 + np.exp(-1.702 * g)) * (u + 1.0)
            else:
                a = g / (1.0 + np.exp(-g)) * u
        y = deq(L["down_q"], L["down"][e * dsz:(e + 1) * dsz], H * I).reshape(H, I) @ a
        if L.get("down_bias") is not None:
            y = y + L["down_bias"].reshape(E, H)[e]
        out += float(wts[k]) * y
    return out
