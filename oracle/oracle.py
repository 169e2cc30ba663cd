"""ctypes view of the CPU oracle (libmsoracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of bench.py, as the checker or the
timed CPU restatement of the reference.  The product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libmsoracle.so")
_lib = None

F32, F16, Q8_0, Q4_K, Q6_K, MXFP4 = 0, 1, 8, 12, 14, 39

_fp = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_vp = C.c_void_p


class MoeLayer(C.Structure):
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("n_experts", C.c_int), ("top_k", C.c_int),
                ("gate_q", C.c_int), ("up_q", C.c_int), ("down_q", C.c_int),
                ("gate", _vp), ("up", _vp), ("down", _vp),
                ("gate_bias", _fp), ("up_bias", _fp), ("down_bias", _fp),
                ("router_w", _fp), ("router_b", _fp),
                ("oai_swiglu", C.c_int), ("norm_topk_prob", C.c_int)]


class AttnLayer(C.Structure):
    _fields_ = [("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int), ("head_dim", C.c_int),
                ("rot_dim", C.c_int), ("eps", C.c_float), ("rope_theta", C.c_float), ("window", C.c_int),
                ("attn_mode", C.c_int), ("attn_norm", _fp), ("wq", _vp), ("wk", _vp), ("wv", _vp), ("wo", _vp),
                ("bq", _fp), ("bk", _fp), ("bv", _fp), ("bo", _fp), ("sinks", _fp), ("q_norm", _fp),
                ("k_norm", _fp), ("q_gate", C.c_int)]


class DeltaNetLayer(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_k_heads", C.c_int), ("head_k_dim", C.c_int), ("n_v_heads", C.c_int),
                ("head_v_dim", C.c_int), ("conv_kernel", C.c_int), ("eps", C.c_float),
                ("qkv_q", C.c_int), ("qkv", _vp), ("gate_q", C.c_int), ("gate", _vp), ("ba_q", C.c_int), ("ba", _vp),
                ("out_q", C.c_int), ("out", _vp), ("conv1d", _fp), ("ssm_a", _fp), ("dt_bias", _fp), ("norm", _fp)]


def build() -> str:
    """Compile the oracle with its Makefile (g++ only; no reference sources involved)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.orc_fp16_to_f32.restype = C.c_float
        L.orc_fp16_to_f32.argtypes = [C.c_uint16]
        L.orc_e8m0_to_f32_half.restype = C.c_float
        L.orc_e8m0_to_f32_half.argtypes = [C.c_uint8]
        L.orc_dequantize.argtypes = [C.c_int, _vp, C.c_int64, _fp]
        L.orc_mxfp4_matvec_mul.argtypes = [_vp, _fp, C.c_int64, C.c_int64, _fp]
        L.orc_gemv.argtypes = [C.c_int, _vp, C.c_int64, C.c_int64, _fp, _fp]
        L.orc_q8_0_gemv.argtypes = [_vp, C.c_int64, C.c_int64, _fp, _fp, C.c_int]
        L.orc_quantize_q8_0.argtypes = [_fp, C.c_int64, _vp]
        L.orc_rms_norm.argtypes = [_fp, _fp, _fp, C.c_int64, C.c_int64, C.c_float]
        L.orc_rope_tables.argtypes = [C.c_int, C.c_int, C.c_double, _fp, _fp]
        L.orc_swiglu_oai.argtypes = [_fp, _fp, _fp, C.c_int64, C.c_float, C.c_float]
        L.orc_silu_and_mul.argtypes = [_fp, _fp, _fp, C.c_int64]
        L.orc_top_k_routing.argtypes = [_fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _i32p, _fp]
        L.orc_moe_forward.argtypes = [C.POINTER(MoeLayer), _fp, C.c_int, _fp, _i32p, _fp]
        L.orc_moe_forward_range.argtypes = [C.POINTER(MoeLayer), _fp, C.c_int, _fp, C.c_int, C.c_int]
        L.orc_rope.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, _fp]
        L.orc_sample.argtypes = [_fp, C.c_int, C.POINTER(C.c_uint32), C.c_float, C.c_float, C.c_float, C.c_float]
        L.orc_sample.restype = C.c_int
        L.orc_attn_decode.argtypes = [C.POINTER(AttnLayer), _fp, _fp, C.c_int, _fp]
        L.orc_deltanet_step.argtypes = [C.POINTER(DeltaNetLayer), _fp, _fp, _fp, _fp]
        L.orc_shared_expert.argtypes = [C.c_int, _vp, _vp, C.c_int, _vp, _fp, C.c_int, C.c_int, _fp, _fp]
        L.orc_model_open.restype = _vp
        L.orc_model_open.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_int]
        L.orc_model_set_attn_mode.argtypes = [_vp, C.c_int]
        L.orc_model_set_dynamic_k.argtypes = [_vp, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_model_set_dynamic_k.restype = C.c_int
        L.orc_model_router_stats.argtypes = [_vp, _fp, _i32p]
        L.orc_model_set_threads.argtypes = [_vp, C.c_int]
        L.orc_model_forward.argtypes = [_vp, _i32p, C.c_int, _fp]
        L.orc_model_generate.argtypes = [_vp, _i32p, C.c_int, C.c_int, _i32p]
        L.orc_model_vocab.argtypes = [_vp]
        L.orc_model_hidden.argtypes = [_vp]
        L.orc_model_seq_len.argtypes = [_vp]
        L.orc_model_clear_cache.argtypes = [_vp]
        L.orc_model_last_hidden.argtypes = [_vp, _fp]
        L.orc_model_last_routing.argtypes = [_vp, _i32p, _fp]
        L.orc_model_layer_trace.argtypes = [_vp, _fp, _fp]
        L.orc_model_lm_head.argtypes = [_vp, _fp, _fp]
        L.orc_model_destroy.argtypes = [_vp]
        _lib = L
    return _lib


def _f(a: np.ndarray):
    return a.ctypes.data_as(_fp)


def _i(a: np.ndarray):
    return a.ctypes.data_as(_i32p)


def dequantize(qtype: int, blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    b = np.ascontiguousarray(blocks)
    if lib().orc_dequantize(qtype, b.ctypes.data, n, _f(out)) != 0:
        raise ValueError(f"unsupported qtype {qtype}")
    return out


def gemv(qtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    lib().orc_gemv(qtype, w.ctypes.data, rows, cols, _f(x), _f(y))
    return y


def mxfp4_matvec_mul(w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    lib().orc_mxfp4_matvec_mul(w.ctypes.data, _f(x), rows, cols, _f(y))
    return y


def q8_0_gemv(w: np.ndarray, rows: int, cols: int, x: np.ndarray, mode: int = 1) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    lib().orc_q8_0_gemv(w.ctypes.data, rows, cols, _f(x), _f(y), mode)
    return y


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib().orc_quantize_q8_0(_f(x), x.size, out.ctypes.data)
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    dim = x.shape[-1]
    lib().orc_rms_norm(_f(x), _f(w), _f(y), x.size // dim, dim, eps)
    return y


def rope_tables(rot_dim: int, max_seq: int, theta: float):
    c = np.empty((max_seq, rot_dim // 2), dtype=np.float32)
    s = np.empty_like(c)
    lib().orc_rope_tables(rot_dim, max_seq, theta, _f(c), _f(s))
    return c, s


def swiglu_oai(g, u, alpha=1.702, limit=7.0):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    o = np.empty_like(g)
    lib().orc_swiglu_oai(_f(g), _f(u), _f(o), g.size, alpha, limit)
    return o


def silu_and_mul(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    o = np.empty_like(g)
    lib().orc_silu_and_mul(_f(g), _f(u), _f(o), g.size)
    return o


def top_k_routing(logits: np.ndarray, k: int, normalize: bool, softmax_weight: bool):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    if logits.ndim == 1:
        logits = logits[None]
    n, e = logits.shape
    idx = np.empty((n, k), dtype=np.int32)
    w = np.empty((n, k), dtype=np.float32)
    lib().orc_top_k_routing(_f(logits), n, e, k, int(normalize), int(softmax_weight), _i(idx), _f(w))
    return idx, w


def moe_forward(layer: dict, x: np.ndarray, expert_range=None):
    """One MoE FFN layer on the default CPU path.  ``layer`` holds numpy arrays:
    gate/up/down (raw stacked blocks), *_bias, router_w, router_b, and ints."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n_tok = x.size // layer["hidden"]
    keep = []

    def ptr(a, fp=False):
        if a is None:
            return None if not fp else _fp()
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data_as(_fp) if fp else a.ctypes.data

    L = MoeLayer(layer["hidden"], layer["inter"], layer["n_experts"], layer["top_k"],
                 layer["gate_q"], layer["up_q"], layer["down_q"],
                 ptr(layer["gate"]), ptr(layer["up"]), ptr(layer["down"]),
                 ptr(layer.get("gate_bias"), True), ptr(layer.get("up_bias"), True),
                 ptr(layer.get("down_bias"), True), ptr(layer["router_w"], True),
                 ptr(layer.get("router_b"), True), int(layer["oai_swiglu"]), int(layer["norm_topk_prob"]))
    out = np.empty((n_tok, layer["hidden"]), dtype=np.float32)
    idx = np.empty((n_tok, layer["top_k"]), dtype=np.int32)
    w = np.empty((n_tok, layer["top_k"]), dtype=np.float32)
    if expert_range is not None:
        lib().orc_moe_forward_range(C.byref(L), _f(x), n_tok, _f(out), int(expert_range[0]), int(expert_range[1]))
        return out, None, None
    lib().orc_moe_forward(C.byref(L), _f(x), n_tok, _f(out), _i(idx), _f(w))
    return out, idx, w


def sample(logits, counts=None, temperature=1.0, top_p=1.0, penalty=1.0, r=0.5):
    """SamplingParams::sample (engine.rs:124-208) with the draw r in [0, 1)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    cp = None
    if counts is not None:
        cts = np.ascontiguousarray(counts, dtype=np.uint32)
        cp = cts.ctypes.data_as(C.POINTER(C.c_uint32))
    return int(lib().orc_sample(_f(lg), lg.size, cp, float(temperature), float(top_p), float(penalty), float(r)))


def rope(x, cos, sin, n_tok, heads, hd, rot):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_rope(_f(x), _f(np.ascontiguousarray(cos, np.float32)), _f(np.ascontiguousarray(sin, np.float32)),
                   n_tok, heads, hd, rot, _f(y))
    return y


class AttnState:
    """One attention half-layer with its f32 K/V history (layer.rs:511-749), stepped a token at a time."""

    def __init__(self, d: dict, attn_mode: int = 1):
        self.keep = []

        def ptr(a, fp=False):
            if a is None:
                return _fp() if fp else None
            a = np.ascontiguousarray(a)
            self.keep.append(a)
            return a.ctypes.data_as(_fp) if fp else a.ctypes.data
        self.d = d
        self.L = AttnLayer(d["hidden"], d["heads"], d["kv_heads"], d["head_dim"], d["rot_dim"], d["eps"],
                           d["rope_theta"], d.get("window", 0), attn_mode, ptr(d["attn_norm"], True),
                           ptr(d["wq"]), ptr(d["wk"]), ptr(d["wv"]), ptr(d["wo"]), ptr(d.get("bq"), True),
                           ptr(d.get("bk"), True), ptr(d.get("bv"), True), ptr(d.get("bo"), True),
                           ptr(d.get("sinks"), True), ptr(d.get("q_norm"), True), ptr(d.get("k_norm"), True),
                           int(d.get("q_gate", 0)))
        self.K = np.zeros((d["kv_heads"], 0, d["head_dim"]), np.float32)
        self.V = np.zeros_like(self.K)

    def step(self, h: np.ndarray) -> np.ndarray:
        """h + attention(RMSNorm(h)) at the next position"""
        pos = self.K.shape[1]
        z = np.zeros((self.K.shape[0], 1, self.K.shape[2]), np.float32)
        K = np.ascontiguousarray(np.concatenate([self.K, z], 1))
        V = np.ascontiguousarray(np.concatenate([self.V, z], 1))
        out = np.ascontiguousarray(h, dtype=np.float32).copy()
        lib().orc_attn_decode(C.byref(self.L), _f(K), _f(V), pos, _f(out))
        self.K, self.V = K, V
        return out


def deltanet_layer(d: dict, keep: list) -> DeltaNetLayer:
    """ctypes view of a DeltaNet layer dict (numpy arrays + ints); keep holds the buffers alive"""
    def ptr(a, fp=False):
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data_as(_fp) if fp else a.ctypes.data
    return DeltaNetLayer(d["hidden"], d["n_k_heads"], d["head_k_dim"], d["n_v_heads"], d["head_v_dim"],
                         d["conv_kernel"], d["eps"], d["qkv_q"], ptr(d["qkv"]), d["gate_q"], ptr(d["gate"]),
                         d["ba_q"], ptr(d["ba"]), d["out_q"], ptr(d["out"]), ptr(d["conv1d"], True),
                         ptr(d["ssm_a"], True), ptr(d["dt_bias"], True), ptr(d["norm"], True))


def deltanet_step(d: dict, x, conv_state, rec_state) -> np.ndarray:
    """one DeltaNet decode token; conv_state / rec_state (f32 numpy) are updated in place"""
    keep = []
    L = deltanet_layer(d, keep)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(d["hidden"], np.float32)
    if lib().orc_deltanet_step(C.byref(L), _f(x), _f(conv_state), _f(rec_state), _f(y)) != 0:
        raise ValueError("unsupported qtype")
    return y


def shared_expert(gu_q, gate, up, down_q, down, gate_inp, hidden, inter, x, y):
    """y += shared expert(x), in place"""
    x = np.ascontiguousarray(x, dtype=np.float32)
    gi = np.ascontiguousarray(gate_inp, dtype=np.float32) if gate_inp is not None else None
    if lib().orc_shared_expert(gu_q, np.ascontiguousarray(gate).ctypes.data, np.ascontiguousarray(up).ctypes.data,
                               down_q, np.ascontiguousarray(down).ctypes.data, _f(gi) if gi is not None else _fp(),
                               hidden, inter, _f(x), _f(y)) != 0:
        raise ValueError("unsupported qtype")
    return y


class Model:
    """Whole-model oracle over a GGUF file (engine.rs forward/generate)."""

    def __init__(self, path: str, max_seq_len: int = 4096, attn_mode: int = 1, threads: int = 0):
        err = C.create_string_buffer(512)
        self.h = lib().orc_model_open(path.encode(), max_seq_len, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        lib().orc_model_set_attn_mode(self.h, attn_mode)
        if threads:
            lib().orc_model_set_threads(self.h, threads)
        self.vocab = lib().orc_model_vocab(self.h)
        self.hidden = lib().orc_model_hidden(self.h)

    def forward(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.vocab, dtype=np.float32)
        rc = lib().orc_model_forward(self.h, _i(t), t.size, _f(logits))
        if rc != 0:
            raise RuntimeError(f"oracle forward failed ({rc})")
        return logits

    def generate(self, prompt, max_new: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(max_new, dtype=np.int32)
        n = lib().orc_model_generate(self.h, _i(p), p.size, max_new, _i(out))
        if n < 0:
            raise RuntimeError("oracle generate failed")
        return out[:n]

    def last_hidden(self) -> np.ndarray:
        o = np.empty(self.hidden, dtype=np.float32)
        lib().orc_model_last_hidden(self.h, _f(o))
        return o

    def last_routing(self, layers: int, k: int):
        """routed experts and weights of the last position, [layers, k] each"""
        idx = np.empty(layers * k, np.int32)
        w = np.empty(layers * k, np.float32)
        lib().orc_model_last_routing(self.h, _i(idx), _f(w))
        return idx.reshape(layers, k), w.reshape(layers, k)

    def set_dynamic_k(self, enable: bool, k_min: int = 2, k_max: int = 0, layer_adaptive: bool = False):
        if lib().orc_model_set_dynamic_k(self.h, int(enable), k_min, k_max, int(layer_adaptive)) != 0:
            raise ValueError("invalid dynamic-K range")

    def router_stats(self, layers: int):
        """(router entropy [layers] f32, K used [layers]) of the last forward"""
        ent = np.empty(layers, np.float32)
        k = np.empty(layers, np.int32)
        lib().orc_model_router_stats(self.h, _f(ent), _i(k))
        return ent, k

    def layer_trace(self, layers: int, experts: int):
        """(hidden after each layer [layers, H], router logits per layer [layers, E]), last position"""
        hid = np.empty(layers * self.hidden, np.float32)
        lg = np.empty(layers * experts, np.float32)
        lib().orc_model_layer_trace(self.h, _f(hid), _f(lg))
        return hid.reshape(layers, self.hidden), lg.reshape(layers, experts)

    def lm_head(self, hidden: np.ndarray) -> np.ndarray:
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        out = np.empty(self.vocab, dtype=np.float32)
        lib().orc_model_lm_head(self.h, _f(hidden), _f(out))
        return out

    def clear_cache(self):
        lib().orc_model_clear_cache(self.h)

    def close(self):
        if self.h:
            lib().orc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
