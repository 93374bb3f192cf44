"""ctypes binding of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

The oracle is a C restatement of the reference's CPU integer path
(curiosity-ai/llm-shield: IntegerGemm.cs, QuantMatMul.cs, Kernels.cs, Rope.cs,
MinistralModel.cs, ShieldstralModerator.cs).  It is the checker the CUDA
library is compared against.  Only tests/, the smoke check in
__graft_entry__.py and the cpu_baseline leg of bench.py may import it; the
product package never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
# capture points (IActivationSink names, MinistralModel.cs:212-237)
CAP_OUTPUT, CAP_Q_ROPE, CAP_K_ROPE, CAP_V, CAP_ATTN_WEIGHTED, CAP_POST_ATTN, CAP_ATTN_NORM = range(7)
BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q5_0: 22, Q5_1: 24, Q8_0: 34}


def build() -> Path:
    """Compiles liboracle.so with the oracle's Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


class OrcConfig(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
        ("vocab", C.c_int32), ("rms_eps", C.c_float), ("rope_half", C.c_int32),
        ("rope_freqs", C.c_float * 256), ("rope_mscale", C.c_float),
        ("attn_temperature_beta", C.c_float), ("rope_orig_ctx", C.c_int32),
        ("attn_operand_bits", C.c_int32),
    ]


class OrcRopeParams(C.Structure):
    _fields_ = [
        ("rope_dim", C.c_int32), ("freq_base", C.c_float), ("scale_factor", C.c_float),
        ("yarn", C.c_int32), ("orig_ctx", C.c_int32), ("beta_fast", C.c_float),
        ("beta_slow", C.c_float), ("ext_factor", C.c_float), ("mscale", C.c_float),
        ("mscale_all_dim", C.c_float), ("attn_factor", C.c_float),
    ]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        L.orc_block_bytes.argtypes = [C.c_int]
        L.orc_row_bytes.argtypes = [C.c_int, C.c_int64]
        L.orc_row_bytes.restype = C.c_int64
        L.orc_half_to_float.argtypes = [C.c_uint16]
        L.orc_half_to_float.restype = C.c_float
        L.orc_set_simd_level.argtypes = [C.c_int]
        L.orc_quantize_activations.argtypes = [P, C.c_int, P, P, P]
        L.orc_unpack_block.argtypes = [C.c_int, P, P, P, P]
        L.orc_dequantize.argtypes = [C.c_int, P, P, C.c_int64]
        L.orc_qmatmul.argtypes = [C.c_int, P, C.c_int64, C.c_int64, P, C.c_int64, P, P, C.c_int64, C.c_int]
        L.orc_qmatmul_scalar.argtypes = [C.c_int, P, C.c_int64, C.c_int64, P, C.c_int64, P]
        L.orc_block_dots.argtypes = [C.c_int, P, C.c_int64, C.c_int64, P, C.c_int64, P]
        L.orc_rmsnorm.argtypes = [P, P, C.c_int, C.c_float, P]
        L.orc_softmax.argtypes = [P, C.c_int]
        L.orc_expf.argtypes = [C.c_float]
        L.orc_expf.restype = C.c_float
        L.orc_swiglu.argtypes = [P, P, P, C.c_int]
        L.orc_rope_freqs.argtypes = [C.POINTER(OrcRopeParams), P, P]
        L.orc_rope_apply.argtypes = [P, C.c_int, C.c_int, C.c_int, P, C.c_int, C.c_float]
        L.orc_model_create.argtypes = [C.POINTER(OrcConfig)]
        L.orc_model_create.restype = C.c_void_p
        L.orc_model_free.argtypes = [P]
        L.orc_model_set_tensor.argtypes = [P, C.c_char_p, C.c_int, C.c_int64, C.c_int64, P]
        L.orc_model_forward.argtypes = [P, P, C.c_int, P, C.c_int, P, C.c_int, C.c_int, C.c_int, P]
        L.orc_score.argtypes = [P, C.c_int, C.c_int, P, P, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def quantize_activations(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    q = np.empty(n, np.int8)
    d = np.empty(n // 32, np.float32)
    s = np.empty(n // 32, np.int32)
    lib().orc_quantize_activations(_p(x), n, _p(q), _p(d), _p(s))
    return q, d, s


def dequantize(qtype: int, raw: np.ndarray, count: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(count, np.float32)
    if lib().orc_dequantize(qtype, _p(raw), _p(out), count) != 0:
        raise ValueError("bad type or count")
    return out


def qmatmul(qtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, tokens: int,
            row_ids=None, threads: int | None = None) -> np.ndarray:
    """QuantMatMul.ForwardAsync / ForwardRowsAsync on the integer path."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if row_ids is not None:
        ids = np.ascontiguousarray(row_ids, dtype=np.int32)
        y = np.empty((tokens, ids.size), np.float32)
        rc = lib().orc_qmatmul(qtype, _p(w), rows, cols, _p(x), tokens, _p(y), _p(ids), ids.size,
                               threads or default_threads())
    else:
        y = np.empty((tokens, rows), np.float32)
        rc = lib().orc_qmatmul(qtype, _p(w), rows, cols, _p(x), tokens, _p(y), None, 0,
                               threads or default_threads())
    if rc == -2:
        raise IndexError("row id outside the matrix")
    if rc != 0:
        raise ValueError("unsupported type or shape")
    return y


def qmatmul_scalar(qtype, w, rows, cols, x, tokens):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty((tokens, rows), np.float32)
    if lib().orc_qmatmul_scalar(qtype, _p(w), rows, cols, _p(x), tokens, _p(y)) != 0:
        raise ValueError("unsupported type or shape")
    return y


def block_dots(qtype, w, rows, cols, x, tokens) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = np.empty((tokens, rows, cols // 32), np.int32)
    if lib().orc_block_dots(qtype, _p(w), rows, cols, _p(x), tokens, _p(d)) != 0:
        raise ValueError("unsupported type or shape")
    return d


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(w), x.size, eps, _p(y))
    return y


def softmax(x):
    x = np.array(x, np.float32, copy=True)
    lib().orc_softmax(_p(x), x.size)
    return x


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.array(u, np.float32, copy=True)
    out = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(u), _p(out), g.size)
    return out


def rope_freqs(rope_dim, freq_base, scale_factor=1.0, yarn=False, orig_ctx=0, beta_fast=32.0,
               beta_slow=1.0, ext_factor=1.0, mscale=0.0, mscale_all_dim=0.0, attn_factor=1.0):
    p = OrcRopeParams(rope_dim, freq_base, scale_factor, int(yarn), orig_ctx, beta_fast, beta_slow,
                      ext_factor, mscale, mscale_all_dim, attn_factor)
    f = np.zeros(rope_dim // 2, np.float32)
    ms = np.zeros(1, np.float32)
    lib().orc_rope_freqs(C.byref(p), _p(f), _p(ms))
    return f, float(ms[0])


def rope_apply(data, heads, head_dim, position, freqs, mscale):
    d = np.array(data, np.float32, copy=True)
    f = np.ascontiguousarray(freqs, np.float32)
    lib().orc_rope_apply(_p(d), heads, head_dim, position, _p(f), f.size, mscale)
    return d


def score(verdict_logits, n_yes, n_no):
    v = np.ascontiguousarray(verdict_logits, np.float32)
    out = np.zeros(3, np.float32)
    lib().orc_score(_p(v), n_yes, n_no, _p(out[0:]), _p(out[1:]), _p(out[2:]))
    return float(out[0]), float(out[1]), float(out[2])


class Model:
    """MinistralModel over borrowed tensor bytes (the GGUF names of MinistralModel.cs:74-96)."""

    def __init__(self, cfg: dict, tensors: dict):
        c = OrcConfig()
        c.n_layers, c.hidden, c.n_heads = cfg["n_layers"], cfg["hidden"], cfg["n_heads"]
        c.n_kv_heads, c.head_dim, c.ffn, c.vocab = cfg["n_kv_heads"], cfg["head_dim"], cfg["ffn"], cfg["vocab"]
        c.rms_eps = cfg["rms_eps"]
        freqs = np.asarray(cfg["rope_freqs"], np.float32)
        c.rope_half = freqs.size
        for i, f in enumerate(freqs):
            c.rope_freqs[i] = float(f)
        c.rope_mscale = cfg["rope_mscale"]
        c.attn_temperature_beta = cfg.get("attn_temperature_beta", 0.0)
        c.rope_orig_ctx = cfg.get("rope_orig_ctx", 0)
        c.attn_operand_bits = cfg.get("attn_operand_bits", 0)
        self.cfg = cfg
        self._keep = []
        self.h = lib().orc_model_create(C.byref(c))
        if not self.h:
            raise ValueError("bad config")
        for name, t in tensors.items():
            data = np.ascontiguousarray(t["data"])
            self._keep.append(data)
            rc = lib().orc_model_set_tensor(self.h, name.encode(), t["type"], t["rows"], t["cols"], _p(data))
            if rc != 0:
                raise ValueError(f"tensor {name} rejected")

    def capture_width(self, what: int) -> int:
        c = self.cfg
        if what in (CAP_Q_ROPE, CAP_ATTN_WEIGHTED):
            return c["n_heads"] * c["head_dim"]
        if what in (CAP_K_ROPE, CAP_V):
            return c["n_kv_heads"] * c["head_dim"]
        return c["hidden"]

    def forward(self, ids, vocab_ids, threads: int | None = None, capture_layer: int = -1,
                capture_what: int = 0):
        ids = np.ascontiguousarray(ids, np.int32)
        v = np.ascontiguousarray(vocab_ids, np.int32)
        out = np.empty(v.size, np.float32)
        cap = None
        if capture_layer >= 0:
            cap = np.empty((ids.size, self.capture_width(capture_what)), np.float32)
        rc = lib().orc_model_forward(self.h, _p(ids), ids.size, _p(v), v.size, _p(out),
                                     threads or default_threads(), capture_layer, capture_what,
                                     _p(cap) if cap is not None else None)
        if rc != 0:
            raise ValueError(f"forward failed ({rc})")
        return (out, cap) if cap is not None else out

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None
