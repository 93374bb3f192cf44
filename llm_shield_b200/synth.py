"""Seeded synthetic Shieldstral-shaped checkpoints (host-side input generation).

Tensor names and layout follow the reference converter
(tools/convert_shieldstral_to_gguf.py:186-203, 277-353): ``token_embd.weight``
quantized (tied head, no ``output.weight``), ``blk.N.attn_q/k/v/output``,
``blk.N.ffn_gate/up/down`` quantized, ``*_norm.weight`` kept F32.  Weights are
N(0, 0.02), norm gains 1 + N(0, 0.01), quantized with gguf-py's block
semantics by libshield_synth.so.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

from . import _build

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1", Q8_0: "Q8_0"}
TYPE_BY_NAME = {v: k for k, v in TYPE_NAMES.items()}
BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q5_0: 22, Q5_1: 24, Q8_0: 34}

# Verdict surface forms at the real vocabulary's ids (7 "yes" forms, 9 "no" forms).
YES_IDS = [13059, 13830, 14842, 16860, 51935, 57445, 58918]
NO_IDS = [1836, 2649, 3501, 4753, 14089, 16071, 45344, 50510, 50683]
FIRST_ORDINARY_ID = 1000  # ids 0..999 are Tekken's control tokens


def row_bytes(qtype: int, cols: int) -> int:
    if qtype == F32:
        return cols * 4
    if qtype == F16:
        return cols * 2
    return cols // 32 * BLOCK_BYTES[qtype]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = _build.synth_lib_path()
        if not path.exists():
            _build.build_synth()
        L = C.CDLL(str(path))
        L.synth_quantize.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_void_p]
        L.synth_tensor.argtypes = [C.c_int, C.c_int64, C.c_int64, C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                                   C.c_void_p, C.c_void_p, C.c_int]
        _lib = L
    return _lib


def threads() -> int:
    env = os.environ.get("SHIELD_SYNTH_THREADS")
    if env:
        return max(1, int(env))
    return max(1, len(os.sched_getaffinity(0)))


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.empty(row_bytes(qtype, x.size), np.uint8)
    if lib().synth_quantize(qtype, x.ctypes.data, x.size, out.ctypes.data) != 0:
        raise ValueError("unsupported type or length")
    return out


def tensor(qtype: int, rows: int, cols: int, seed: int, stream: int, mean: float = 0.0, std: float = 0.02,
           want_float: bool = False):
    """rows x cols of N(mean, std) quantized to qtype; optionally also the floats."""
    out = np.empty(rows * row_bytes(qtype, cols), np.uint8)
    fl = np.empty((rows, cols), np.float32) if want_float else None
    rc = lib().synth_tensor(qtype, rows, cols, seed, stream, mean, std, out.ctypes.data,
                            fl.ctypes.data if fl is not None else None, threads())
    if rc != 0:
        raise ValueError("unsupported type or shape")
    return (out, fl) if want_float else out


@dataclass
class ModelSpec:
    n_layers: int = 26
    hidden: int = 3072
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 9216
    vocab: int = 131072
    rms_eps: float = 1e-5
    rope_theta: float = 1.0e6
    # YaRN as Shieldstral's params.json has it: factor 16 over a 16384 window,
    # magnitude correction cancelled (mscale == mscale_all_dim == 1).
    yarn_factor: float = 16.0
    yarn_orig_ctx: int = 16384
    yarn_beta_fast: float = 32.0
    yarn_beta_slow: float = 1.0
    attn_temperature_beta: float = 0.1
    qtype: int = Q4_0
    seed: int = 20261201
    yes_ids: list = field(default_factory=lambda: list(YES_IDS))
    no_ids: list = field(default_factory=lambda: list(NO_IDS))

    @property
    def qdim(self):
        return self.n_heads * self.head_dim

    @property
    def kvdim(self):
        return self.n_kv_heads * self.head_dim

    @property
    def verdict_ids(self):
        return list(self.yes_ids) + list(self.no_ids)


SHIELDSTRAL_3B = ModelSpec()


def small_spec(qtype: int = Q4_0, n_layers: int = 2, seed: int = 7) -> ModelSpec:
    """A reduced model with the same structure (GQA 4:1, head_dim 128) for fast tests."""
    return ModelSpec(n_layers=n_layers, hidden=256, n_heads=4, n_kv_heads=1, head_dim=128, ffn=512,
                     vocab=2048, qtype=qtype, seed=seed, yes_ids=[1013, 1500, 2001], no_ids=[1100, 1999])


def tensor_list(spec: ModelSpec):
    """(name, type, rows, cols, mean, std) for every tensor, in upload order."""
    q = spec.qtype
    out = [("token_embd.weight", q, spec.vocab, spec.hidden, 0.0, 0.02),
           ("output_norm.weight", F32, 1, spec.hidden, 1.0, 0.01)]
    for l in range(spec.n_layers):
        p = f"blk.{l}."
        out += [
            (p + "attn_norm.weight", F32, 1, spec.hidden, 1.0, 0.01),
            (p + "attn_q.weight", q, spec.qdim, spec.hidden, 0.0, 0.02),
            (p + "attn_k.weight", q, spec.kvdim, spec.hidden, 0.0, 0.02),
            (p + "attn_v.weight", q, spec.kvdim, spec.hidden, 0.0, 0.02),
            (p + "attn_output.weight", q, spec.hidden, spec.qdim, 0.0, 0.02),
            (p + "ffn_norm.weight", F32, 1, spec.hidden, 1.0, 0.01),
            (p + "ffn_gate.weight", q, spec.ffn, spec.hidden, 0.0, 0.02),
            (p + "ffn_up.weight", q, spec.ffn, spec.hidden, 0.0, 0.02),
            (p + "ffn_down.weight", q, spec.hidden, spec.ffn, 0.0, 0.02),
        ]
    return out


def make_model(spec: ModelSpec, want_float: bool = False) -> dict:
    """{name: {"type", "rows", "cols", "data" (uint8 bytes), ["float"]}}."""
    tensors = {}
    for stream, (name, qt, rows, cols, mean, std) in enumerate(tensor_list(spec)):
        if want_float:
            data, fl = tensor(qt, rows, cols, spec.seed, stream, mean, std, want_float=True)
        else:
            data, fl = tensor(qt, rows, cols, spec.seed, stream, mean, std), None
        t = {"type": qt, "rows": rows, "cols": cols, "data": data}
        if fl is not None:
            t["float"] = fl
        tensors[name] = t
    return tensors


def random_requests(n_req: int, lengths, seed: int, vocab: int) -> list[np.ndarray]:
    rng = np.random.default_rng(seed)
    return [rng.integers(FIRST_ORDINARY_ID, vocab, size=int(s), dtype=np.int32) for s in lengths]


def lognormal_lengths(n_req: int, seed: int, median: float = 300.0, sigma: float = 0.6,
                      lo: int = 32, hi: int = 4096) -> np.ndarray:
    rng = np.random.default_rng(seed)
    s = np.round(rng.lognormal(np.log(median), sigma, size=n_req))
    return np.clip(s, lo, hi).astype(np.int64)
