"""ctypes binding of the C ABI in include/shield_b200.h (libshield_b200.so).

This is the harness-side view of the boundary a .NET host would P/Invoke:
the same entry points, the same arguments, host numpy buffers.  There is no
fallback: if the CUDA library is missing or no GPU is visible, calls fail.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _build
from . import synth

ACT_OUTPUT, ACT_Q_ROPE, ACT_K_ROPE, ACT_V, ACT_ATTN_WEIGHTED, ACT_POST_ATTN, ACT_ATTN_NORM = range(7)
OK, ERR_ARG, ERR_RANGE, ERR_UNSUPPORTED, ERR_CANCELLED, ERR_CUDA, ERR_TIMEOUT, ERR_SHAPE, ERR_STATE, ERR_NOMEM = range(10)


class ShieldError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class ShieldArgumentOutOfRange(ShieldError, IndexError):
    pass


class ShieldCancelled(ShieldError):
    pass


class ShieldConfig(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32), ("ffn", C.c_int32), ("vocab", C.c_int32), ("rms_eps", C.c_float),
        ("rope_freq_base", C.c_float), ("rope_dim", C.c_int32), ("rope_scale_factor", C.c_float),
        ("rope_yarn", C.c_int32), ("rope_orig_ctx", C.c_int32), ("yarn_beta_fast", C.c_float),
        ("yarn_beta_slow", C.c_float), ("yarn_ext_factor", C.c_float), ("yarn_mscale", C.c_float),
        ("yarn_mscale_all_dim", C.c_float), ("rope_attn_factor", C.c_float),
        ("attn_temperature_beta", C.c_float), ("n_rope_freqs", C.c_int32),
        ("rope_freqs", C.POINTER(C.c_float)), ("rope_mscale", C.c_float),
        ("max_positions", C.c_int32), ("max_batch_tokens", C.c_int32),
    ]


class ShieldTiming(C.Structure):
    _fields_ = [("forward_ms", C.c_double), ("gemm_ms", C.c_double), ("gemm_ops", C.c_double),
                ("gemm_bytes", C.c_double), ("gemm_launches", C.c_int64), ("kernel_launches", C.c_int64),
                ("tokens", C.c_int64), ("requests", C.c_int64), ("h2d_bytes", C.c_int64),
                ("d2h_bytes", C.c_int64), ("attn_ms", C.c_double), ("attn_flops", C.c_double)]


EXPORTS = [
    "shield_open", "shield_close", "shield_device_count", "shield_set_config", "shield_upload_tensor",
    "shield_score_batch", "shield_last_logits", "shield_set_prefix", "shield_get_prefix_state", "shield_prefix_length",
    "shield_set_prefix_state", "shield_seq_create", "shield_seq_forward",
    "shield_seq_length", "shield_seq_reset", "shield_seq_release", "shield_qmatmul", "shield_qmatmul_device", "shield_qmatmul_noalloc",
    "shield_debug_block_dots",
    "shield_set_gemm_path", "shield_set_gemm_tile_width", "shield_set_attention_rows", "shield_debug_activation", "shield_set_timing", "shield_read_timing",
    "shield_device_stream", "shield_last_error",
]

_lib = None


def lib() -> C.CDLL:
    """Loads libshield_b200.so (building it in-tree if it is absent)."""
    global _lib
    if _lib is None:
        path = _build.main_lib_path()
        if not path.exists():
            _build.build_main()
        L = C.CDLL(str(path))
        P = C.c_void_p
        L.shield_open.argtypes = [C.c_int32, C.POINTER(P)]
        L.shield_close.argtypes = [P]
        L.shield_close.restype = None
        L.shield_device_count.argtypes = [P]
        L.shield_set_config.argtypes = [P, C.POINTER(ShieldConfig)]
        L.shield_upload_tensor.argtypes = [P, C.c_char_p, C.c_uint32, C.c_int64, C.c_int64, P, C.c_size_t]
        L.shield_score_batch.argtypes = [P, P, P, C.c_int32, P, C.c_int32, C.c_int32, P, P, P, P, P]
        L.shield_last_logits.argtypes = [P, P, P, C.c_int32, P, P]
        L.shield_set_prefix.argtypes = [P, P, C.c_int32]
        L.shield_get_prefix_state.argtypes = [P, P, C.c_int64]
        L.shield_prefix_length.argtypes = [P, C.POINTER(C.c_int32)]
        L.shield_set_prefix_state.argtypes = [P, P, C.c_int32, P, C.c_int64]
        L.shield_seq_create.argtypes = [P, C.c_int32, C.c_int32, C.POINTER(C.c_int64)]
        L.shield_seq_forward.argtypes = [P, P, P, P, C.c_int32, P, P]
        L.shield_seq_length.argtypes = [P, C.c_int64, C.POINTER(C.c_int32)]
        L.shield_seq_reset.argtypes = [P, C.c_int64]
        L.shield_seq_release.argtypes = [P, C.c_int64]
        L.shield_qmatmul.argtypes = [P, C.c_int32, C.c_char_p, P, C.c_int64, P, P, C.c_int32]
        L.shield_qmatmul_device.argtypes = [P, C.c_int32, C.c_char_p, P, C.c_int64, P]
        L.shield_qmatmul_noalloc.argtypes = [P, C.c_int32, C.c_char_p, P, C.c_int64, P]
        L.shield_debug_block_dots.argtypes = [P, C.c_int32, C.c_char_p, P, C.c_int64, P, C.c_int32]
        L.shield_set_gemm_path.argtypes = [P, C.c_int32]
        L.shield_set_gemm_tile_width.argtypes = [P, C.c_int32]
        L.shield_set_attention_rows.argtypes = [P, C.c_int32]
        L.shield_debug_activation.argtypes = [P, C.c_int32, P, C.c_int32, C.c_int32, C.c_int32, P]
        L.shield_device_stream.argtypes = [P, C.c_int32, C.POINTER(P)]
        L.shield_set_timing.argtypes = [P, C.c_int32]
        L.shield_read_timing.argtypes = [P, C.c_int32, C.POINTER(ShieldTiming), C.c_int32]
        L.shield_last_error.restype = C.c_char_p
        for name in EXPORTS:
            f = getattr(L, name)
            if name not in ("shield_close", "shield_last_error", "shield_device_count"):
                f.restype = C.c_int32
        _lib = L
    return _lib


def _check(rc: int):
    if rc == OK:
        return
    msg = (lib().shield_last_error() or b"").decode(errors="replace")
    if rc == ERR_RANGE:
        raise ShieldArgumentOutOfRange(rc, msg)
    if rc == ERR_CANCELLED:
        raise ShieldCancelled(rc, msg)
    raise ShieldError(rc, msg)


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def config_from_spec(spec: "synth.ModelSpec", max_positions: int = 0, max_batch_tokens: int = 0) -> ShieldConfig:
    c = ShieldConfig()
    c.n_layers, c.hidden, c.n_heads, c.n_kv_heads = spec.n_layers, spec.hidden, spec.n_heads, spec.n_kv_heads
    c.head_dim, c.ffn, c.vocab, c.rms_eps = spec.head_dim, spec.ffn, spec.vocab, spec.rms_eps
    c.rope_freq_base, c.rope_dim = spec.rope_theta, spec.head_dim
    yarn = spec.yarn_factor > 1.0 and spec.yarn_orig_ctx > 0
    c.rope_scale_factor = spec.yarn_factor if yarn else 1.0
    c.rope_yarn = int(yarn)
    c.rope_orig_ctx = spec.yarn_orig_ctx
    c.yarn_beta_fast, c.yarn_beta_slow, c.yarn_ext_factor = spec.yarn_beta_fast, spec.yarn_beta_slow, 1.0
    c.yarn_mscale, c.yarn_mscale_all_dim, c.rope_attn_factor = 1.0, 1.0, 1.0
    c.attn_temperature_beta = spec.attn_temperature_beta
    c.n_rope_freqs = 0
    c.rope_mscale = 1.0
    c.max_positions, c.max_batch_tokens = max_positions, max_batch_tokens
    return c


class ShieldContext:
    """One shield_ctx spanning the GPUs in device_mask."""

    def __init__(self, device_mask: int = 1):
        self._h = C.c_void_p()
        _check(lib().shield_open(device_mask, C.byref(self._h)))

    def close(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.shield_close(h)
        self._h = None  # module globals may already be gone at interpreter exit

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def device_count(self) -> int:
        return lib().shield_device_count(self._h)

    def set_config(self, spec, max_positions: int = 0, max_batch_tokens: int = 0):
        self.spec = spec
        c = config_from_spec(spec, max_positions, max_batch_tokens)
        _check(lib().shield_set_config(self._h, C.byref(c)))

    def upload(self, name: str, qtype: int, rows: int, cols: int, data: np.ndarray):
        data = np.ascontiguousarray(data, np.uint8)
        _check(lib().shield_upload_tensor(self._h, name.encode(), qtype, rows, cols, _p(data), data.nbytes))

    def upload_model(self, tensors: dict):
        for name, t in tensors.items():
            self.upload(name, t["type"], t["rows"], t["cols"], t["data"])

    @staticmethod
    def _pack(requests):
        lens = np.array([len(r) for r in requests], np.int64)
        offsets = np.zeros(len(requests) + 1, np.int64)
        np.cumsum(lens, out=offsets[1:])
        ids = np.ascontiguousarray(np.concatenate(requests) if requests else np.zeros(0, np.int32), np.int32)
        return ids, offsets

    def score_batch(self, requests, verdict_ids, n_yes: int, cancel: np.ndarray | None = None):
        """requests: list of int32 arrays. Returns (yes, no, score, logits)."""
        ids, offsets = self._pack(requests)
        return self.score_packed(ids, offsets, verdict_ids, n_yes, cancel)

    def last_logits(self, requests, cancel: np.ndarray | None = None) -> np.ndarray:
        """The whole tied head at each request's last position: (n_req, vocab)."""
        ids, offsets = self._pack(requests)
        out = np.zeros((len(requests), self.spec.vocab), np.float32)
        _check(lib().shield_last_logits(self._h, _p(ids), _p(offsets), len(requests), _p(out),
                                        _p(cancel) if cancel is not None else None))
        return out

    def seq_create(self, capacity: int, device: int = 0) -> int:
        """An empty KV cache for up to `capacity` positions on one GPU."""
        out = C.c_int64()
        _check(lib().shield_seq_create(self._h, device, capacity, C.byref(out)))
        return out.value

    def seq_forward(self, seqs, chunks, want_logits: bool = True, cancel: np.ndarray | None = None):
        """Appends chunks[i] (int32 ids) to sequence seqs[i]; returns the
        (n, vocab) logits at each sequence's new last position."""
        s = np.ascontiguousarray(seqs, np.int64)
        ids, offsets = self._pack(chunks)
        out = np.zeros((len(chunks), self.spec.vocab), np.float32) if want_logits else None
        _check(lib().shield_seq_forward(self._h, _p(s), _p(ids), _p(offsets), len(chunks),
                                        _p(out) if out is not None else None,
                                        _p(cancel) if cancel is not None else None))
        return out

    def seq_length(self, seq: int) -> int:
        out = C.c_int32()
        _check(lib().shield_seq_length(self._h, seq, C.byref(out)))
        return out.value

    def seq_reset(self, seq: int) -> None:
        _check(lib().shield_seq_reset(self._h, seq))

    def seq_release(self, seq: int) -> None:
        _check(lib().shield_seq_release(self._h, seq))

    def set_prefix(self, ids) -> None:
        """Caches the keys and values of a shared prompt prefix on every GPU
        (empty: drop the cache)."""
        a = np.ascontiguousarray(ids, np.int32)
        _check(lib().shield_set_prefix(self._h, _p(a) if a.size else None, a.size))

    def prefix_length(self) -> int:
        """Token ids in the cached prefix (0: none)."""
        n = C.c_int32()
        _check(lib().shield_prefix_length(self._h, C.byref(n)))
        return n.value

    def get_prefix_state(self) -> np.ndarray:
        """The cached prefix's keys and values in KvCache.Snapshot's layout
        (KvCache.cs:102-118): [2][layer][kv head][position][head_dim] floats,
        keys (after RoPE) first, flattened as SystemPromptCache.State."""
        s = self.spec
        out = np.zeros(2 * s.n_layers * s.kvdim * self.prefix_length(), np.float32)
        _check(lib().shield_get_prefix_state(self._h, _p(out), out.size))
        return out

    def set_prefix_state(self, ids, state) -> None:
        """Restores a snapshot (layout of get_prefix_state) as the cached
        prefix for ids on every GPU, without forwarding it
        (SystemPromptCache.RestoreInto, SystemPromptCache.cs:66-74)."""
        a = np.ascontiguousarray(ids, np.int32)
        st = np.ascontiguousarray(state, np.float32).reshape(-1)
        _check(lib().shield_set_prefix_state(self._h, _p(a) if a.size else None, a.size,
                                             _p(st) if st.size else None, st.size))

    def score_packed(self, ids: np.ndarray, offsets: np.ndarray, verdict_ids, n_yes: int, cancel=None):
        v = np.ascontiguousarray(verdict_ids, np.int32)
        n_req = offsets.size - 1
        yes = np.zeros(n_req, np.float32)
        no = np.zeros(n_req, np.float32)
        score = np.zeros(n_req, np.float32)
        logits = np.zeros((n_req, v.size), np.float32)
        _check(lib().shield_score_batch(self._h, _p(ids), _p(np.ascontiguousarray(offsets, np.int64)), n_req,
                                        _p(v), n_yes, v.size - n_yes, _p(yes), _p(no), _p(score), _p(logits),
                                        _p(cancel) if cancel is not None else None))
        return yes, no, score, logits

    def qmatmul(self, weight: str, x: np.ndarray, M: int, n_out: int, row_ids=None, device: int = 0):
        x = np.ascontiguousarray(x, np.float32)
        if row_ids is not None:
            ids = np.ascontiguousarray(row_ids, np.int32)
            y = np.zeros((M, ids.size), np.float32)
            _check(lib().shield_qmatmul(self._h, device, weight.encode(), _p(x), M, _p(y), _p(ids), ids.size))
        else:
            y = np.zeros((M, n_out), np.float32)
            _check(lib().shield_qmatmul(self._h, device, weight.encode(), _p(x), M, _p(y), None, 0))
        return y

    def qmatmul_device(self, weight: str, d_x: int, M: int, d_y: int, device: int = 0):
        _check(lib().shield_qmatmul_device(self._h, device, weight.encode(), C.c_void_p(d_x), M, C.c_void_p(d_y)))

    def qmatmul_noalloc(self, weight: str, d_x: int, M: int, d_y: int, device: int = 0):
        """shield_qmatmul_noalloc: the GEMM on device buffers, allocating nothing."""
        _check(lib().shield_qmatmul_noalloc(self._h, device, weight.encode(), C.c_void_p(d_x), M, C.c_void_p(d_y)))

    def block_dots(self, weight: str, x: np.ndarray, M: int, rows: int, cols: int, path: int = 0, device: int = 0):
        x = np.ascontiguousarray(x, np.float32)
        d = np.zeros((M, rows, cols // 32), np.int32)
        _check(lib().shield_debug_block_dots(self._h, device, weight.encode(), _p(x), M, _p(d), path))
        return d

    def set_gemm_path(self, path: int):
        _check(lib().shield_set_gemm_path(self._h, path))

    def set_gemm_tile_width(self, width: int):
        """0: automatic; 64 or 128: the tensor-core GEMM's tile width only."""
        _check(lib().shield_set_gemm_tile_width(self._h, width))

    def set_attention_rows(self, rows: int):
        """0: automatic; 64 or 128 query rows per attention CTA only."""
        _check(lib().shield_set_attention_rows(self._h, rows))

    def activation(self, ids, layer: int, what: int = ACT_OUTPUT, device: int = 0):
        """Tensor `what` (ACT_*) of layer `layer` for one request."""
        ids = np.ascontiguousarray(ids, np.int32)
        s = self.spec
        width = {ACT_Q_ROPE: s.qdim, ACT_ATTN_WEIGHTED: s.qdim, ACT_K_ROPE: s.kvdim, ACT_V: s.kvdim}.get(what, s.hidden)
        out = np.zeros((ids.size, width), np.float32)
        _check(lib().shield_debug_activation(self._h, device, _p(ids), ids.size, layer, what, _p(out)))
        return out

    def set_timing(self, level: int):
        _check(lib().shield_set_timing(self._h, level))

    def read_timing(self, device: int = 0, reset: bool = True) -> dict:
        t = ShieldTiming()
        _check(lib().shield_read_timing(self._h, device, C.byref(t), int(reset)))
        return {name: getattr(t, name) for name, _ in ShieldTiming._fields_}

    def stream(self, device: int = 0) -> int:
        s = C.c_void_p()
        _check(lib().shield_device_stream(self._h, device, C.byref(s)))
        return s.value or 0
