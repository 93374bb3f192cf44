"""The system-prompt snapshot file ("SHKV") of SystemPromptCache
(src/LlmShield.Shieldstral/SystemPromptCache.cs:23-186), read and written on
the host so that a snapshot goes straight to the GPUs
(ShieldContext.set_prefix_state) instead of being prefilled again.

Format (SystemPromptCache.Save, :110-127; .NET BinaryWriter, little-endian):
    uint32 magic 0x53484B56, int32 version 1,
    string fingerprint (7-bit encoded UTF-8 byte count, then the bytes),
    int32 token count, int32 tokens[count],
    int64 float count, float32 state[count]   (KvCache.Snapshot's layout)

The fingerprint (:88-104) is the lowercase hex SHA-256 of
    "<file name>|<file length>|<last write, .NET ticks UTC>|<architecture>|
     <layers>x<kv heads>x<head dim>|<token count>:<t0>,<t1>,...,"
(one line, no spaces), with -1 for the length and ticks of a missing file.
"""
from __future__ import annotations

import hashlib
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = 0x53484B56  # "SHKV"
VERSION = 1
_UNIX_EPOCH_TICKS = 621355968000000000  # DateTime(1970, 1, 1).Ticks


@dataclass(frozen=True)
class ModelIdentity:
    """What a snapshot is tied to: the model file and the cache geometry
    (MinistralModel.ModelPath and ModelConfig, SystemPromptCache.cs:95-101)."""
    model_path: str
    architecture: str
    n_layers: int
    n_kv_heads: int
    head_dim: int


@dataclass
class PrefixSnapshot:
    """SystemPromptCache: the prefix's token ids, its flat KV state and the
    fingerprint it was captured under."""
    tokens: np.ndarray
    state: np.ndarray
    fingerprint: str

    @property
    def token_count(self) -> int:
        return int(self.tokens.size)

    def is_prefix_of(self, ids) -> bool:
        """SystemPromptCache.IsPrefixOf (:81-82)."""
        ids = np.asarray(ids)
        n = self.tokens.size
        return ids.size >= n and bool(np.array_equal(ids[:n], self.tokens))


def fingerprint(model: ModelIdentity, tokens) -> str:
    """SystemPromptCache.ComputeFingerprint (:88-104)."""
    p = Path(model.model_path)
    try:
        st = p.stat()
        length, ticks = st.st_size, _UNIX_EPOCH_TICKS + st.st_mtime_ns // 100
    except OSError:
        length, ticks = -1, -1
    toks = np.asarray(tokens, np.int64).reshape(-1)
    text = (f"{p.name}|{length}|{ticks}|{model.architecture}|"
            f"{model.n_layers}x{model.n_kv_heads}x{model.head_dim}|{toks.size}:"
            + "".join(f"{int(t)}," for t in toks))
    return hashlib.sha256(text.encode("utf-8")).hexdigest()


def _write_string(out: bytearray, s: str) -> None:
    data = s.encode("utf-8")
    n = len(data)
    while n >= 0x80:  # BinaryWriter.Write7BitEncodedInt
        out.append((n & 0x7F) | 0x80)
        n >>= 7
    out.append(n)
    out += data


def _read_string(buf: bytes, at: int) -> tuple[str, int]:
    n = shift = 0
    for i in range(5):
        if at >= len(buf):
            raise EOFError
        b = buf[at]
        at += 1
        n |= (b & 0x7F) << shift
        shift += 7
        if not b & 0x80:
            break
    else:  # BinaryReader throws FormatException, which TryLoad does not catch
        raise ValueError("bad 7-bit encoded string length")
    if at + n > len(buf):
        raise EOFError
    return buf[at:at + n].decode("utf-8", errors="replace"), at + n


def encode(snap: PrefixSnapshot) -> bytes:
    """The bytes SystemPromptCache.Save writes (:110-127)."""
    out = bytearray(struct.pack("<Ii", MAGIC, VERSION))
    _write_string(out, snap.fingerprint)
    toks = np.ascontiguousarray(snap.tokens, "<i4")
    out += struct.pack("<i", toks.size) + toks.tobytes()
    state = np.ascontiguousarray(snap.state, "<f4").reshape(-1)
    out += struct.pack("<q", state.size) + state.tobytes()
    return bytes(out)


def save(path, snap: PrefixSnapshot) -> None:
    with open(path, "wb") as f:
        f.write(encode(snap))


def decode(buf: bytes, model: ModelIdentity) -> PrefixSnapshot | None:
    """SystemPromptCache.TryLoad (:133-162) on a file's bytes: None for a wrong
    magic or version, implausible counts, a short file, or a fingerprint that
    does not match `model` and the file's own tokens."""
    try:
        if len(buf) < 8:
            raise EOFError
        magic, version = struct.unpack_from("<Ii", buf, 0)
        if magic != MAGIC or version != VERSION:
            return None
        fp, at = _read_string(buf, 8)
        if at + 4 > len(buf):
            raise EOFError
        (count,) = struct.unpack_from("<i", buf, at)
        at += 4
        if count < 0 or count > 1_000_000:
            return None
        if at + 4 * count + 8 > len(buf):
            raise EOFError
        tokens = np.frombuffer(buf, "<i4", count, at).astype(np.int32)
        at += 4 * count
        (n_state,) = struct.unpack_from("<q", buf, at)
        at += 8
        if n_state < 0 or n_state > 2**31 - 1:
            return None
        if at + 4 * n_state > len(buf):
            raise EOFError
        state = np.frombuffer(buf, "<f4", n_state, at).astype(np.float32)
    except EOFError:
        return None
    if fingerprint(model, tokens) != fp:
        return None
    return PrefixSnapshot(tokens, state, fp)


def try_load(path, model: ModelIdentity) -> PrefixSnapshot | None:
    """SystemPromptCache.TryLoad (:133-162): a missing or unreadable file is a
    miss (None), as is a stale one."""
    try:
        with open(path, "rb") as f:
            buf = f.read()
    except OSError:
        return None
    return decode(buf, model)


def load_or_capture(ctx, model: ModelIdentity, tokens, path) -> PrefixSnapshot:
    """SystemPromptCache.LoadOrCaptureAsync (:168-185) on a ShieldContext: a
    valid file for exactly these tokens is copied to the GPUs without a
    prefill; otherwise the prefix is forwarded on the GPUs, its snapshot read
    back and written to `path` (a read-only or full directory costs the
    prefill, not a failure). Either way the context caches the prefix."""
    toks = np.ascontiguousarray(tokens, np.int32)
    cached = try_load(path, model)
    if cached is not None and np.array_equal(cached.tokens, toks):
        ctx.set_prefix_state(cached.tokens, cached.state)
        return cached
    ctx.set_prefix(toks)
    fresh = PrefixSnapshot(toks.copy(), ctx.get_prefix_state(), fingerprint(model, toks))
    try:
        save(path, fresh)
    except OSError:
        pass
    return fresh
