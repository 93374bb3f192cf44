"""GGUF files for the synthetic checkpoints.

``write_model`` lays a model out as the reference's converter does
(tools/convert_shieldstral_to_gguf.py:277-353): architecture ``mistral3``,
the llama.cpp metadata keys that ``ModelConfig.FromGguf`` reads
(Model/ModelConfig.cs:62-112), a 131072-entry vocabulary whose ids 0..999
are control tokens (:147-168), quantized ``token_embd`` and layer matrices,
F32 norm vectors, no ``output.weight`` (tied head).  ``GgufFile`` maps a file
read-only and hands out each tensor's bytes in place, as
``GgufFile.GetTensorPointer`` does (Gguf/GgufFile.cs:195-199), so an upload
goes from the mapping straight into the library's pinned staging.

The container is GGUF version 3: magic, version, tensor and key counts, the
key/value pairs, the tensor infos (name, dims innermost first, type, offset),
then the tensor data, each tensor aligned to ``general.alignment`` (32).
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

from . import synth

MAGIC = b"GGUF"
VERSION = 3
ALIGN = 32
ARCH = "mistral3"

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
           U64: "<Q", I64: "<q", F64: "<d"}
# llama.cpp's general.file_type for the legacy 32-blocks
_FILE_TYPE = {synth.Q4_0: 2, synth.Q4_1: 3, synth.Q8_0: 7, synth.Q5_0: 8, synth.Q5_1: 9}
# surface forms placed at the verdict ids (7 "yes", 9 "no")
YES_FORMS = ["yes", "Yes", "YES", "Ġyes", "ĠYes", "ĠYES", "_yes"]
NO_FORMS = ["no", "No", "NO", "Ġno", "ĠNo", "ĠNO", "_no", "No.", "no."]


def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STR:
        return _str(v)
    if vtype == ARR:
        etype, items = v
        head = struct.pack("<IQ", etype, len(items))
        if etype == STR:
            return head + b"".join(_str(s) for s in items)
        return head + np.asarray(items, np.dtype(_SCALAR[etype])).tobytes()
    return struct.pack(_SCALAR[vtype], v)


def vocabulary(spec: synth.ModelSpec) -> tuple[list[str], list[int]]:
    """Token strings and llama.cpp token types: ids 0..999 control (3), the
    verdict ids given yes/no surface forms, the rest placeholders (1)."""
    tokens = [f"<SPECIAL_{i}>" if i < synth.FIRST_ORDINARY_ID else f"<tok_{i}>" for i in range(spec.vocab)]
    types = [3 if i < synth.FIRST_ORDINARY_ID else 1 for i in range(spec.vocab)]
    for ids, forms in ((spec.yes_ids, YES_FORMS), (spec.no_ids, NO_FORMS)):
        for k, i in enumerate(ids):
            tokens[i] = forms[k % len(forms)] + ("" if k < len(forms) else f"#{k}")
    return tokens, types


def model_metadata(spec: synth.ModelSpec) -> list[tuple[str, int, object]]:
    """(key, value type, value) in the converter's order."""
    a = ARCH
    yarn = spec.yarn_factor > 1.0 and spec.yarn_orig_ctx > 0
    tokens, types = vocabulary(spec)
    kv = [("general.architecture", STR, a), ("general.name", STR, "Shieldstral-shaped synthetic"),
          ("general.alignment", U32, ALIGN), ("general.file_type", U32, _FILE_TYPE.get(spec.qtype, 0)),
          (f"{a}.context_length", U32, int(max(spec.yarn_orig_ctx, 1) * max(spec.yarn_factor, 1.0))),
          (f"{a}.embedding_length", U32, spec.hidden), (f"{a}.block_count", U32, spec.n_layers),
          (f"{a}.feed_forward_length", U32, spec.ffn), (f"{a}.attention.head_count", U32, spec.n_heads),
          (f"{a}.attention.head_count_kv", U32, spec.n_kv_heads), (f"{a}.attention.key_length", U32, spec.head_dim),
          (f"{a}.attention.value_length", U32, spec.head_dim),
          (f"{a}.attention.layer_norm_rms_epsilon", F32, spec.rms_eps), (f"{a}.vocab_size", U32, spec.vocab),
          (f"{a}.rope.freq_base", F32, spec.rope_theta), (f"{a}.rope.dimension_count", U32, spec.head_dim)]
    if yarn:
        kv += [(f"{a}.rope.scaling.type", STR, "yarn"), (f"{a}.rope.scaling.factor", F32, spec.yarn_factor),
               (f"{a}.rope.scaling.original_context_length", U32, spec.yarn_orig_ctx),
               (f"{a}.rope.scaling.yarn_beta_fast", F32, spec.yarn_beta_fast),
               (f"{a}.rope.scaling.yarn_beta_slow", F32, spec.yarn_beta_slow),
               (f"{a}.rope.scaling.yarn_ext_factor", F32, 1.0), (f"{a}.rope.scaling.mscale", F32, 1.0),
               (f"{a}.rope.scaling.yarn_log_multiplier", F32, 1.0), (f"{a}.rope.scaling.attn_factor", F32, 1.0)]
    if spec.attn_temperature_beta:
        kv += [(f"{a}.attention.temperature_scale", F32, spec.attn_temperature_beta),
               (f"{a}.attention.temperature_length", U32, spec.yarn_orig_ctx)]
    kv += [("tokenizer.ggml.model", STR, "gpt2"), ("tokenizer.ggml.pre", STR, "tekken"),
           ("tokenizer.ggml.tokens", ARR, (STR, tokens)), ("tokenizer.ggml.token_type", ARR, (I32, types)),
           ("tokenizer.ggml.bos_token_id", U32, 1), ("tokenizer.ggml.eos_token_id", U32, 2),
           ("tokenizer.ggml.unknown_token_id", U32, 0), ("tokenizer.ggml.padding_token_id", U32, 11),
           ("tokenizer.ggml.add_bos_token", BOOL, True), ("tokenizer.ggml.add_eos_token", BOOL, False)]
    return kv


def _pad(n: int) -> int:
    return (ALIGN - n % ALIGN) % ALIGN


def write_model(path, spec: synth.ModelSpec, tensors: dict | None = None) -> Path:
    """Writes spec's model (synth.make_model(spec) unless tensors are given)
    to path as a GGUF file; returns the path."""
    path = Path(path)
    tensors = synth.make_model(spec) if tensors is None else tensors
    kv = model_metadata(spec)
    infos, offset = [], 0
    for name, t in tensors.items():
        ne = [t["cols"]] if t["rows"] == 1 and name.endswith("norm.weight") else [t["cols"], t["rows"]]
        infos.append((name, ne, t["type"], offset, t["data"]))
        offset += t["data"].nbytes
        offset += _pad(offset)
    with open(path, "wb") as f:
        head = MAGIC + struct.pack("<IQQ", VERSION, len(infos), len(kv))
        head += b"".join(_str(k) + struct.pack("<I", vt) + _value(vt, v) for k, vt, v in kv)
        for name, ne, qt, off, _ in infos:
            head += _str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
            head += struct.pack("<IQ", qt, off)
        head += b"\0" * _pad(len(head))
        f.write(head)
        pos = 0
        for _, _, _, off, data in infos:
            f.write(b"\0" * (off - pos))
            f.write(memoryview(np.ascontiguousarray(data, np.uint8)))
            pos = off + data.nbytes
    return path


class GgufFile:
    """A GGUF file mapped read-only: its key/value metadata, and every
    tensor's bytes as a view into the mapping (no copy)."""

    def __init__(self, path):
        self.path = Path(path)
        self.map = np.memmap(self.path, np.uint8, mode="r")
        buf = memoryview(self.map)
        if bytes(buf[:4]) != MAGIC:
            raise ValueError(f"{self.path} is not a GGUF file")
        version, n_tensors, n_kv = struct.unpack_from("<IQQ", buf, 4)
        if version not in (2, 3):
            raise ValueError(f"{self.path}: GGUF version {version} is not supported")
        pos = 24
        self.kv = {}
        for _ in range(n_kv):
            key, pos = self._read_str(buf, pos)
            (vt,), pos = struct.unpack_from("<I", buf, pos), pos + 4
            self.kv[key], pos = self._read_value(buf, pos, vt)
        self.infos = {}
        for _ in range(n_tensors):
            name, pos = self._read_str(buf, pos)
            (nd,), pos = struct.unpack_from("<I", buf, pos), pos + 4
            ne, pos = list(struct.unpack_from(f"<{nd}Q", buf, pos)), pos + 8 * nd
            qt, off = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            self.infos[name] = (qt, ne, off)
        align = int(self.kv.get("general.alignment", ALIGN))
        self.data_start = pos + (align - pos % align) % align

    @staticmethod
    def _read_str(buf, pos):
        (n,) = struct.unpack_from("<Q", buf, pos)
        return bytes(buf[pos + 8:pos + 8 + n]).decode("utf-8"), pos + 8 + n

    def _read_value(self, buf, pos, vt):
        if vt == STR:
            return self._read_str(buf, pos)
        if vt == ARR:
            et, n = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            if et == STR:
                out = []
                for _ in range(n):
                    s, pos = self._read_str(buf, pos)
                    out.append(s)
                return out, pos
            dt = np.dtype(_SCALAR[et])
            return np.frombuffer(buf, dt, n, pos).copy(), pos + n * dt.itemsize
        fmt = _SCALAR[vt]
        return struct.unpack_from(fmt, buf, pos)[0], pos + struct.calcsize(fmt)

    def tensor(self, name: str) -> dict:
        """{"type", "rows", "cols", "data"}: data is a uint8 view of the mapping."""
        qt, ne, off = self.infos[name]
        cols = int(ne[0])
        rows = int(np.prod(ne[1:])) if len(ne) > 1 else 1
        n = rows * synth.row_bytes(qt, cols)
        start = self.data_start + off
        return {"type": qt, "rows": rows, "cols": cols, "data": self.map[start:start + n]}

    def tensors(self) -> dict:
        return {name: self.tensor(name) for name in self.infos}

    def spec(self) -> synth.ModelSpec:
        """ModelConfig.FromGguf (ModelConfig.cs:62-112) for the fields the
        synthetic model has, as a ModelSpec; verdict ids are found by their
        surface forms."""
        a = self.kv.get("general.architecture")
        if a not in ("mistral3", "ministral3", "llama"):
            raise ValueError(f"{self.path} is architecture {a!r}, not the Ministral-3 backbone")
        g = self.kv.get
        heads = int(g(f"{a}.attention.head_count"))
        hidden = int(g(f"{a}.embedding_length"))
        tokens = g("tokenizer.ggml.tokens")
        yarn = g(f"{a}.rope.scaling.type", "") == "yarn"
        index = {s: i for i, s in enumerate(tokens or [])}
        yes = [index[s] for s in YES_FORMS if s in index]
        no = [index[s] for s in NO_FORMS if s in index]
        return synth.ModelSpec(
            n_layers=int(g(f"{a}.block_count")), hidden=hidden, n_heads=heads,
            n_kv_heads=int(g(f"{a}.attention.head_count_kv", heads)),
            head_dim=int(g(f"{a}.attention.key_length", hidden // max(1, heads))),
            ffn=int(g(f"{a}.feed_forward_length")),
            vocab=len(tokens) if tokens is not None else int(g(f"{a}.vocab_size")),
            rms_eps=float(g(f"{a}.attention.layer_norm_rms_epsilon", 1e-5)),
            rope_theta=float(g(f"{a}.rope.freq_base", 10000.0)),
            yarn_factor=float(g(f"{a}.rope.scaling.factor", 1.0)) if yarn else 1.0,
            yarn_orig_ctx=int(g(f"{a}.rope.scaling.original_context_length", 0)),
            yarn_beta_fast=float(g(f"{a}.rope.scaling.yarn_beta_fast", 32.0)),
            yarn_beta_slow=float(g(f"{a}.rope.scaling.yarn_beta_slow", 1.0)),
            attn_temperature_beta=float(g(f"{a}.attention.temperature_scale", 0.0)),
            qtype=self.infos["token_embd.weight"][0], yes_ids=yes, no_ids=no)

    def close(self):
        """Drops this object's mapping; tensor views handed out keep theirs
        alive until they are released."""
        self.map = None
