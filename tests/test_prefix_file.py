"""CPU tests of the system-prompt snapshot file (SystemPromptCache.Save /
TryLoad / LoadOrCaptureAsync, SystemPromptCache.cs:110-185): byte layout,
fingerprint, the misses TryLoad reports, and the load-or-capture decision
driven against a host-side stand-in for the GPU context."""
from __future__ import annotations

import hashlib
import os
import struct

import numpy as np
import pytest

from llm_shield_b200 import prefix_file as pf


@pytest.fixture
def model(tmp_path):
    path = tmp_path / "shieldstral.gguf"
    path.write_bytes(b"12345")
    os.utime(path, ns=(1_700_000_000_123_456_789, 1_700_000_000_123_456_789))
    return pf.ModelIdentity(str(path), "mistral3", 26, 8, 128)


def _snapshot(model, n=3, seed=0):
    rng = np.random.default_rng(seed)
    toks = rng.integers(1, 131072, size=n, dtype=np.int32)
    state = rng.standard_normal(2 * 2 * 8 * n * 4).astype(np.float32)
    return pf.PrefixSnapshot(toks, state, pf.fingerprint(model, toks))


def test_fingerprint_known_answer(model):
    # .NET ticks: 100 ns since 0001-01-01 UTC; the Unix epoch is 621355968000000000
    text = "shieldstral.gguf|5|638355968001234567|mistral3|26x8x128|2:1,2,"
    assert pf.fingerprint(model, [1, 2]) == hashlib.sha256(text.encode()).hexdigest()
    missing = pf.ModelIdentity(model.model_path + ".gone", "mistral3", 26, 8, 128)
    text = "shieldstral.gguf.gone|-1|-1|mistral3|26x8x128|0:"
    assert pf.fingerprint(missing, []) == hashlib.sha256(text.encode()).hexdigest()


def test_byte_layout(model):
    snap = _snapshot(model, n=2)
    b = pf.encode(snap)
    assert b[:4] == b"VKHS"  # 0x53484B56 little-endian
    assert struct.unpack_from("<i", b, 4)[0] == 1
    assert b[8] == 64 and b[9:73].decode() == snap.fingerprint  # one-byte 7-bit length
    assert struct.unpack_from("<i", b, 73)[0] == 2
    assert list(struct.unpack_from("<2i", b, 77)) == list(snap.tokens)
    assert struct.unpack_from("<q", b, 85)[0] == snap.state.size
    np.testing.assert_array_equal(np.frombuffer(b, "<f4", offset=93), snap.state)
    assert len(b) == 93 + 4 * snap.state.size


def test_long_strings_use_multibyte_lengths():
    out = bytearray()
    s = "x" * 300
    pf._write_string(out, s)
    assert out[:2] == bytes([0xAC, 0x02])
    assert pf._read_string(bytes(out), 0) == (s, len(out))
    with pytest.raises(ValueError):
        pf._read_string(bytes([0x80] * 5 + [0]), 0)


def test_round_trip_and_misses(model, tmp_path):
    snap = _snapshot(model)
    path = tmp_path / "prefix.shkv"
    pf.save(path, snap)
    back = pf.try_load(path, model)
    assert back is not None and back.fingerprint == snap.fingerprint
    np.testing.assert_array_equal(back.tokens, snap.tokens)
    np.testing.assert_array_equal(back.state, snap.state)
    assert back.is_prefix_of(np.concatenate([snap.tokens, [7, 8]]))
    assert not back.is_prefix_of(snap.tokens[:-1])

    assert pf.try_load(tmp_path / "absent.shkv", model) is None
    good = path.read_bytes()
    for cut in (0, 3, 8, 40, 75, 80, 90, len(good) - 1):  # every field cut short
        assert pf.decode(good[:cut], model) is None, cut
    bad = bytearray(good)
    bad[0] ^= 1
    assert pf.decode(bytes(bad), model) is None
    bad = bytearray(good)
    bad[4] = 2  # version
    assert pf.decode(bytes(bad), model) is None
    # a stale snapshot: other geometry, architecture, or a rewritten model file
    for other in (pf.ModelIdentity(model.model_path, "mistral3", 26, 8, 64),
                  pf.ModelIdentity(model.model_path, "llama", 26, 8, 128)):
        assert pf.try_load(path, other) is None
    os.utime(model.model_path, ns=(1_800_000_000_000_000_000,) * 2)
    assert pf.try_load(path, model) is None


class FakeContext:
    """Stands in for ShieldContext's prefix calls (the GPU side is tested in
    the gpu-marked tests)."""

    def __init__(self):
        self.calls = []
        self.state = None

    def set_prefix(self, ids):
        self.calls.append(("prefill", list(ids)))
        self.state = np.arange(2 * len(ids), dtype=np.float32)

    def get_prefix_state(self):
        return self.state.copy()

    def set_prefix_state(self, ids, state):
        self.calls.append(("restore", list(ids)))
        self.state = np.asarray(state).copy()


def test_load_or_capture(model, tmp_path):
    path = tmp_path / "prefix.shkv"
    ctx = FakeContext()
    toks = [5, 6, 7]
    first = pf.load_or_capture(ctx, model, toks, path)
    assert ctx.calls == [("prefill", toks)] and path.exists()
    second = pf.load_or_capture(ctx, model, toks, path)
    assert ctx.calls[-1] == ("restore", toks)
    np.testing.assert_array_equal(second.state, first.state)
    # other tokens: the file is stale for them, so prefill and overwrite
    pf.load_or_capture(ctx, model, [5, 6], path)
    assert ctx.calls[-1] == ("prefill", [5, 6])
    np.testing.assert_array_equal(pf.try_load(path, model).tokens, [5, 6])
    # an unwritable destination costs the prefill, not a failure
    pf.load_or_capture(ctx, model, toks, tmp_path / "no-such-dir" / "p.shkv")
    assert ctx.calls[-1] == ("prefill", toks)
