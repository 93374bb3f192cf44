"""The synthetic checkpoint as a GGUF file (llm_shield_b200/gguf_file.py):
written with the converter's keys and tensor names
(tools/convert_shieldstral_to_gguf.py:186-203,277-353), read back through a
read-only mapping with every tensor's bytes unchanged, and cross-checked with
gguf-py 0.19.0 (the converter's own GGUF library) reading the same file."""
from __future__ import annotations

import numpy as np
import pytest

from llm_shield_b200 import gguf_file, synth


@pytest.fixture(scope="module")
def written(tmp_path_factory):
    spec = synth.small_spec(qtype=synth.Q5_1, n_layers=2, seed=3)
    tensors = synth.make_model(spec)
    path = gguf_file.write_model(tmp_path_factory.mktemp("gguf") / "small.gguf", spec, tensors)
    return spec, tensors, path


def test_tensors_round_trip_through_the_mapping(written):
    spec, tensors, path = written
    g = gguf_file.GgufFile(path)
    assert set(g.infos) == set(tensors)
    assert "output.weight" not in g.infos  # tied head
    for name, t in tensors.items():
        got = g.tensor(name)
        assert (got["type"], got["rows"], got["cols"]) == (t["type"], t["rows"], t["cols"]), name
        assert isinstance(got["data"], np.memmap)  # a view of the file, not a copy
        np.testing.assert_array_equal(got["data"], t["data"], err_msg=name)
        assert (g.data_start + g.infos[name][2]) % gguf_file.ALIGN == 0


def test_metadata_gives_back_the_model_config(written):
    spec, _, path = written
    s = gguf_file.GgufFile(path).spec()
    for f in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "yarn_orig_ctx",
              "qtype", "yes_ids", "no_ids"):
        assert getattr(s, f) == getattr(spec, f), f
    for f in ("rms_eps", "rope_theta", "yarn_factor", "yarn_beta_fast", "yarn_beta_slow", "attn_temperature_beta"):
        assert np.float32(getattr(s, f)) == np.float32(getattr(spec, f)), f


def test_gguf_py_reads_the_same_file(written):
    gguf = pytest.importorskip("gguf")
    spec, tensors, path = written
    r = gguf.GGUFReader(str(path))
    assert r.fields["general.architecture"].contents() == "mistral3"
    assert r.fields["mistral3.block_count"].contents() == spec.n_layers
    assert r.fields["mistral3.attention.head_count_kv"].contents() == spec.n_kv_heads
    toks = r.fields["tokenizer.ggml.tokens"].contents()
    types = r.fields["tokenizer.ggml.token_type"].contents()
    assert len(toks) == spec.vocab and types[:1000] == [3] * 1000 and types[1000] == 1
    assert toks[spec.yes_ids[0]] == "yes" and toks[spec.no_ids[0]] == "no"
    assert {t.name for t in r.tensors} == set(tensors)
    for t in r.tensors:
        ref = tensors[t.name]
        assert int(t.tensor_type) == ref["type"]
        assert list(t.shape) == ([ref["cols"]] if t.name.endswith("norm.weight") else [ref["cols"], ref["rows"]])
        np.testing.assert_array_equal(np.asarray(t.data).reshape(-1).view(np.uint8), ref["data"])
