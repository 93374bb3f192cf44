#!/usr/bin/env python3
"""Generates the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the reference project is mounted (its path is the
first argument; it is read, never modified).  The GPU tests never run this
script: they only read the JSON it writes.

1. quantization_cases.json — the legacy-block cases (F32, F16, Q4_0, Q4_1,
   Q5_0, Q5_1, Q8_0) of the reference's own dequantizer oracle,
   tests/fixtures/quantization.json (made by its tools/gen_quant_fixtures.py
   with gguf-py), re-keyed unchanged.

2. float_model.json — outputs of the reference's NumPy model
   (tools/reference_shieldstral.py, ReferenceModel.forward) on small synthetic
   checkpoints.  The checkpoint is this package's seeded synthetic model,
   written in Mistral format (consolidated.safetensors + params.json) with the
   *dequantized* weights, so the reference float model and the integer path
   see the same weights and differ only by activation quantization.

Usage:  python tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import base64
import json
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402
from llm_shield_b200 import synth  # noqa: E402

LEGACY = {0, 1, 2, 3, 6, 7, 8}

# Mistral-format names (tools/convert_shieldstral_to_gguf.py:186-203).
LAYER_NAMES = {
    "attn_norm.weight": "attention_norm.weight",
    "attn_q.weight": "attention.wq.weight",
    "attn_k.weight": "attention.wk.weight",
    "attn_v.weight": "attention.wv.weight",
    "attn_output.weight": "attention.wo.weight",
    "ffn_norm.weight": "ffn_norm.weight",
    "ffn_gate.weight": "feed_forward.w1.weight",
    "ffn_down.weight": "feed_forward.w2.weight",
    "ffn_up.weight": "feed_forward.w3.weight",
}


def gguf_to_mistral(name: str) -> str:
    if name == "token_embd.weight":
        return "tok_embeddings.weight"
    if name == "output_norm.weight":
        return "norm.weight"
    _, idx, rest = name.split(".", 2)
    return f"layers.{idx}.{LAYER_NAMES[rest]}"


def write_safetensors(path: Path, tensors: dict[str, np.ndarray]) -> None:
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr, np.float32)
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [off, off + arr.nbytes]}
        blobs.append(arr.tobytes())
        off += arr.nbytes
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def dequantized(t: dict) -> np.ndarray:
    return oracle.dequantize(t["type"], t["data"], t["rows"] * t["cols"]).reshape(t["rows"], t["cols"])


def make_quantization_cases(ref: Path) -> dict:
    src = json.loads((ref / "tests/fixtures/quantization.json").read_text())
    cases = [c for c in src["cases"] if c["ggml_type"] in LEGACY]
    return {"source": "reference tests/fixtures/quantization.json (gguf-py decoded), legacy types only",
            "cases": cases}


def make_float_model(ref: Path) -> dict:
    sys.path.insert(0, str(ref / "tools"))
    import reference_shieldstral as R  # the reference's NumPy model

    out = {"source": "reference tools/reference_shieldstral.py ReferenceModel.forward", "models": []}
    for qtype in (synth.Q8_0, synth.Q4_0, synth.Q5_1):
        spec = synth.small_spec(qtype=qtype, n_layers=2, seed=11 + qtype)
        tensors = synth.make_model(spec)
        with tempfile.TemporaryDirectory() as td:
            d = Path(td)
            write_safetensors(d / "consolidated.safetensors",
                              {gguf_to_mistral(n): (dequantized(t) if t["type"] != synth.F32
                                                    else t["data"].view(np.float32).reshape(-1))
                               for n, t in tensors.items()})
            params = {
                "dim": spec.hidden, "n_layers": spec.n_layers, "n_heads": spec.n_heads,
                "n_kv_heads": spec.n_kv_heads, "head_dim": spec.head_dim, "hidden_dim": spec.ffn,
                "norm_eps": spec.rms_eps, "vocab_size": spec.vocab, "rope_theta": spec.rope_theta,
                "yarn": {"factor": spec.yarn_factor,
                         "original_max_position_embeddings": spec.yarn_orig_ctx,
                         "beta": spec.yarn_beta_fast, "alpha": spec.yarn_beta_slow, "apply_scale": False},
                "llama_4_scaling": {"beta": spec.attn_temperature_beta,
                                    "original_max_position_embeddings": spec.yarn_orig_ctx},
            }
            (d / "params.json").write_text(json.dumps(params))
            model = R.ReferenceModel(d)
            rng = np.random.default_rng(100 + qtype)
            cases = []
            for n in (1, 7, 33):
                ids = rng.integers(synth.FIRST_ORDINARY_ID, spec.vocab, size=n).tolist()
                cap = {}
                logits = model.forward(ids, capture=cap)
                score, zy, zn = R.safety_score(logits, spec.yes_ids, spec.no_ids)
                cases.append({
                    "ids": ids,
                    "verdict_logits": [float(logits[i]) for i in spec.verdict_ids],
                    "score": score, "yes": zy, "no": zn,
                    "final_norm": [float(v) for v in cap["final_norm"].reshape(-1)],
                    "layer0_output_last": [float(v) for v in cap["blk.0.output"][-1]],
                })
            out["models"].append({"qtype": qtype, "seed": spec.seed, "n_layers": spec.n_layers, "cases": cases})
            print(f"  {synth.TYPE_NAMES[qtype]}: {len(cases)} cases")
    return out


def main() -> int:
    if len(sys.argv) < 2:
        print(__doc__)
        return 2
    ref = Path(sys.argv[1])
    (HERE / "quantization_cases.json").write_text(json.dumps(make_quantization_cases(ref), indent=1))
    print("wrote quantization_cases.json")
    (HERE / "float_model.json").write_text(json.dumps(make_float_model(ref)))
    print("wrote float_model.json")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
