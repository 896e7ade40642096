"""Safetensors reader (no torch): header parsing, dtypes, sharded
checkpoints, validation; and a model built from a checkpoint (GPU)."""

from __future__ import annotations

import json
import os
import struct

import numpy as np
import pytest

from triton_llm import safetensors as st


def test_round_trip_f32_bf16_int(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    b = rng.standard_normal((7,)).astype(np.float32)
    ids = np.arange(6, dtype=np.int64).reshape(2, 3)
    p32 = tmp_path / "f32.safetensors"
    st.save_file({"a": a, "ids": ids}, str(p32), metadata={"format": "np"})
    sd = st.load_state_dict(str(p32))
    assert set(sd) == {"a", "ids"} and len(sd) == 2
    np.testing.assert_array_equal(sd["a"], a)
    np.testing.assert_array_equal(sd["ids"], ids)
    assert sd.files[0].metadata == {"format": "np"}
    p16 = tmp_path / "bf16.safetensors"
    st.save_file({"b": b}, str(p16), bf16=True)
    dt, raw = st.load_state_dict(str(p16)).raw("b")
    assert dt == "BF16" and raw.dtype == np.uint16
    got = st.load_state_dict(str(p16))["b"]
    # bf16 keeps 8 mantissa bits (round to nearest even)
    np.testing.assert_allclose(got, b, rtol=2 ** -8)
    u = b.view(np.uint32)
    want = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    np.testing.assert_array_equal(raw, want)


def test_known_bytes(tmp_path):
    """A file assembled by hand from the published layout."""
    header = {"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
              "y": {"dtype": "BF16", "shape": [1], "data_offsets": [8, 10]}}
    h = json.dumps(header).encode()
    data = struct.pack("<2f", 1.5, -2.0) + struct.pack("<H", 0x3FC0)   # bf16 1.5
    p = tmp_path / "hand.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + data)
    sd = st.load_state_dict(str(p))
    np.testing.assert_array_equal(sd["x"], [1.5, -2.0])
    np.testing.assert_array_equal(sd["y"], [1.5])


def test_sharded_directory(tmp_path):
    rng = np.random.default_rng(1)
    t = {f"w{i}": rng.standard_normal((4, 4)).astype(np.float32) for i in range(4)}
    st.save_file({"w0": t["w0"], "w1": t["w1"]}, str(tmp_path / "model-00001-of-00002.safetensors"))
    st.save_file({"w2": t["w2"], "w3": t["w3"]}, str(tmp_path / "model-00002-of-00002.safetensors"))
    wm = {k: f"model-0000{1 + int(k[1]) // 2}-of-00002.safetensors" for k in t}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    sd = st.load_state_dict(str(tmp_path))
    assert sorted(sd) == sorted(t)
    for k, v in t.items():
        np.testing.assert_array_equal(sd[k], v)


def test_rejects_malformed(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        st.load_state_dict(str(p))
    h = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 8]}}).encode()
    p.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(ValueError):          # 4 floats need 16 bytes
        st.load_state_dict(str(p))
    empty = tmp_path / "nothing"
    empty.mkdir()
    with pytest.raises(FileNotFoundError):   # a directory without checkpoints
        st.load_state_dict(str(empty))


@pytest.mark.gpu
def test_smollm2_from_safetensors_matches_dict(tmp_path):
    """The tiny SmolLM2 built from a bf16 checkpoint directory generates the
    same tokens and logits as the same weights passed as a dict."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import inputs
    from smollm2_triton import SmolLM2Config, SmolLM2ForCausalLM
    w = inputs.round_linear_weights_bf16(inputs.llama_weights(inputs.SMOL_TINY, 0))
    st.save_file(w, str(tmp_path / "model.safetensors"), bf16=True)
    cfg = SmolLM2Config(**inputs.SMOL_TINY.config_kwargs())
    (tmp_path / "config.json").write_text(json.dumps(inputs.SMOL_TINY.config_kwargs()))
    m1 = SmolLM2ForCausalLM.from_safetensors(str(tmp_path), dtype="bfloat16")
    w_bf16 = {k: st.load_state_dict(str(tmp_path))[k] for k in w}
    m2 = SmolLM2ForCausalLM(cfg, w_bf16, dtype="bfloat16")
    prompt = np.array([[5, 12, 7]], np.int32)
    a = m1.generate_gpu(prompt, 8, temperature=0.0)
    b = m2.generate_gpu(prompt, 8, temperature=0.0)
    np.testing.assert_array_equal(a, b)
