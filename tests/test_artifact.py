"""The artifact reader against the reference exporter's bytes (pinned by the
sha256 the golden generator recorded from tools/export_decoder.py)."""
import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN
from leaf_b200 import LeafError
from leaf_b200.artifact import Artifact

import decoder_fixture as fx  # tests/golden on sys.path (conftest)


@pytest.mark.parametrize("name", ["tiny_w8", "tiny_w4"])
def test_fixture_writer_matches_reference_exporter(tmp_path, name):
    meta = json.loads((GOLDEN / f"decoder_{name}.json").read_text())
    path = tmp_path / "model.leaf"
    fx.write_artifact(path, fx.TINY, fx.llama_tensors(fx.TINY, meta["weight_seed"], meta["norm_noise"]),
                      meta["bits"], meta["group"])
    assert hashlib.sha256(path.read_bytes()).hexdigest() == meta["artifact_sha256"]


def test_reader_parses_config_and_payloads(tmp_path):
    path = tmp_path / "model.leaf"
    tensors = dict(fx.llama_tensors(fx.TINY, 2024, 0.1))
    fx.write_artifact(path, fx.TINY, tensors.items(), 8, 64)
    art = Artifact(path)
    c = art.config
    assert (c.hidden, c.intermediate, c.heads, c.kv_heads, c.layers, c.vocab) == (128, 256, 4, 2, 2, 256)
    assert (c.head_dim, c.rotary_dim, c.gated, c.final_norm, c.eos_tokens) == (32, 32, 1, 1, [])
    assert np.float32(c.epsilon) == np.float32(1e-5)
    q = art.get("model.layers.1.self_attn.q_proj.weight")
    codes, scales = fx.quantize(tensors["model.layers.1.self_attn.q_proj.weight"], 8, 128)
    assert q.bits == 8 and q.group == 128
    assert np.array_equal(q.data, codes) and np.array_equal(q.scales, scales)
    norm = art.get("model.layers.0.input_layernorm.weight")
    assert norm.bits == 32 and np.array_equal(norm.data.reshape(-1), tensors["model.layers.0.input_layernorm.weight"])


def test_reader_rejects_bad_files(tmp_path):
    path = tmp_path / "model.leaf"
    fx.write_artifact(path, fx.TINY, fx.llama_tensors(fx.TINY, 1, 0.0), 8, 64)
    blob = bytearray(path.read_bytes())
    bad = tmp_path / "bad.leaf"
    bad.write_bytes(b"LEAFDC99" + bytes(blob[8:]))
    with pytest.raises(LeafError):
        Artifact(bad)
    truncated = tmp_path / "short.leaf"
    truncated.write_bytes(bytes(blob[:200]))
    with pytest.raises(LeafError):
        Artifact(truncated)
