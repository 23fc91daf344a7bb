"""The CPU decoder restatement (oracle/decoder.py) against the reference
decoder's own outputs: bit-identical logits for every prefill row and every
decode step of the tiny fixture models, including one with SmoothQuant input
scales on every projection and q / k / v biases (decoder.cpp:1003-1019,
:1229)."""
import json

import numpy as np
import pytest

from conftest import GOLDEN
import decoder_fixture as fx  # tests/golden
from leaf_b200.artifact import Artifact
from oracle.decoder import OracleDecoder


def write_fixture(path, name, meta):
    """The fixture model `name` as the artifact the golden data came from."""
    tensors = fx.llama_tensors(fx.TINY, meta["weight_seed"], meta["norm_noise"])
    extras = ()
    if name == "tiny_smooth":
        tensors, extras = fx.smooth_variant(fx.TINY, tensors, meta["weight_seed"] + 1)
    fx.write_artifact(path, fx.TINY, tensors, meta["bits"], meta["group"], extras=extras)


@pytest.mark.parametrize("name", ["tiny_w8", "tiny_w4", "tiny_smooth"])
def test_oracle_decoder_bit_exact(tmp_path, name):
    meta = json.loads((GOLDEN / f"decoder_{name}.json").read_text())
    with np.load(GOLDEN / f"decoder_{name}.npz") as data:
        golden = {k: data[k] for k in data.files}
    path = tmp_path / "m.leaf"
    write_fixture(path, name, meta)
    dec = OracleDecoder(Artifact(path))
    pre = dec.forward(golden["prompt"].tolist(), all_logits=True)
    assert np.array_equal(pre.view(np.uint32), golden["prefill_logits"].view(np.uint32))
    dec.reset()
    sequence = golden["prompt"].tolist() + golden["generated"][:-1].tolist()
    for i, tok in enumerate(sequence):
        logits = dec.forward([tok])[0]
        assert np.array_equal(logits.view(np.uint32), golden["decode_logits"][i].view(np.uint32)), i
    # Greedy tokens follow from the decode logits.
    assert [int(np.argmax(golden["decode_logits"][len(golden["prompt"]) - 1 + j]))
            for j in range(len(golden["generated"]))] == golden["generated"].tolist()
