"""The CPU decoder restatement (oracle/decoder.py) against the reference
decoder's own outputs: bit-identical logits for every prefill row and every
decode step of the tiny fixture models."""
import json

import numpy as np
import pytest

from conftest import GOLDEN
import decoder_fixture as fx  # tests/golden
from leaf_b200.artifact import Artifact
from oracle.decoder import OracleDecoder


@pytest.mark.parametrize("name", ["tiny_w8", "tiny_w4"])
def test_oracle_decoder_bit_exact(tmp_path, name):
    meta = json.loads((GOLDEN / f"decoder_{name}.json").read_text())
    with np.load(GOLDEN / f"decoder_{name}.npz") as data:
        golden = {k: data[k] for k in data.files}
    path = tmp_path / "m.leaf"
    fx.write_artifact(path, fx.TINY, fx.llama_tensors(fx.TINY, meta["weight_seed"], meta["norm_noise"]),
                      meta["bits"], meta["group"])
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
