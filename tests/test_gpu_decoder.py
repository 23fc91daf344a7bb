"""The GPU decoder against the reference decoder (oracle/_ref/leaf_decoder
outputs recorded by tests/golden/make_decoder_golden.py): identical greedy
tokens and bit-identical logits (prefill and every decode step), for per-row
INT8, INT4, and an artifact with SmoothQuant input scales on every
projection and q / k / v biases.
"""
import hashlib
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
import decoder_fixture as fx  # tests/golden

pytestmark = pytest.mark.gpu

def _artifact(tmp_path, name, shape):
    meta = json.loads((GOLDEN / f"decoder_{name}.json").read_text())
    path = tmp_path / f"{name}.leaf"
    tensors = fx.llama_tensors(shape, meta["weight_seed"], meta["norm_noise"])
    extras = ()
    if name == "tiny_smooth":  # SmoothQuant input scales + q / k / v biases
        tensors, extras = fx.smooth_variant(shape, tensors, meta["weight_seed"] + 1)
    fx.write_artifact(path, shape, tensors, meta["bits"], meta["group"], extras=extras)
    h = hashlib.sha256()
    with path.open("rb") as f:
        for block in iter(lambda: f.read(1 << 24), b""):
            h.update(block)
    assert h.hexdigest() == meta["artifact_sha256"], "fixture artifact differs from the reference export"
    with np.load(GOLDEN / f"decoder_{name}.npz") as data:
        golden = {k: data[k] for k in data.files}
    return path, golden


def _close(got, ref):
    got = np.ascontiguousarray(got, dtype=np.float32)
    ref = np.ascontiguousarray(ref, dtype=np.float32)
    return np.array_equal(got.view(np.uint32), ref.view(np.uint32)), float(np.max(np.abs(got - ref)))


@pytest.mark.parametrize("name", ["tiny_w8", "tiny_w4", "tiny_smooth"])
def test_tiny_decoder_matches_reference(cuda_device, tmp_path, name):
    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, name, fx.TINY)
    dec = Decoder(path)
    prompt, generated = golden["prompt"].tolist(), golden["generated"].tolist()
    assert dec.generate(prompt, len(generated)) == generated
    # Prefill logits of the prompt's last position (reference verify mode).
    dec.reset()
    ok, err = _close(dec.forward(prompt).cpu().numpy()[0], golden["prefill_logits"][-1])
    assert ok, f"prefill logits differ by {err}"
    # Token-by-token decode logits over prompt + generated (chunked mode).
    dec.reset()
    sequence = prompt + generated[:-1]
    for i, tok in enumerate(sequence):
        ok, err = _close(dec.forward([tok]).cpu().numpy()[0], golden["decode_logits"][i])
        assert ok, f"decode logits at step {i} differ by {err}"
    assert dec.device_status() == 0


def test_tiny_fused_decode_step(cuda_device, tmp_path):
    """The one-launch decode step: same tokens and bit-identical logits at
    every step (W8A8 fixture)."""
    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, "tiny_w8", fx.TINY)
    dec = Decoder(path)
    prompt, generated = golden["prompt"].tolist(), golden["generated"].tolist()
    assert dec.generate_fused(prompt, len(generated)) == generated
    dec.reset()
    n = len(prompt)
    dec.forward(prompt)
    for j, tok in enumerate(generated[:-1]):
        dec.token.fill_(tok)
        dec.step_fused()
        ok, err = _close(dec.step_logits.cpu().numpy(), golden["decode_logits"][n + j])
        assert ok, f"fused step {j} logits differ by {err}"
        assert int(dec.token.item()) == generated[j + 1]
    assert dec.device_status() == 0
    dec.close()


def test_tiny_stream_step_graph(cuda_device, tmp_path):
    """The streaming-step graph (token in from pinned host memory, the fused
    step, token out to pinned host memory) gives the reference's tokens."""
    import torch

    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, "tiny_w8", fx.TINY)
    dec = Decoder(path)
    prompt, generated = golden["prompt"].tolist(), golden["generated"].tolist()
    logits = dec.forward(prompt)
    first = int(np.argmax(logits.cpu().numpy().reshape(-1, dec.cfg.vocab)[-1]))
    assert first == generated[0]
    tok_in = torch.empty(1, dtype=torch.int32).pin_memory()
    tok_out = torch.empty(1, dtype=torch.int32).pin_memory()
    graph = dec.capture_stream_step(tok_in, tok_out)
    tok_in[0] = first
    got = [first]
    stream = torch.cuda.current_stream()
    for _ in generated[1:]:
        graph.replay()
        stream.synchronize()
        got.append(int(tok_out[0]))
        tok_in.copy_(tok_out)
    assert got == generated
    assert dec.device_status() == 0
    del graph
    dec.close()


def test_tinyllama_greedy_tokens(cuda_device, tmp_path):
    """Config 3: TinyLlama-1.1B-shape W8A8 decoder, 128-token random prompt,
    128 greedy tokens, identical to the reference's."""
    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, "tinyllama_w8", fx.TINYLLAMA)
    dec = Decoder(path)
    path.unlink()
    prompt, generated = golden["prompt"].tolist(), golden["generated"].tolist()
    logits = dec.forward(prompt).cpu().numpy()[0]
    ok, err = _close(logits, golden["prefill_last_logits"])
    assert ok, f"prefill logits differ by {err}"
    dec.reset()
    got = dec.generate(prompt, len(generated))
    assert got == generated, next(i for i, (a, b) in enumerate(zip(got, generated)) if a != b)
    dec.reset()
    got = dec.generate_fused(prompt, len(generated))
    assert got == generated, next(i for i, (a, b) in enumerate(zip(got, generated)) if a != b)
    assert dec.device_status() == 0
    dec.close()


def test_expf_matches_libm(cuda_device):
    """leafq_expf against the host libm expf: 32M random bit patterns plus
    every float of [-2, -1) and [1, 2) and the whole softmax range near 0."""
    import leaf_b200 as lq
    import oracle

    rng = np.random.default_rng(4)
    parts = [rng.integers(0, 2**32, size=1 << 25, dtype=np.uint64).astype(np.uint32),
             np.arange(0x3F800000, 0x40000000, dtype=np.uint32),
             np.arange(0xBF800000, 0xC0000000, dtype=np.uint32),
             np.arange(0xB8000000, 0xB8800000, dtype=np.uint32)]
    bits = np.concatenate(parts)
    x = bits.view(np.float32)
    x = x[~np.isnan(x)]
    expect = oracle.expf(x)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty_like(xd)
    lq._lib.check(lq.load().leafq_expf(torch.cuda.current_stream().cuda_stream, xd.data_ptr(), x.size,
                                       y.data_ptr()))
    got = y.cpu().numpy()
    bad = np.flatnonzero(got.view(np.uint32) != expect.view(np.uint32))
    assert bad.size == 0, (x[bad[:5]], got[bad[:5]], expect[bad[:5]])


def test_smooth_decoder_batched_prefill_matches_reference(cuda_device, tmp_path):
    """The SmoothQuant + bias model with several sequences (every linear over
    all rows, the tcgen05 GEMM for more than 8 rows): each sequence's last
    prefill logits equal the reference's for its prompt."""
    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, "tiny_smooth", fx.TINY)
    prompt = golden["prompt"].tolist()
    dec = Decoder(path, sequences=3)
    logits = dec.forward_batch([prompt, prompt, prompt]).cpu().numpy()
    for s in range(3):
        ok, err = _close(logits[s], golden["prefill_logits"][-1])
        assert ok, f"sequence {s}: prefill logits differ by {err}"
    assert dec.device_status() == 0
