"""Golden decoder outputs from the reference itself (run where the reference
tree is available: LEAF_REFERENCE, or a ``reference`` directory beside this
repository; needs the oracle/_ref build).

For each fixture model of decoder_fixture.py:
  1. write the seeded weights as a Hugging Face snapshot and export it with the
     reference's own exporter (tools/export_decoder.py, run unmodified);
  2. check that decoder_fixture.write_artifact produces the identical bytes
     (so tests on machines without the reference rebuild the same artifact);
  3. run the reference decoder executable (oracle/_ref/leaf_decoder, built
     from engine/src/decoder.cpp with leaf/cli.py:66 flags) with activation
     bits 8: `generate` for the greedy tokens, `chunked` (chunk 1) over
     prompt + tokens for the per-step decode logits and `verify` over the
     prompt for the prefill logits.

    python tests/golden/make_decoder_golden.py [tiny] [tinyllama]

Writes tests/golden/decoder_<name>.npz (+ .json with the metrics).  The
TinyLlama-shape model (config 3: 22 layers, 1.1 GB of INT8 weights) keeps
only the tokens and the first decode step's logits.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
import oracle as _oracle  # noqa: E402

REF = _oracle.reference_root() or Path(os.environ.get("LEAF_REFERENCE", "reference"))
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(REPO))

import decoder_fixture as fx  # noqa: E402
import oracle  # noqa: E402

MODELS = {
    # name: (shape, weight seed, norm noise, prompt seed, prompt length, new tokens, bits, group)
    "tiny_w8": (fx.TINY, 2024, 0.1, 11, 24, 32, 8, 64),
    "tiny_w4": (fx.TINY, 2025, 0.1, 12, 24, 32, 4, 32),
    "tinyllama_w8": (fx.TINYLLAMA, 7, 0.0, 3, 128, 128, 8, 64),
    # SmoothQuant input scales on every projection and q / k / v biases
    # (fx.smooth_variant).  The reference exporter writes input scales only
    # from calibration files, so this artifact is written by
    # decoder_fixture.write_artifact alone and run by the reference decoder.
    "tiny_smooth": (fx.TINY, 2026, 0.1, 13, 24, 32, 8, 64),
}
SMOOTH = {"tiny_smooth"}


def sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for block in iter(lambda: f.read(1 << 24), b""):
            h.update(block)
    return h.hexdigest()


def tokens_file(path: Path, requests) -> None:
    with path.open("wb") as f:
        f.write(struct.pack("<I", len(requests)))
        for ids in requests:
            f.write(struct.pack("<I", len(ids)))
            f.write(np.asarray(ids, dtype="<u4").tobytes())


def run_decoder(artifact: Path, work: Path, mode: str, ids, generate: int, threads: int):
    tokens_file(work / "tokens.bin", [ids])
    cmd = [str(oracle.REF_DECODER), str(artifact), str(work / "tokens.bin"), str(work / "logits.bin"),
           str(work / "metrics.json"), mode, str(threads), "1", "0", str(generate), "0", "1", "8"]
    out = subprocess.run(cmd, check=True, capture_output=True, text=True)
    metrics = json.loads((work / "metrics.json").read_text())
    logits = np.fromfile(work / "logits.bin", dtype="<f4")
    return out.stdout, metrics, logits


def make(name: str) -> None:
    shape, seed, noise, pseed, plen, new, bits, group = MODELS[name]
    threads = os.cpu_count() or 1
    with tempfile.TemporaryDirectory(dir=os.environ.get("TMPDIR")) as tmp:
        work = Path(tmp)
        if name in SMOOTH:
            tensors, extras = fx.smooth_variant(shape, fx.llama_tensors(shape, seed, noise), seed + 1)
            reference_artifact = work / "mine.leaf"
            fx.write_artifact(reference_artifact, shape, tensors, bits, group, extras=extras)
            digest = sha256(reference_artifact)
        else:
            fx.write_snapshot(work / "snapshot", shape, fx.llama_tensors(shape, seed, noise))
            reference_artifact = work / "reference.leaf"
            subprocess.run([sys.executable, str(REF / "tools" / "export_decoder.py"), "--model",
                            str(work / "snapshot"), "--output", str(reference_artifact), "--bits", str(bits),
                            "--group-size", str(group)], check=True, capture_output=True)
            mine = work / "mine.leaf"
            fx.write_artifact(mine, shape, fx.llama_tensors(shape, seed, noise), bits, group)
            digest = sha256(reference_artifact)
            if digest != sha256(mine):
                raise SystemExit(f"{name}: decoder_fixture.write_artifact differs from the reference exporter")
        ids = fx.prompt_ids(shape, pseed, plen)
        stdout, metrics, _ = run_decoder(reference_artifact, work, "generate", ids, new, threads)
        generated = np.asarray(metrics["generated_tokens"], dtype=np.uint32)
        streamed = [int(line.split()[1]) for line in stdout.splitlines() if line.startswith("TOKEN ")]
        assert streamed == generated.tolist()
        record = {"model": name, "artifact_sha256": digest, "bits": bits, "group": group,
                  "weight_seed": seed, "norm_noise": noise, "prompt_seed": pseed,
                  "prompt_length": plen, "new_tokens": new, "threads": threads,
                  "reference_metrics": metrics}
        arrays = {"prompt": ids, "generated": generated}
        if shape is fx.TINY:
            sequence = np.concatenate([ids, generated[:-1]])
            _, _, decode = run_decoder(reference_artifact, work, "chunked", sequence, 1, threads)
            arrays["decode_logits"] = decode.reshape(len(sequence), shape.vocab)
            _, _, prefill = run_decoder(reference_artifact, work, "verify", ids, 1, threads)
            arrays["prefill_logits"] = prefill.reshape(len(ids), shape.vocab)
        else:
            sequence = np.concatenate([ids, generated[:1]])
            _, _, last = run_decoder(reference_artifact, work, "verify", ids, 1, threads)
            arrays["prefill_last_logits"] = last.reshape(len(ids), shape.vocab)[-1]
        np.savez_compressed(HERE / f"decoder_{name}.npz", **arrays)
        (HERE / f"decoder_{name}.json").write_text(json.dumps(record, indent=1, sort_keys=True) + "\n")
        print(name, "generated", generated[:16].tolist(), "...")


if __name__ == "__main__":
    for model in sys.argv[1:] or ["tiny_w8", "tiny_w4"]:
        make(model)
