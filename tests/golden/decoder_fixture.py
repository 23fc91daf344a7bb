"""Decoder fixtures for the tests: the seeded models and artifact writer of
oracle/fixture.py."""
from oracle.fixture import *  # noqa: F401,F403
from oracle.fixture import LlamaShape, TINY, TINYLLAMA, llama_tensors, prompt_ids, quantize, smooth_variant, write_artifact, write_snapshot  # noqa: F401
