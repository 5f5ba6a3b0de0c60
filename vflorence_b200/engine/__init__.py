"""A decode engine around the paged path, used to measure end-to-end decode tokens/s and to check
token parity with the reference engine: continuous batching over whole requests, greedy and beam
search with copy-on-write block sharing, encoder K/V paged once per request. The models are
HuggingFace transformers modules (BART, Florence-2) running as stock torch on the GPU; their
decoder attention goes through the ``vflorence::`` custom ops (the paged kernels)."""

from .engine import Engine, Request
from .sampling import SamplingParams

__all__ = ["Engine", "Request", "SamplingParams"]
