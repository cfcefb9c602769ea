"""B200 (sm_100a) speculative-decoding verify path with the API of jax_ssd.

The CUDA library ``libssdverify.so`` (built in this directory) is loaded on
first use; every compute call goes through it, there is no CPU fallback.
"""

from .config import DecodeMode, SSDConfig
from .sampling_params import SamplingParams

__all__ = ["LLM", "DecodeMode", "SSDConfig", "SamplingParams"]


def __getattr__(name):
    if name == "LLM":
        from .llm import LLM

        return LLM
    raise AttributeError(name)
