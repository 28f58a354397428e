"""vllm_b200: B200-native paged-attention + continuous-batching hot path of vllm-jax.

The CUDA kernels live in libvjattn.so (built by `python -m vllm_b200.build`);
`Engine` / `LLM` keep vllm-jax's `generate` API."""
from .config import Config
from .sampling_params import SamplingParams

__all__ = ["Config", "SamplingParams", "Engine", "LLM"]


def __getattr__(name):
    if name in ("Engine", "LLM"):
        from .src.engine import Engine
        return Engine
    raise AttributeError(name)
