"""vllm_moet_b200: a B200-native (sm_100a) MoE inference engine with 2-bit
codebook experts, MLA attention and MTP speculative decoding."""
import torch  # noqa: F401  (loads libc10 before the native extension)

__version__ = "0.1.0"

from .config import EngineConfig, ModelConfig, MoetConfig, ParallelConfig, get_preset  # noqa: F401
from .engine.sampling_params import RequestOutput, SamplingParams  # noqa: F401
from .engine.beam_search import BeamSearchOutput, BeamSearchParams  # noqa: F401


def __getattr__(name):
    if name == "LLM":
        from .engine.llm import LLM
        return LLM
    raise AttributeError(name)
