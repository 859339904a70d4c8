"""On-disk / in-memory formats: 2-bit codebook, fragment-major planes,
FP8 UE8M0 block formats, NVFP4 KV rows."""
from . import codebook, fp8, kv_nvfp4, planes  # noqa: F401
from .codebook import QUANTIZER_ABI  # noqa: F401
