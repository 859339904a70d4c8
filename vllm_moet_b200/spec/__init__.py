"""Speculative decoding beyond MTP: the DSpark block drafter and its
hardware-aware width scheduler, and the rejection samplers."""
from .dspark import DSparkDrafter, allocate_widths, swa_indices, swa_indices_batch  # noqa: F401
from .rejection import greedy_accept, rejection_sample  # noqa: F401
