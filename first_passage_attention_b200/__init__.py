"""B200-native First Passage Attention (sm_100a CUDA kernels behind a C ABI, PyTorch host side).

Drop-in for yliu-fort/first-passage-attention's ``kernel.py`` public API:
``first_passage_attention``, ``first_passage_bias``, ``Field``, ``FirstPassageAttention``.
"""
from .ops import (Field, FirstPassageAttention, LaunchStats, first_passage_attention, first_passage_bias,  # noqa: F401
                  fpa_backward, fpa_forward)

__all__ = ["first_passage_attention", "first_passage_bias", "Field", "FirstPassageAttention"]
