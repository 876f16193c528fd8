"""Drop-in module with the reference's module name and public names (``from kernel import ...``).

Re-exports the B200-native operator so code written against yliu-fort/first-passage-attention's ``kernel.py``
(its tests and benchmark included) runs unchanged; ``impl="triton"`` selects the native CUDA kernels.
"""
from first_passage_attention_b200 import Field, FirstPassageAttention, first_passage_attention, first_passage_bias  # noqa: F401

__all__ = ["first_passage_attention", "first_passage_bias", "Field", "FirstPassageAttention"]
