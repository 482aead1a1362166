"""Drop-in module for spanqr's entry point (reference orth.py:13-20): `from orth import orth`.

    from orth import orth
    Q = orth(X)          # X: fp32 CUDA [K, r] -> Q: fp32 CUDA [K, r], orthonormal columns, span(Q) = span(X)
"""
from spanqr_b200 import orth, orth_batched

__all__ = ["orth", "orth_batched"]
