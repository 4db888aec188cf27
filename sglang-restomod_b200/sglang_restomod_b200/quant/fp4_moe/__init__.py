"""NVFP4 fused MoE on B200 (the ``fp4_moe`` component); see :mod:`.method`."""

from __future__ import annotations


def register() -> None:
    from .method import install

    install()
