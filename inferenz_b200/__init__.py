"""inferenz_b200 -- inferenZ's mixture-of-experts layer on B200 (sm_100a).

The product is ``libinzg.so`` (C ABI: include/inzg.h, include/inzg_tools.h). This package binds it for Python hosts:
:class:`MoePool` mirrors the reference's moe_block operator, :mod:`inferenz_b200.synth` builds the seeded synthetic
configurations. Importing the package requires the built library (no fallback path exists).
"""
from ._lib import LIB_PATH, InzgError, T_F16, T_Q4L, T_Q8G, lib  # noqa: F401
from .moe import MoePool  # noqa: F401
from .gguf import GgufExperts  # noqa: F401
from . import synth  # noqa: F401
