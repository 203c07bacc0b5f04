"""Blackwell-native (sm_100a) executor for the nvcr.intconv.v1 exact-convolution path.

The compute path is hand-written CUDA in ``nvcr_b200/csrc`` built into
``nvcr_b200/_build/libnvcr_sm100.so`` and reached through the C ABI declared in
``include/nvcr_sm100.h``. This package holds the host-side mirror of the
reference's program model (``program``) and executor (``executor``) and the
benchmark workloads (``workloads``).
"""
from .program import INTCONV_PROFILE, Node, OpKind, Program, SeededStream  # noqa: F401
