"""rbk — host side of the B200 backward-pass library for rubidium-train.

``rbk.ops`` wraps the individual kernels (the reference's cuda_kernels.cuh
operators); ``rbk.model`` is the RubidiumTransformer drop-in (src/model.h).
Everything dispatches to librbk.so through its C ABI (include/rbk.h).
"""
from ._lib import LIB_PATH, RbkError, declared_symbols, lib  # noqa: F401
