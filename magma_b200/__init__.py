"""magma_b200 — sm_100a (B200) execution backend for Magma's training hot path.

The kernels live in ``libmagma_cuda.so`` (C ABI in ``include/magma_cuda.h``);
``magma_b200.lib`` binds it with ctypes, ``magma_b200.ops`` is the torch-tensor
front end, ``magma_b200.gpt`` / ``magma_b200.mlp`` are the training steps built
only from those ops, and ``magma_b200.dp`` the data-parallel gradient sync.
"""
from . import lib  # noqa: F401

__all__ = ["lib"]
__version__ = "0.1.0"
