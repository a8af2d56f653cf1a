"""sycl_minimax_h3_b200 - the MiniMax-H3 denoiser self-attention path on NVIDIA B200 (sm_100a).

The product is two C-ABI libraries built from ``csrc/`` into ``lib/``:

* ``libh3cuda.so`` - the attention subset of the reference's ``kernels/h3sycl.h`` (contexts, device memory, copies,
  ``h3s_attention``, ``h3s_attention_batch``), declared in ``include/h3cuda.h``;
* ``libh3sage.so`` - the SageAttention plugin (``include/h3sage.h``), loaded by libh3cuda.so from its own directory.

This package is the Python host side over that ABI: ``native`` (ctypes bindings, fails loudly when the libraries are
missing), ``ops`` (``Rows`` / ``attention`` / ``attention_batch``, the reference engine's operator interface from
``engine/h3-core/src/ops.rs``) and ``ulysses`` (the sequence-parallel all-to-all over NCCL).
"""
from .native import H3Error, Context, lib, sage_lib, LIB_DIR  # noqa: F401

__all__ = ["H3Error", "Context", "lib", "sage_lib", "LIB_DIR"]
