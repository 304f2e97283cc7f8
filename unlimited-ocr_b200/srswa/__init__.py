"""srswa -- B200 (sm_100a) SR-SWA hot path of Unlimited-OCR 2.

Python side of libsrswa.so: the reference's operator interface for the
Sparse-Reference Sliding-Window Attention path, with the same names and
contracts, running on hand-written CUDA kernels.

Modules (each mirrors a reference module):
  sparse_gather       hf-model-code/sparse_gather_triton.py
  sparse_gather_e2e   hf-model-code/sparse_gather_e2e_triton.py
  dash_infer          router/decode functions of hf-model-code/modeling_deepseekv2.py
  paged               SGLang unlimited_dash_ops (paged decode, k_bar cache, routing)
  ops                 one wrapper per C entry point (include/srswa.h)
  dropin              installs the above into the reference's module namespace
"""

from ._lib import LIB_PATH, SrswaError, lib  # noqa: F401

__version__ = "0.1.0"
