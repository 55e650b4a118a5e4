"""Drop-in replacement for the reference ``cuda_transformer`` package.

Importing it loads ``_C`` (the sm_100a operator library, which registers
``torch.ops.cuda_transformer.*``) and ``ops`` (the Python wrappers), exactly
like ``cuda_transformer/__init__.py:3`` of the reference.  ``_C`` is built in
tree by ``python -m cuda_transformer_b200.build``; there is no fallback when
it is missing.
"""
from . import _C, ops  # noqa: F401
