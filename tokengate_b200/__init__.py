"""tokengate_b200 — B200-native (sm_100a) kernels for TokenGate's gated prefill.

The compute path is a C-ABI shared library (include/tokengate_b200.h) with
four hand-written kernels: key-bias causal GQA attention (tcgen05/TMEM),
the gate scorer, the radix top-K selection and the row compaction. The
Python modules mirror the reference's operator surface on top of it.
"""
from . import _lib
from ._lib import TokenGateKernelError, TokenGateArgumentError, TokenGateUnsupportedError

__all__ = ["TokenGateKernelError", "TokenGateArgumentError", "TokenGateUnsupportedError"]
