"""B200 (sm_100a) Gated DeltaNet decode and prefill kernels.

Drop-in replacements for the two flashinfer-bench solution entry points of the
MLSys26 FlashInfer contest GDN track:

* ``gdn_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)``
* ``gdn_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state)``

(``decode_kernel`` / ``prefill_kernel`` are the exact-arity DPS forms, also
exposed as ``decode.kernel`` / ``prefill.kernel``), plus the multi-token decode of
the ``gdn_mtp`` definition (``gdn_mtp`` / ``mtp_kernel``) for speculative-decoding
verification over a state pool, and ``chunk_gated_delta_rule`` (FlashInfer's prefill
argument order: precomputed gates, state checkpoints every N tokens).  All compute runs
in the in-tree CUDA library ``libgdn_b200.so`` through its C ABI
(``include/gdn_b200.h``); importing this package fails if it is not built.

The directory name is not a Python identifier; import it with
``importlib.import_module("mlsys26-flashinfer-ai-kernel-generation-contest_b200")``.
"""
from ._lib import LIB, LIB_PATH, GDNError, device_error  # noqa: F401
from .decode import gdn_decode, kernel as decode_kernel  # noqa: F401
from .prefill import (chunk_gated_delta_rule, gdn_prefill, gdn_prefill_recurrent,  # noqa: F401
                      gdn_prefill_segmented, kernel as prefill_kernel, workspace_bytes)
from .mtp import gdn_mtp, kernel as mtp_kernel  # noqa: F401
from . import decode, mtp, prefill, sharding, workloads  # noqa: F401

__all__ = ["gdn_decode", "gdn_prefill", "gdn_prefill_recurrent", "gdn_prefill_segmented",
           "gdn_mtp", "decode_kernel",
           "mtp_kernel", "chunk_gated_delta_rule",
           "prefill_kernel", "workloads", "sharding", "GDNError", "LIB", "LIB_PATH", "workspace_bytes",
           "device_error"]
