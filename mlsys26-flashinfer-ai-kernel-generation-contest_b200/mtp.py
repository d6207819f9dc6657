"""GDN multi-token decode (speculative-decoding verification) over a state pool.

Mirrors the flashinfer-bench definition ``gdn_mtp`` (``_gdn_mtp_reference``,
flashinfer/trace/templates/gdn.py:379-466; inputs and outputs as gdn.py:469-560):
``seq_len`` tokens per batch row applied in order to the state of pool slot
``initial_state_indices[row]``, with an optional buffer that receives the state
after every token (for rollback of rejected draft tokens).  One launch of the
sm_100a kernel in ``csrc/gdn_mtp.cu`` through the C ABI ``gdn_mtp_launch``.

Pool semantics: ``final_state`` is the pool with each row's slot replaced by its
state after the last token.  Passing ``final_state=initial_state`` (or nothing)
updates the pool in place, which is what a serving stack does; a separate
``final_state`` buffer is first filled with the initial pool (one device copy), so
the result equals the definition's.  A row whose slot lies outside [0, pool_size)
is padding: zero output, no state change.  Rows must use distinct slots.
"""
from __future__ import annotations

import torch

from . import _checks as C
from ._lib import LIB, check


def gdn_mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
            output=None, final_state=None, intermediate_states_buffer=None, *,
            use_qk_l2norm: bool = False):
    """Returns ``(output, final_state)``; ``use_qk_l2norm`` L2-normalises q and k in-kernel.

    The pool (and the rollback buffer, which must match it) may be fp32 or bf16
    (``gdn_mtp_launch_bf16state``: carried in fp32 through the tokens, rounded on store)."""
    dev = C.cuda_device(q)
    C.tensor("q", q, torch.bfloat16, 4, dev)
    C.tensor("k", k, torch.bfloat16, 4, dev)
    C.tensor("v", v, torch.bfloat16, 4, dev)
    B, T, HQ, D = q.shape
    HK = k.shape[2]
    HV = v.shape[2]
    C.heads(HQ, HK, HV, D)
    C.shape("k", k, (B, T, HK, D))
    C.shape("v", v, (B, T, HV, D))
    if not isinstance(initial_state, torch.Tensor):
        raise TypeError("initial_state must be a torch.Tensor")
    sdt = initial_state.dtype
    if sdt not in (torch.float32, torch.bfloat16):
        raise TypeError(f"initial_state must be float32 or bfloat16, got {sdt}")
    C.tensor("initial_state", initial_state, sdt, 4, dev)
    P = initial_state.shape[0]
    C.shape("initial_state", initial_state, (P, HV, D, D))
    idx = initial_state_indices
    if not isinstance(idx, torch.Tensor) or idx.dtype not in (torch.int32, torch.int64):
        raise TypeError("initial_state_indices must be an int32 or int64 tensor")
    if idx.dim() != 1 or idx.numel() != B or idx.device != dev or not idx.is_contiguous():
        raise ValueError(f"initial_state_indices must be a contiguous [{B}] tensor on {dev}")
    C.tensor("A_log", A_log, torch.float32, 1, dev)
    C.shape("A_log", A_log, (HV,))
    C.tensor("dt_bias", dt_bias, torch.float32, 1, dev)
    C.shape("dt_bias", dt_bias, (HV,))
    C.tensor("a", a, torch.bfloat16, 3, dev)
    C.shape("a", a, (B, T, HV))
    C.tensor("b", b, torch.bfloat16, 3, dev)
    C.shape("b", b, (B, T, HV))
    sc = C.scale_arg(scale)
    if output is None:
        output = torch.empty(B, T, HV, D, dtype=torch.bfloat16, device=dev)
    else:
        C.tensor("output", output, torch.bfloat16, 4, dev)
        C.shape("output", output, (B, T, HV, D))
    if final_state is None:
        final_state = initial_state
    else:
        C.tensor("final_state", final_state, sdt, 4, dev)
        C.shape("final_state", final_state, (P, HV, D, D))
        if final_state.data_ptr() != initial_state.data_ptr():
            final_state.copy_(initial_state)  # slots no row references keep their value
    inter = intermediate_states_buffer
    if inter is not None:
        C.tensor("intermediate_states_buffer", inter, sdt, 5, dev)
        C.shape("intermediate_states_buffer", inter, (P, T, HV, D, D))
    launch = LIB.gdn_mtp_launch if sdt == torch.float32 else LIB.gdn_mtp_launch_bf16state
    status = launch(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), final_state.data_ptr(), idx.data_ptr(),
        int(idx.dtype == torch.int64), A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(),
        b.data_ptr(), sc, output.data_ptr(), final_state.data_ptr(),
        inter.data_ptr() if inter is not None else None, B, T, P, HQ, HK, HV, D,
        int(bool(use_qk_l2norm)), C.stream_handle(dev))
    check("gdn_mtp_launch" + ("" if sdt == torch.float32 else "_bf16state"), status)
    return output, final_state


def kernel(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
           intermediate_states_buffer, output, final_state):
    """flashinfer-bench DPS form of the ``gdn_mtp`` definition: its inputs in order
    (``intermediate_states_buffer`` may be None), then the outputs; no normalisation."""
    return gdn_mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
                   output, final_state, intermediate_states_buffer)
