"""GDN decode entry point: drop-in for the reference's ``gdn_decode`` / ``kernel``.

Mirrors ``gdn_decode`` of the reference (gdn_decode/solution/triton/kernel.py:221-272):
same positional arguments, destination-passing outputs, same defaults
(``state=None`` -> zero state, ``scale`` None/0 -> 1/sqrt(head_size),
``output``/``new_state`` None -> allocated), same return value
``(output, new_state)``.  The work is one launch of the sm_100a kernel in
``csrc/gdn_decode.cu`` through the C ABI ``gdn_decode_launch``, on the current
CUDA stream, with no host synchronisation.
"""
from __future__ import annotations

import torch

from . import _checks as C
from ._lib import LIB, check


def gdn_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output=None, new_state=None,
               *, use_qk_l2norm: bool = False):
    """One decode step; ``use_qk_l2norm`` L2-normalises q and k in-kernel (fp32).

    ``state`` / ``new_state`` may be fp32 (``gdn_decode_launch``) or bf16
    (``gdn_decode_launch_bf16state``: widened on load, updated in fp32, rounded on
    store; half the state traffic); both must then have the same dtype, which is taken
    from ``state``, else from ``new_state``, else fp32.

    Like the reference, which hands every stride to its kernel, q, k, v, a, b and
    ``output`` may be views whose batch rows are strided (slices of a fused projection,
    say): with fp32 state they go to ``gdn_decode_launch_strided`` as they are.  Other
    layouts, strided rows with bf16 state, and q / k not 8-byte aligned (or a state not
    16-byte aligned) are copied into dense tensors on the device first, and a non-dense
    ``output`` / ``new_state`` is written through a dense temporary."""
    dev = C.cuda_device(q)
    C.tensor("q", q, torch.bfloat16, 4, dev, strided=True)
    C.tensor("k", k, torch.bfloat16, 4, dev, strided=True)
    C.tensor("v", v, torch.bfloat16, 4, dev, strided=True)
    B, T, HQ, D = q.shape
    HK = k.shape[2]
    HV = v.shape[2]
    if T != 1:
        raise ValueError(f"decode expects seq_len == 1, got {T}")
    C.heads(HQ, HK, HV, D)
    C.shape("k", k, (B, 1, HK, D))
    C.shape("v", v, (B, 1, HV, D))
    sdt = state.dtype if isinstance(state, torch.Tensor) else (
        new_state.dtype if isinstance(new_state, torch.Tensor) else torch.float32)
    if sdt not in (torch.float32, torch.bfloat16):
        raise TypeError(f"state must be float32 or bfloat16, got {sdt}")
    if state is not None:
        C.tensor("state", state, sdt, 4, dev, strided=True)
        C.shape("state", state, (B, HV, D, D))
    C.tensor("A_log", A_log, torch.float32, 1, dev, strided=True)
    C.shape("A_log", A_log, (HV,))
    C.tensor("dt_bias", dt_bias, torch.float32, 1, dev, strided=True)
    C.shape("dt_bias", dt_bias, (HV,))
    C.tensor("a", a, torch.bfloat16, 3, dev, strided=True)
    C.shape("a", a, (B, 1, HV))
    C.tensor("b", b, torch.bfloat16, 3, dev, strided=True)
    C.shape("b", b, (B, 1, HV))
    sc = C.scale_arg(scale)
    if output is None:
        output = torch.empty(B, 1, HV, D, dtype=torch.bfloat16, device=dev)
    else:
        C.tensor("output", output, torch.bfloat16, 4, dev, strided=True)
        C.shape("output", output, (B, 1, HV, D))
    if new_state is None:
        new_state = torch.empty(B, HV, D, D, dtype=sdt, device=dev)
    else:
        C.tensor("new_state", new_state, sdt, 4, dev, strided=True)
        C.shape("new_state", new_state, (B, HV, D, D))
    if B == 0:
        return output, new_state
    state_in, A_log, dt_bias = C.dense_or_copy(state, 16), C.dense_or_copy(A_log), \
        C.dense_or_copy(dt_bias)
    ns = new_state if (new_state.is_contiguous() and new_state.data_ptr() % 16 == 0) else \
        torch.empty(new_state.shape, dtype=sdt, device=dev)
    if ns is not new_state and state is not None and state_in.data_ptr() == new_state.data_ptr():
        state_in = state_in.clone()  # keep the in-place contract through the temporary
    if sdt == torch.bfloat16:  # dense rows only
        q, k, v, a, b = (C.dense_or_copy(x) for x in (q, k, v, a, b))
    (q, qs), (k, ks) = C.rows_in(q, 4, 8), C.rows_in(k, 4, 8)  # 8-byte q / k loads
    (v, vs), (a, as_), (b, bs) = C.rows_in(v), C.rows_in(a), C.rows_in(b)
    out, os_, out_back = C.rows_out(output) if sdt == torch.float32 else (
        (output, None, False) if output.is_contiguous() else
        (torch.empty(output.shape, dtype=output.dtype, device=dev), None, True))
    common = (q.data_ptr(), k.data_ptr(), v.data_ptr(),
              state_in.data_ptr() if state_in is not None else None,
              A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), sc,
              out.data_ptr(), ns.data_ptr(), B, HQ, HK, HV, D, int(bool(use_qk_l2norm)))
    dense = (HQ * D, HQ * D, HV * D, HV, HV, HV * D)
    if sdt == torch.bfloat16:
        name = "gdn_decode_launch_bf16state"
        status = LIB.gdn_decode_launch_bf16state(*common, C.stream_handle(dev))
    elif (qs, ks, vs, as_, bs, os_) == dense:
        name = "gdn_decode_launch"
        status = LIB.gdn_decode_launch(*common, C.stream_handle(dev))
    else:
        name = "gdn_decode_launch_strided"
        status = LIB.gdn_decode_launch_strided(*common, qs, ks, vs, as_, bs, os_,
                                               C.stream_handle(dev))
    check(name, status)
    if out_back:
        output.copy_(out)
    if ns is not new_state:
        new_state.copy_(ns)
    return output, new_state


def kernel(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    """flashinfer-bench DPS entry point (11 parameters, no normalisation)."""
    return gdn_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)
