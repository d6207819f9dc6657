"""GDN prefill entry point: drop-in for the reference's ``gdn_prefill`` / ``kernel``.

Mirrors ``gdn_prefill`` of the reference (gdn_prefill/solution/triton/kernel.py:253-337):
same positional arguments, destination-passing outputs, same defaults
(``state=None`` -> zero initial state, ``scale`` None/0 -> 1/sqrt(head_size),
outputs allocated when None), same return ``(output, new_state)``.  Unlike the
reference wrapper it accepts any head counts with num_v_heads a multiple of
num_q_heads == num_k_heads (the reference asserts 4/4/8, kernel.py:271-274),
and it issues no zero-fill or state-copy passes: the kernels write every
output element themselves.  ``cu_seqlens`` is read on the device only (int32
or int64), so the call never synchronises the host.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _checks as C
from ._lib import (GDN_PREFILL_AUTO, GDN_PREFILL_FUSED, GDN_PREFILL_RECURRENT, GDN_PREFILL_SPLIT,
                   LIB, check)

# kernel= choices of gdn_prefill (see gdn_prefill_launch_variant in include/gdn_b200.h)
KERNELS = {"auto": GDN_PREFILL_AUTO, "recurrent": GDN_PREFILL_RECURRENT,
           "fused": GDN_PREFILL_FUSED, "split": GDN_PREFILL_SPLIT}
_LPT_MAX_SEQS = 8192  # the longest-first ordering kernel's capacity

_ws_lock = threading.Lock()
_ws_cache = {}
_ws_retired = []  # superseded buffers: a CUDA graph captured over an earlier call still uses them


def _workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    """Persistent per-device scratch buffer, grown on demand (contents are
    rewritten by every call that uses them).  A buffer that is outgrown is kept
    alive, not freed, so that CUDA graphs captured over earlier calls stay valid;
    growth at least doubles, so few are ever retired."""
    key = (dev.index if dev.index is not None else torch.cuda.current_device())
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            grow = max(nbytes, 1 << 20, 2 * buf.numel() if buf is not None else 0)
            if buf is not None:
                _ws_retired.append(buf)
            buf = torch.empty(grow, dtype=torch.uint8, device=dev)
            _ws_cache[key] = buf
        return buf


def workspace_bytes(total_tokens: int, num_seqs: int, num_q_heads: int, num_v_heads: int,
                    head_size: int = 128, kernel: str = "auto") -> int:
    return int(LIB.gdn_prefill_workspace_size_variant(KERNELS[kernel], total_tokens, num_seqs,
                                                      num_q_heads, num_v_heads, head_size))


def resolved_kernel(total_tokens: int, num_seqs: int, num_q_heads: int, num_v_heads: int,
                    kernel: str = "auto") -> str:
    """The kernel family `kernel` runs for these sizes (16-byte aligned buffers)."""
    if kernel != "auto" or total_tokens <= 0 or num_seqs <= 0:
        return kernel if total_tokens > 0 else "recurrent"
    split = LIB.gdn_prefill_workspace_size_variant(GDN_PREFILL_SPLIT, total_tokens, num_seqs,
                                                   num_q_heads, num_v_heads, 128)
    auto = LIB.gdn_prefill_workspace_size_variant(GDN_PREFILL_AUTO, total_tokens, num_seqs,
                                                  num_q_heads, num_v_heads, 128)
    return "split" if auto == split else "fused"


def launches_per_call(total_tokens: int, num_seqs: int, num_q_heads: int = 16,
                      num_v_heads: int = 32, kernel: str = "auto") -> int:
    """Number of this library's kernels one prefill call launches."""
    if num_seqs <= 0:
        return 0
    kind = resolved_kernel(total_tokens, num_seqs, num_q_heads, num_v_heads, kernel)
    lpt = 1 if 1 < num_seqs <= _LPT_MAX_SEQS else 0
    if kind == "split":  # order, chunk offsets, preparation, state
        return lpt + 3
    if kind == "fused":
        return lpt + 1
    return 1


def gdn_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output=None,
                new_state=None, *, use_qk_l2norm: bool = False, kernel: str = "auto"):
    """Varlen prefill; ``use_qk_l2norm`` L2-normalises q and k in-kernel (fp32).

    ``kernel="auto"`` calls ``gdn_prefill_launch`` (the reference-facing entry
    point); "split", "fused" and "recurrent" force one kernel family through
    ``gdn_prefill_launch_variant``."""
    if kernel not in KERNELS:
        raise ValueError(f"kernel must be one of {sorted(KERNELS)}, got {kernel!r}")
    if kernel == "auto":
        launch, name = LIB.gdn_prefill_launch, "gdn_prefill_launch"
    else:
        variant = KERNELS[kernel]
        name = f"gdn_prefill_launch_variant({kernel})"

        def launch(*args):
            return LIB.gdn_prefill_launch_variant(variant, *args)
    return _prefill(launch, name, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
                    output, new_state, use_qk_l2norm, kernel, KERNELS[kernel])


def gdn_prefill_recurrent(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output=None,
                          new_state=None, *, use_qk_l2norm: bool = False):
    """Same contract as :func:`gdn_prefill` through the token-serial CUDA-core kernel
    (``gdn_prefill_launch_recurrent``): the definition's recurrence step by step."""
    return _prefill(LIB.gdn_prefill_launch_recurrent, "gdn_prefill_launch_recurrent", q, k, v,
                    state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                    use_qk_l2norm, "recurrent", GDN_PREFILL_RECURRENT)


def _prefill(launch, name, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
             new_state, use_qk_l2norm, kernel, variant):
    """Checks, then one launch.  Like the reference, which hands every stride to its
    kernel, q, k, v, a, b and ``output`` may be views whose token rows are strided (slices
    of a fused projection, say): those go to ``gdn_prefill_launch_strided`` as they are.
    Other layouts, and q / k / v / output whose rows or first element are not 16-byte
    aligned, are copied into dense tensors on the device first (a non-dense or unaligned
    ``output`` / ``new_state`` is written through a dense temporary), so that the
    tensor-core kernels always apply; the C ABI itself runs the token-serial kernel for
    such buffers."""
    dev = C.cuda_device(q)
    C.tensor("q", q, torch.bfloat16, 3, dev, strided=True)
    C.tensor("k", k, torch.bfloat16, 3, dev, strided=True)
    C.tensor("v", v, torch.bfloat16, 3, dev, strided=True)
    T, HQ, D = q.shape
    HK = k.shape[1]
    HV = v.shape[1]
    C.heads(HQ, HK, HV, D)
    C.shape("k", k, (T, HK, D))
    C.shape("v", v, (T, HV, D))
    if not isinstance(cu_seqlens, torch.Tensor):
        raise TypeError("cu_seqlens must be a torch.Tensor")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"cu_seqlens must be int32 or int64, got {cu_seqlens.dtype}")
    if cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
        raise ValueError("cu_seqlens must be 1-D with num_seqs + 1 entries")
    if cu_seqlens.device != dev:
        raise ValueError("cu_seqlens must be on the same device as q")
    N = cu_seqlens.numel() - 1
    H = max(HQ, HV)
    if state is not None:
        C.tensor("state", state, torch.float32, 4, dev, strided=True)
        C.shape("state", state, (N, HV, D, D))
    C.tensor("A_log", A_log, torch.float32, 1, dev, strided=True)
    C.shape("A_log", A_log, (HV,))
    C.tensor("dt_bias", dt_bias, torch.float32, 1, dev, strided=True)
    C.shape("dt_bias", dt_bias, (HV,))
    C.tensor("a", a, torch.bfloat16, 2, dev, strided=True)
    C.shape("a", a, (T, HV))
    C.tensor("b", b, torch.bfloat16, 2, dev, strided=True)
    C.shape("b", b, (T, HV))
    sc = C.scale_arg(scale)
    if output is None:
        output = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
    else:
        C.tensor("output", output, torch.bfloat16, 3, dev, strided=True)
        C.shape("output", output, (T, H, D))
    if new_state is None:
        new_state = torch.empty(N, H, D, D, dtype=torch.float32, device=dev)
    else:
        C.tensor("new_state", new_state, torch.float32, 4, dev, strided=True)
        C.shape("new_state", new_state, (N, H, D, D))
    if N == 0:
        return output, new_state
    cu_seqlens = C.dense_or_copy(cu_seqlens, 8)
    state_in, A_log, dt_bias = C.dense_or_copy(state, 16), C.dense_or_copy(A_log), \
        C.dense_or_copy(dt_bias)
    ns = new_state if (new_state.is_contiguous() and new_state.data_ptr() % 16 == 0) else \
        torch.empty(new_state.shape, dtype=torch.float32, device=dev)
    if ns is not new_state and state is not None and state_in.data_ptr() == new_state.data_ptr():
        state_in = state_in.clone()  # keep the in-place contract through the temporary
    # the tensor-core kernels read q / k / v tiles by TMA and store 16-byte output pieces:
    # views whose rows or first element are not 16-byte aligned are copied (else the call
    # would fall back to the token-serial kernel)
    (q, qs), (k, ks), (v, vs) = C.rows_in(q, 8, 16), C.rows_in(k, 8, 16), C.rows_in(v, 8, 16)
    (a, as_), (b, bs) = C.rows_in(a), C.rows_in(b)
    out, os_, out_back = C.rows_out(output, 8, 16)
    ws_n = workspace_bytes(T, N, HQ, HV, D, kernel)
    ws = _workspace(dev, ws_n) if ws_n > 0 else None
    head = (q.data_ptr(), k.data_ptr(), v.data_ptr(),
            state_in.data_ptr() if state_in is not None else None,
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
            cu_seqlens.data_ptr(), int(cu_seqlens.dtype == torch.int64), sc,
            out.data_ptr(), ns.data_ptr(), T, N, HQ, HK, HV, D, int(bool(use_qk_l2norm)))
    tail = (ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            C.stream_handle(dev))
    if (qs, ks, vs, as_, bs, os_) == (HQ * D, HQ * D, HV * D, HV, HV, H * D):
        status = launch(*head, *tail)
    else:
        name = f"gdn_prefill_launch_strided({kernel})"
        status = LIB.gdn_prefill_launch_strided(variant, *head, qs, ks, vs, as_, bs, os_, *tail)
    check(name, status)
    if out_back:
        output.copy_(out)
    if ns is not new_state:
        new_state.copy_(ns)
    return output, new_state


def segments_auto(total_tokens: int, num_v_heads: int) -> int:
    """Segment count gdn_prefill_segmented picks for `segments` = 0 on the current device:
    the largest S whose 2 S - 1 runs (four state CTAs per run and v-head) fit on the SMs
    at once, capped at the number of 64-token chunks."""
    return int(LIB.gdn_prefill_segments_auto(total_tokens, num_v_heads))


def segment_plan(total_tokens: int, num_v_heads: int, segments: int = 0, sms: int = 0):
    """Token bounds [0, b_1, .., T] of the segments gdn_prefill_segmented cuts: `segments`
    equal shares of the chunks, or for 0 the plan of the library's cost model on `sms`
    SMs (0: the current device's)."""
    buf = (ctypes.c_int * 66)()
    S = int(LIB.gdn_prefill_segment_plan(total_tokens, num_v_heads, segments, sms, buf, 66))
    if S < 1:
        raise ValueError(f"gdn_prefill_segment_plan: {LIB.gdn_status_string(S).decode()}")
    return [int(buf[i]) for i in range(S + 1)]


def segmented_launches(segments: int) -> int:
    """Number of this library's kernels one gdn_prefill_segmented call launches."""
    if segments <= 1:  # run and chunk offsets, preparation, state
        return 3
    # + state-map chain, outputs
    return 5


def gdn_prefill_segmented(q, k, v, state, A_log, a, dt_bias, b, scale, output=None,
                          new_state=None, *, segments: int = 0, bounds=None,
                          use_qk_l2norm: bool = False):
    """Prefill of ONE sequence whose v-heads alone leave most SMs idle (a sequence sharded
    by q/k-head group over several GPUs, or a model with few heads per GPU), split into
    token segments that run side by side in a single launch of the split kernels
    (``gdn_prefill_segmented_launch``): segment 0 from the initial state, every later
    segment twice, from a zero state (its map's B and outputs o^0) and from the identity
    with v = 0 (A and o^I), all reading the tokens in place.  Over a segment the recurrence
    is affine in its start state, so the library's chain kernel then composes the maps and
    its output kernel forms o = S_start o^I + o^0 for every later segment.  The serial
    chunk chain shrinks from the whole sequence to one segment; there is no collective.

    q, k [T, HQ, 128], v [T, HV, 128], a, b [T, HV] bf16 (token rows may be strided);
    state [1, HV, 128, 128] fp32 or None; returns (output [T, HV, 128] bf16, new_state
    [1, HV, 128, 128] fp32).  `segments` = S > 0 cuts S equal segments, 0 takes the
    library's plan for the device (segment_plan); `bounds` = [0, b_1, .., T] (interior
    bounds multiples of 64) gives the segments explicitly.  One segment is an ordinary
    split-kernel prefill.  The outputs of the later segments carry one more bf16 rounding
    (of o^I); the final state is fp32 throughout."""
    dev = C.cuda_device(q)
    C.tensor("q", q, torch.bfloat16, 3, dev, strided=True)
    C.tensor("k", k, torch.bfloat16, 3, dev, strided=True)
    C.tensor("v", v, torch.bfloat16, 3, dev, strided=True)
    T, HQ, D = q.shape
    HK, HV = k.shape[1], v.shape[1]
    C.heads(HQ, HK, HV, D)
    C.shape("k", k, (T, HK, D))
    C.shape("v", v, (T, HV, D))
    for name, x, shp in (("A_log", A_log, (HV,)), ("dt_bias", dt_bias, (HV,))):
        C.tensor(name, x, torch.float32, 1, dev, strided=True)
        C.shape(name, x, shp)
    for name, x in (("a", a), ("b", b)):
        C.tensor(name, x, torch.bfloat16, 2, dev, strided=True)
        C.shape(name, x, (T, HV))
    if state is not None:
        C.tensor("state", state, torch.float32, 4, dev, strided=True)
        C.shape("state", state, (1, HV, D, D))
    for name, x, shp, dt in (("output", output, (T, HV, D), torch.bfloat16),
                             ("new_state", new_state, (1, HV, D, D), torch.float32)):
        if x is not None:
            C.tensor(name, x, dt, len(shp), dev, strided=True)
            C.shape(name, x, shp)
    if segments < 0:
        raise ValueError("segments must be >= 0")
    sc = C.scale_arg(scale)
    if output is None:
        output = torch.empty(T, HV, D, dtype=torch.bfloat16, device=dev)
    if new_state is None:
        new_state = torch.empty(1, HV, D, D, dtype=torch.float32, device=dev)
    if T == 0:  # an empty sequence's final state is zero (definition semantics)
        return output, new_state.zero_()
    state_in, A_log, dt_bias = C.dense_or_copy(state, 16), C.dense_or_copy(A_log), \
        C.dense_or_copy(dt_bias)
    dense = lambda x: x.is_contiguous() and x.data_ptr() % 16 == 0  # noqa: E731
    ns = new_state if dense(new_state) else torch.empty(1, HV, D, D, dtype=torch.float32,
                                                        device=dev)
    if ns is not new_state and state is not None and state_in.data_ptr() == new_state.data_ptr():
        state_in = state_in.clone()  # keep the in-place contract through the temporary
    out = output if dense(output) else torch.empty(T, HV, D, dtype=torch.bfloat16, device=dev)
    (q, qs), (k, ks), (v, vs) = C.rows_in(q, 8, 16), C.rows_in(k, 8, 16), C.rows_in(v, 8, 16)
    (a, as_), (b, bs) = C.rows_in(a), C.rows_in(b)
    cb = None
    if bounds is not None:
        bounds = [int(x) for x in bounds]
        segments = len(bounds) - 1
        cb = (ctypes.c_int * len(bounds))(*bounds)
    ws_n = int(LIB.gdn_prefill_segmented_workspace_size(T, HV, segments, cb))
    ws = _workspace(dev, ws_n + 1024) if ws_n > 0 else None
    ws_ptr = ws_len = 0
    if ws is not None:  # the launch wants its workspace 1024-byte aligned
        ws_ptr = (ws.data_ptr() + 1023) // 1024 * 1024
        ws_len = ws.numel() - (ws_ptr - ws.data_ptr())
    check("gdn_prefill_segmented_launch", LIB.gdn_prefill_segmented_launch(
        q.data_ptr(), k.data_ptr(), v.data_ptr(),
        state_in.data_ptr() if state_in is not None else None, A_log.data_ptr(), a.data_ptr(),
        dt_bias.data_ptr(), b.data_ptr(), sc, out.data_ptr(), ns.data_ptr(), T, HQ, HK, HV, D,
        int(bool(use_qk_l2norm)), segments, cb, qs, ks, vs, as_, bs, ws_ptr or None, ws_len,
        C.stream_handle(dev)))
    if out is not output:
        output.copy_(out)
    if ns is not new_state:
        new_state.copy_(ns)
    return output, new_state


def kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state):
    """flashinfer-bench DPS entry point (12 parameters, no normalisation)."""
    return gdn_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                       new_state)


def chunk_gated_delta_rule(q, k, v, g=None, beta=None, scale=None, initial_state=None,
                           output_final_state: bool = False, cu_seqlens=None,
                           use_qk_l2norm_in_kernel: bool = False, output=None, output_state=None,
                           state_checkpoints=None, checkpoint_cu_starts=None,
                           checkpoint_every_n_tokens: int = 0, *, kernel: str = "auto"):
    """Prefill with precomputed gates and optional state checkpoints, in the argument
    order and meaning of FlashInfer's ``chunk_gated_delta_rule``
    (flashinfer/gdn_prefill.py:99-185).

    ``g`` is the decay itself (alpha in [0, 1]) and ``beta`` the update gate, both fp32
    [T, num_v_heads]; None means all ones.  ``cu_seqlens`` (int32 or int64) None means one
    sequence of all T tokens.  With ``checkpoint_every_n_tokens`` = N > 0 (a multiple of
    64) the state after every N tokens of sequence i is written to
    ``state_checkpoints[checkpoint_cu_starts[i] + j]`` (``checkpoint_cu_starts`` int64
    [num_seqs + 1], the prefix sums of len_i // N).  Returns ``output`` or
    ``(output, final_state)`` when ``output_final_state``.
    """
    if kernel not in KERNELS:
        raise ValueError(f"kernel must be one of {sorted(KERNELS)}, got {kernel!r}")
    dev = C.cuda_device(q)
    C.tensor("q", q, torch.bfloat16, 3, dev)
    C.tensor("k", k, torch.bfloat16, 3, dev)
    C.tensor("v", v, torch.bfloat16, 3, dev)
    T, HQ, D = q.shape
    HK, HV = k.shape[1], v.shape[1]
    C.heads(HQ, HK, HV, D)
    C.shape("k", k, (T, HK, D))
    C.shape("v", v, (T, HV, D))
    for name, x in (("g", g), ("beta", beta)):
        if x is not None:
            C.tensor(name, x, torch.float32, 2, dev)
            C.shape(name, x, (T, HV))
    if cu_seqlens is None:
        cu_seqlens = torch.tensor([0, T], dtype=torch.int64, device=dev)
    if not isinstance(cu_seqlens, torch.Tensor) or cu_seqlens.dtype not in (torch.int32,
                                                                             torch.int64):
        raise TypeError("cu_seqlens must be an int32 or int64 tensor")
    if cu_seqlens.dim() != 1 or cu_seqlens.device != dev or not cu_seqlens.is_contiguous():
        raise ValueError("cu_seqlens must be a contiguous 1-D tensor on the same device as q")
    N = cu_seqlens.numel() - 1
    if initial_state is not None:
        C.tensor("initial_state", initial_state, torch.float32, 4, dev)
        C.shape("initial_state", initial_state, (N, HV, D, D))
    sc = C.scale_arg(scale)
    if output is None:
        output = torch.empty(T, HV, D, dtype=torch.bfloat16, device=dev)
    else:
        C.tensor("output", output, torch.bfloat16, 3, dev)
        C.shape("output", output, (T, HV, D))
    if output_state is None:
        output_state = torch.empty(max(N, 0), HV, D, D, dtype=torch.float32, device=dev)
    else:
        C.tensor("output_state", output_state, torch.float32, 4, dev)
        C.shape("output_state", output_state, (N, HV, D, D))
    every = int(checkpoint_every_n_tokens)
    cap = 0
    if every < 0 or (every > 0 and every % 64 != 0):
        raise ValueError("checkpoint_every_n_tokens must be 0 or a positive multiple of 64")
    if every > 0:
        if state_checkpoints is None or checkpoint_cu_starts is None:
            raise ValueError("checkpoints need state_checkpoints and checkpoint_cu_starts")
        C.tensor("state_checkpoints", state_checkpoints, torch.float32, 4, dev)
        if tuple(state_checkpoints.shape[1:]) != (HV, D, D):
            raise ValueError(f"state_checkpoints must be [n, {HV}, {D}, {D}]")
        C.tensor("checkpoint_cu_starts", checkpoint_cu_starts, torch.int64, 1, dev)
        C.shape("checkpoint_cu_starts", checkpoint_cu_starts, (N + 1,))
        cap = state_checkpoints.shape[0]
    if N > 0:
        ws_n = int(LIB.gdn_prefill_workspace_size_ext(KERNELS[kernel], T, N, HQ, HV, D,
                                                      int(bool(use_qk_l2norm_in_kernel)), 1,
                                                      every))
        ws = _workspace(dev, ws_n) if ws_n > 0 else None
        status = LIB.gdn_prefill_launch_ext(
            KERNELS[kernel], q.data_ptr(), k.data_ptr(), v.data_ptr(),
            initial_state.data_ptr() if initial_state is not None else None, 1,
            None, None, None, None,
            g.data_ptr() if g is not None else None, beta.data_ptr() if beta is not None else None,
            cu_seqlens.data_ptr(), int(cu_seqlens.dtype == torch.int64), sc, output.data_ptr(),
            output_state.data_ptr(),
            state_checkpoints.data_ptr() if every > 0 else None,
            checkpoint_cu_starts.data_ptr() if every > 0 else None, cap, every,
            T, N, HQ, HK, HV, D, int(bool(use_qk_l2norm_in_kernel)),
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            C.stream_handle(dev))
        check(f"gdn_prefill_launch_ext({kernel})", status)
    return (output, output_state) if output_final_state else output
