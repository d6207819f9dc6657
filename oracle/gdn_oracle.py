"""CPU oracle for the Gated DeltaNet (GDN) decode and prefill hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or the timed CPU baseline.  The product path
(the CUDA library behind ``kernel(...)``) never calls into it.

What it restates
----------------
The algorithm is the flashinfer-bench *definition reference* that the
reference repository is scored against, i.e. third-party code that is not in
the reference tree:

* package ``flashinfer-python`` (pinned ``0.6.4`` in the reference's
  ``requirements.txt:29``; ``0.6.11.post2`` installed here), file
  ``flashinfer/trace/templates/gdn.py``:
  ``_gdn_decode_reference`` (lines 27-94) and ``_gdn_prefill_reference``
  (lines 189-273).

The reference repository's own Triton kernels compute the same recurrence:
``gdn_decode/solution/triton/kernel.py:122-170`` (gates, S.k readout, rank-1
delta update, output) and ``gdn_prefill/solution/triton/kernel.py:60-79``
(the chunked restatement of the same recurrence).

This file restates the per-token recurrence from the mathematics in fp32
torch on the CPU, vectorised over (batch, v-head) instead of the definition's
Python loops over them:

    g    = exp(-exp(A_log) * softplus(a + dt_bias))          # gdn.py:51-52
    beta = sigmoid(b)                                        # gdn.py:53
    H    = S^T            (state is stored k-last: S[v, k])  # gdn.py:76-78
    H'   = g * H
    old  = k^T H'                                            # [V]
    H    = H' + k (beta * (v - old))^T                       # gdn.py:82-87
    o    = scale * q^T H  -> bf16                            # gdn.py:89

GVA: v-head ``h`` reads q/k head ``h // (HV // HQ)`` (``repeat_interleave``,
gdn.py:67-68).  ``scale`` of 0 or None means 1/sqrt(head_size)
(gdn.py:47-48).  ``state=None`` means a zero initial state (gdn.py:61-64,
237-246).  In prefill an empty sequence is skipped, which leaves its
``new_state`` slice at ZERO (gdn.py:224-226 allocate zeros; 231-232
``continue``).  The prefill output has ``max(HQ, HV)`` heads (gdn.py:218-221).

Parity is pinned by ``tests/golden/`` fixtures that were produced by running
the definition reference itself (and, for decode, the reference repository's
own Triton kernel under the Triton CPU interpreter); see
``tests/golden/make_golden.py``.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

__all__ = [
    "gates",
    "l2norm",
    "decode",
    "prefill",
    "flashinfer_allclose",
    "state_rel_err",
]

L2NORM_EPS = 1e-6


def gates(A_log: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor,
          b: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """g = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b), fp32.

    Follows ``flashinfer/trace/templates/gdn.py:51-53`` (decode) and
    ``:211-213`` (prefill); softplus is torch's (threshold 20, identical to the
    reference kernel's ``x > 20 -> x`` cut-off at
    ``gdn_decode/solution/triton/kernel.py:129``).
    """
    x = a.float() + dt_bias.float()
    g = torch.exp(-torch.exp(A_log.float()) * F.softplus(x))
    beta = torch.sigmoid(b.float())
    return g, beta


def l2norm(x: torch.Tensor, eps: float = L2NORM_EPS) -> torch.Tensor:
    """fp32 L2 normalisation over the last (head_dim) axis: x * rsqrt(sum x^2 + eps).

    This is the host-side form of the kernels' ``use_qk_l2norm`` option; the
    oracle is fed its result when that option is on (the definition reference
    itself never normalises, gdn.py:51-91).
    """
    xf = x.float()
    return xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)


def _default_scale(scale: Optional[float], head_size: int) -> float:
    if scale is None or scale == 0.0:
        return 1.0 / math.sqrt(head_size)
    return float(scale)


@torch.no_grad()
def decode(q, k, v, state, A_log, a, dt_bias, b, scale, *, dtype=torch.float32):
    """One decode step.  Shapes as ``flashinfer/trace/templates/gdn.py:125-176``.

    q [B,1,HQ,D], k [B,1,HK,D], v [B,1,HV,D] (bf16 or fp32), state [B,HV,D,D]
    fp32 k-last or None, A_log [HV], a [B,1,HV], dt_bias [HV], b [B,1,HV].
    Returns (output [B,1,HV,D] bf16, new_state [B,HV,D,D] fp32).

    ``dtype=torch.float64`` runs the same recurrence in double precision (used by
    tests to bound the fp32 rounding of this oracle itself).
    """
    B, T, HQ, D = q.shape
    HK = k.shape[2]
    HV = v.shape[2]
    if T != 1:
        raise ValueError("decode oracle expects seq_len == 1")
    sc = _default_scale(scale, D)
    g, beta = gates(A_log, a, dt_bias, b)                      # [B,1,HV]
    g = g[:, 0].to(dtype)                                      # [B,HV]
    beta = beta[:, 0].to(dtype)
    qe = q[:, 0].to(dtype).repeat_interleave(HV // HQ, dim=1)  # [B,HV,D]
    ke = k[:, 0].to(dtype).repeat_interleave(HV // HK, dim=1)
    ve = v[:, 0].to(dtype)                                     # [B,HV,D]
    if state is None:
        S = torch.zeros(B, HV, D, D, dtype=dtype)
    else:
        S = state.to(dtype)
    Sg = g[..., None, None] * S                                # g * S   [B,HV,V,K]
    old = torch.einsum("bhvk,bhk->bhv", Sg, ke)                # (gS) k
    delta = beta[..., None] * (ve - old)                       # beta (v - old)
    S_new = Sg + delta[..., :, None] * ke[..., None, :]        # + delta k^T  (k-last)
    out = sc * torch.einsum("bhvk,bhk->bhv", S_new, qe)
    # a bf16 state (the bf16-state storage format) is widened above and the new state
    # rounded to nearest bf16 for storage; the output uses the unrounded state
    sdt = torch.bfloat16 if (state is not None and state.dtype == torch.bfloat16) else torch.float32
    return out[:, None].to(torch.bfloat16), S_new.to(sdt)


@torch.no_grad()
def mtp(q, k, v, initial_state, state_indices, A_log, a, dt_bias, b, scale, *,
        intermediate=False, dtype=torch.float32):
    """Multi-token decode (speculative-decoding verification): the recurrence of
    ``_gdn_mtp_reference`` (``flashinfer/trace/templates/gdn.py:379-466``), shapes as
    ``gdn.py:469-560``, one decode step per token (:func:`decode`), batched over rows.

    q/k [B,T,HQ,D], v [B,T,HV,D], initial_state [P,HV,D,D] fp32 k-last pool,
    state_indices [B] int (pool slot of each row), A_log/dt_bias [HV], a/b [B,T,HV].
    Returns (output [B,T,HV,D] bf16, final_state [P,HV,D,D] fp32 = the pool with the
    rows' slots replaced by their state after T tokens, intermediate [P,T,HV,D,D] fp32
    with the state after every token in the rows' slots (zeros elsewhere) or None).

    Every row starts from the initial pool, as in the definition.  A row whose index
    lies outside [0, P) is padding: zero output and no state change (the definition
    would index the pool with Python's negative-index wrap; the kernels skip such rows).
    A bf16 pool (the bf16-state storage format) is widened on load, carried in fp32
    through the T tokens and rounded to nearest bf16 in final_state and intermediate.
    """
    B, T = q.shape[:2]
    HV, D = v.shape[2], v.shape[3]
    P = initial_state.shape[0]
    sdt = initial_state.dtype if initial_state.dtype == torch.bfloat16 else torch.float32
    final = initial_state.clone().to(sdt)
    inter = torch.zeros((P, T) + tuple(initial_state.shape[1:]), dtype=sdt) \
        if intermediate else None
    out = torch.zeros(B, T, HV, D, dtype=torch.bfloat16)
    idx = [int(i) for i in state_indices.tolist()]
    rows = [r for r in range(B) if 0 <= idx[r] < P]
    if not rows or T == 0:
        return out, final, inter
    sel = torch.tensor(rows, dtype=torch.long)
    slots = torch.tensor([idx[r] for r in rows], dtype=torch.long)
    S = initial_state[slots].float()
    for t in range(T):
        o, S = decode(q[sel, t:t + 1], k[sel, t:t + 1], v[sel, t:t + 1], S, A_log,
                      a[sel, t:t + 1], dt_bias, b[sel, t:t + 1], scale, dtype=dtype)
        out[sel, t] = o[:, 0]
        if inter is not None:
            inter[slots, t] = S.to(sdt)
    final[slots] = S.to(sdt)
    return out, final, inter


@torch.no_grad()
def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, *,
            dtype=torch.float32):
    """Variable-length prefill.  Shapes as ``gdn.py:303-363``.

    q [T,HQ,D], k [T,HK,D], v [T,HV,D], state [N,HV,D,D] fp32 or None,
    A_log/dt_bias [HV], a/b [T,HV], cu_seqlens [N+1] (int32 or int64).
    Returns (output [T, max(HQ,HV), D] bf16, new_state [N, max(HQ,HV), D, D] fp32).

    Token loop per sequence, vectorised over heads (``gdn.py:228-271``).
    """
    g, beta = gates(A_log, a, dt_bias, b)                      # [T,HV]
    out, new_state, _ = _prefill_core(q, k, v, state, g, beta, cu_seqlens, scale, dtype, 0)
    return out, new_state


@torch.no_grad()
def prefill_gated(q, k, v, state, alpha, beta, cu_seqlens, scale, *, checkpoint_every=0,
                  dtype=torch.float32):
    """Prefill with precomputed per-token gates and optional state checkpoints, the
    contract of FlashInfer's ``chunk_gated_delta_rule`` (``flashinfer/gdn_prefill.py:99-185``):
    alpha = the decay g itself and beta, fp32 [T, HV] (None = all ones); with
    ``checkpoint_every`` = N > 0 the state after every N tokens of each sequence is
    returned, ``len // N`` per sequence in sequence order.

    Same recurrence as :func:`prefill` with g, beta given instead of computed.
    Returns (output, new_state, checkpoints [sum(len // N), HV, D, D] fp32 or None).
    """
    T, HV = q.shape[0], v.shape[1]
    g = alpha.float() if alpha is not None else torch.ones(T, HV)
    bt = beta.float() if beta is not None else torch.ones(T, HV)
    return _prefill_core(q, k, v, state, g, bt, cu_seqlens, scale, dtype, checkpoint_every)


def _prefill_core(q, k, v, state, g, beta, cu_seqlens, scale, dtype, checkpoint_every):
    """Token loop per sequence, vectorised over heads (``gdn.py:228-271``)."""
    T, HQ, D = q.shape
    HK = k.shape[1]
    HV = v.shape[1]
    H = max(HQ, HV)
    N = int(cu_seqlens.numel()) - 1
    sc = _default_scale(scale, D)
    g = g.to(dtype)
    beta = beta.to(dtype)
    qe = q.to(dtype).repeat_interleave(HV // HQ, dim=1)        # [T,HV,D]
    ke = k.to(dtype).repeat_interleave(HV // HK, dim=1)
    ve = v.to(dtype)
    out = torch.zeros(T, H, D, dtype=torch.bfloat16)
    new_state = torch.zeros(N, H, D, D, dtype=torch.float32)
    ckpts = []
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(N):
        s0, s1 = cu[n], cu[n + 1]
        if s1 - s0 <= 0:
            continue                                            # gdn.py:231-232
        if state is not None:
            S = state[n].to(dtype).clone()                      # [HV,V,K]
        else:
            S = torch.zeros(HV, D, D, dtype=dtype)
        for t in range(s0, s1):
            S.mul_(g[t][:, None, None])
            old = torch.einsum("hvk,hk->hv", S, ke[t])
            delta = beta[t][:, None] * (ve[t] - old)
            S.add_(delta[:, :, None] * ke[t][:, None, :])
            out[t, :HV] = (sc * torch.einsum("hvk,hk->hv", S, qe[t])).to(torch.bfloat16)
            if checkpoint_every > 0 and (t - s0 + 1) % checkpoint_every == 0:
                ckpts.append(S.float().clone())
        new_state[n, :HV] = S.float()
    ck = None
    if checkpoint_every > 0:
        ck = torch.stack(ckpts) if ckpts else torch.zeros(0, HV, D, D)
    return out, new_state, ck


def flashinfer_allclose(actual: torch.Tensor, expected: torch.Tensor,
                        atol: float, rtol: float) -> Tuple[bool, float, float, float]:
    """flashinfer-bench element test: an element FAILS iff |d| > atol AND |d|/|ref| > rtol.

    Returns (all_match, matched_fraction, max_abs_err, max_rel_err).  This is the
    reference harness's rule (reference ``FAQ.md:104-110``: atol, rtol and a
    required matched ratio of 1.0).
    """
    a = actual.float()
    e = expected.float()
    d = (a - e).abs()
    rel = d / e.abs().clamp_min(1e-30)
    bad = (d > atol) & (rel > rtol)
    frac = 1.0 - bad.float().mean().item() if d.numel() else 1.0
    max_abs = d.max().item() if d.numel() else 0.0
    max_rel = rel[e != 0].max().item() if (e != 0).any() else 0.0
    return (not bool(bad.any())), frac, max_abs, max_rel


def state_rel_err(actual: torch.Tensor, expected: torch.Tensor) -> float:
    """Norm-wise relative error ||A - E||_F / ||E||_F (0 when both are zero)."""
    a = actual.double()
    e = expected.double()
    den = e.norm().item()
    num = (a - e).norm().item()
    if den == 0.0:
        return num
    return num / den
