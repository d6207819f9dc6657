"""Multi-GPU partitioning of the GDN workloads (one process per GPU).

Every unit of GDN work is independent of every other one:

* decode: each (batch row, v-head) state is updated from that row's own q/k/v,
  so a batch splits into contiguous row ranges, one per rank;
* prefill: each sequence's scan touches only its own tokens and state slice,
  so whole sequences are dealt to ranks; the packed token ranges of a rank's
  sequences are gathered into a rank-local packed layout with re-based
  ``cu_seqlens`` (0, len0, len0+len1, ...);
* prefill with fewer sequences than ranks (one long sequence): each v-head's
  scan reads only its own q/k head (v-head h uses q/k head h // (HV/HQ)), so
  q/k-head groups are dealt to ranks together with the v-heads that use them.

Load balance for prefill uses longest-processing-time bin packing on token
counts.  There is no exchange step on the data path, so there is no NCCL
call in the timed region; results are gathered (to the host, outside timing)
only for verification.

One long sequence can also be split into consecutive token segments, one per rank, with a
segment-level scan of its affine state map (``segment_scan_rank``, end of this file): that
has one real exchange step, an all-gather of each segment's (A, B) state map.
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import torch


def batch_range(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) row range of `rank` when `batch` rows are split over `world`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def lpt_assign(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Longest-first greedy bin packing: sequence indices per rank (each sorted).

    Every index appears in exactly one bin; ties go to the lowest rank, so the
    plan is deterministic.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    bins: List[List[int]] = [[] for _ in range(world)]
    load = [0] * world
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        j = min(range(world), key=lambda r: (load[r], r))
        bins[j].append(i)
        load[j] += int(lengths[i])
    return [sorted(b) for b in bins]


def seqlens_from_cu(cu_seqlens: torch.Tensor) -> List[int]:
    cu = [int(x) for x in cu_seqlens.tolist()]
    return [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]


def prefill_shard(inp: Dict[str, torch.Tensor], seq_ids: Sequence[int]) -> Dict[str, torch.Tensor]:
    """The rank-local prefill problem for sequences `seq_ids` (host or device tensors).

    Token-indexed tensors (q, k, v, a, b) are gathered, the initial state (if
    any) is sliced, and cu_seqlens is re-based.  Per-head parameters and
    scale are shared.
    """
    cu = [int(x) for x in inp["cu_seqlens"].tolist()]
    dev = inp["q"].device
    idx = [torch.arange(cu[i], cu[i + 1], device=dev) for i in seq_ids]
    take = torch.cat(idx) if idx else torch.zeros(0, dtype=torch.long, device=dev)
    out = dict(inp)
    for key in ("q", "k", "v", "a", "b"):
        out[key] = inp[key].index_select(0, take).contiguous()
    if inp.get("state") is not None:
        sel = torch.tensor(list(seq_ids), dtype=torch.long, device=inp["state"].device)
        out["state"] = inp["state"].index_select(0, sel).contiguous()
    lens = [cu[i + 1] - cu[i] for i in seq_ids]
    c = torch.zeros(len(lens) + 1, dtype=inp["cu_seqlens"].dtype)
    if lens:
        c[1:] = torch.tensor(lens, dtype=torch.int64).cumsum(0).to(c.dtype)
    out["cu_seqlens"] = c.to(inp["cu_seqlens"].device)
    return out


def prefill_unshard(full_tokens: int, num_seqs: int, cu_seqlens: torch.Tensor,
                    plan: Sequence[Sequence[int]],
                    outputs: Sequence[torch.Tensor], states: Sequence[torch.Tensor]
                    ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Reassemble per-rank (output, new_state) into the unsharded layout."""
    cu = [int(x) for x in cu_seqlens.tolist()]
    o0, s0 = outputs[0], states[0]
    out = torch.zeros((full_tokens,) + tuple(o0.shape[1:]), dtype=o0.dtype)
    st = torch.zeros((num_seqs,) + tuple(s0.shape[1:]), dtype=s0.dtype)
    for ids, o, s in zip(plan, outputs, states):
        pos = 0
        for j, i in enumerate(ids):
            n = cu[i + 1] - cu[i]
            out[cu[i]:cu[i + 1]] = o[pos:pos + n].cpu()
            st[i] = s[j].cpu()
            pos += n
    return out, st


def head_range(num_qk_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) range of q/k heads of `rank` (head-group sharding)."""
    return batch_range(num_qk_heads, world, rank)


def prefill_head_shard(inp: Dict[str, torch.Tensor], qk_lo: int, qk_hi: int
                       ) -> Dict[str, torch.Tensor]:
    """The rank-local prefill problem for q/k heads [qk_lo, qk_hi) and their v-heads.

    All sequences and tokens stay; q and k keep heads [qk_lo, qk_hi), and v, a,
    b, A_log, dt_bias and the initial state keep the v-heads
    [qk_lo * r, qk_hi * r) with r = HV / HQ, each copied into a contiguous
    tensor.  cu_seqlens and scale are shared.
    """
    HQ, HV = inp["q"].shape[1], inp["v"].shape[1]
    if HQ <= 0 or HV % HQ != 0:
        raise ValueError(f"head-group sharding needs HV ({HV}) to be a multiple of HQ ({HQ})")
    if not 0 <= qk_lo < qk_hi <= HQ:
        raise ValueError(f"bad q/k head range [{qk_lo}, {qk_hi}) for {HQ} heads")
    r = HV // HQ
    v_lo, v_hi = qk_lo * r, qk_hi * r
    out = dict(inp)
    for key in ("q", "k"):
        out[key] = inp[key][:, qk_lo:qk_hi].contiguous()
    for key in ("v", "a", "b"):
        out[key] = inp[key][:, v_lo:v_hi].contiguous()
    for key in ("A_log", "dt_bias"):
        out[key] = inp[key][v_lo:v_hi].contiguous()
    if inp.get("state") is not None:
        out["state"] = inp["state"][:, v_lo:v_hi].contiguous()
    return out


def prefill_head_unshard(outputs: Sequence[torch.Tensor], states: Sequence[torch.Tensor]
                         ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Reassemble per-rank (output, new_state) of consecutive head ranges (rank order)."""
    out = torch.cat([o.cpu() for o in outputs], dim=1)
    st = torch.cat([s.cpu() for s in states], dim=1)
    return out, st


# --------------------------------------------------------------------------------------
# One long sequence over several ranks: a segment-level scan of the state map.
#
# Over a segment of tokens the recurrence is affine in the state: with the k-last state
# S[v, k], every token applies S <- S g (I - beta k k^T) + beta v k^T, so a segment maps
# S_in to S_out = S_in A + B, where A (k x k) is what the segment makes of the identity
# when v = 0 (row v of the identity evolves like state row v) and B is the segment's final
# state from a zero state.  The outputs are affine in S_in too: o_t = scale S_t q_t =
# S_in o^I_t + o^0_t, with o^I_t the output of the identity run (v = 0) and o^0_t that of
# the run from zero.  Rank r takes segment r: rank 0 runs its segment from the caller's
# initial state (its outputs and final state are final); every other rank runs its
# segment from the identity with v = 0 and from a zero state (one call of two sequences),
# the (A, B) of all ranks are exchanged (the one collective), each rank chains
# S_start(r) = S_start(r-1) A_{r-1} + B_{r-1}, with (A_0, B_0) = (0, rank 0's final state),
# and assembles its outputs S_start(r) o^I_t + o^0_t and final state S_start(r) A_r + B_r
# with fp32 matrix products.  The serial chain shrinks from the whole sequence to the
# first segment; the price is two runs of each other segment, on ranks whose SMs would
# otherwise sit idle.
# `run(segment_inputs, state, zero_v)` is the prefill call (it returns (output,
# final_state)); states are [1, HV, 128, 128] fp32.


def segment_bounds(total_tokens: int, world: int, align: int = 64,
                   first_weight: int = 2) -> List[Tuple[int, int]]:
    """[start, end) token ranges of `world` consecutive segments of one sequence, the
    boundaries on multiples of `align` (the prefill chunk) and the last one ending at the
    sequence's end; a segment may be empty when the sequence is short.  The first segment
    gets `first_weight` shares and every other one share: its rank runs it once, while the
    others run their segment twice (from the identity with v = 0 and from zero; as one call
    of two sequences that is two waves of the state kernel), all before the exchange."""
    if world <= 0:
        raise ValueError("world must be positive")
    chunks = (total_tokens + align - 1) // align
    shares = [first_weight] + [1] * (world - 1)
    total_share, cum = sum(shares), 0
    bounds, start = [], 0
    for r in range(world):
        cum += shares[r]
        end = min((chunks * cum // total_share) * align, total_tokens)
        if r == world - 1:
            end = total_tokens
        bounds.append((start, end))
        start = end
    return bounds


def segment_inputs(inp: Dict[str, torch.Tensor], lo: int, hi: int) -> Dict[str, torch.Tensor]:
    """Tokens [lo, hi) of a single-sequence prefill problem as a one-sequence problem."""
    out = dict(inp)
    for key in ("q", "k", "v", "a", "b"):
        out[key] = inp[key][lo:hi].contiguous()
    out["cu_seqlens"] = torch.tensor([0, hi - lo], dtype=inp["cu_seqlens"].dtype,
                                     device=inp["cu_seqlens"].device)
    return out


def segment_map(run, seg: Dict[str, torch.Tensor]
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(A, B, o^I, o^0) of one segment: A and o^I from the identity with v = 0, B and o^0
    from a zero state (an empty segment is the identity map with no outputs: the prefill
    call would return a zero state)."""
    HV = seg["v"].shape[1]
    dev = seg["v"].device
    eye = torch.eye(128, dtype=torch.float32, device=dev).expand(1, HV, 128, 128).contiguous()
    zero = torch.zeros(1, HV, 128, 128, dtype=torch.float32, device=dev)
    if seg["q"].shape[0] == 0:
        none = torch.empty((0, HV, 128), dtype=torch.bfloat16, device=dev)
        return eye, zero, none, none
    o_id, A = run(seg, eye, True)
    o_zero, B = run(seg, zero, False)
    return A, B, o_id, o_zero


def segment_finish(start: torch.Tensor, A: torch.Tensor, B: torch.Tensor, o_id: torch.Tensor,
                   o_zero: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """A segment's outputs and final state from its start state [1, HV, 128, 128] and its
    map: o_t[h, v] = sum_j start[h, v, j] o^I_t[h, j] + o^0_t[h, v] (bf16, summed in fp32)
    and start A + B (fp32).  On the GPU the outputs come from one kernel of the library
    (gdn_segment_outputs_launch: start split into bf16 hi + lo, bf16 tensor-core products
    with fp32 sums, o^0 added before the bf16 rounding)."""
    fin = torch.baddbmm(B[0], start[0], A[0]).unsqueeze(0)
    if o_id.is_cuda:
        from ._checks import stream_handle
        from ._lib import LIB, check
        out = torch.empty_like(o_zero)
        st = start[0].contiguous()
        o_id, o_zero = o_id.contiguous(), o_zero.contiguous()
        check("gdn_segment_outputs_launch", LIB.gdn_segment_outputs_launch(
            o_id.data_ptr(), o_zero.data_ptr(), st.data_ptr(), out.data_ptr(),
            o_id.shape[0], o_id.shape[1], o_id.shape[2], stream_handle(o_id.device)))
        return out, fin
    out = torch.einsum("thj,hvj->thv", o_id.float(), start[0]) + o_zero.float()
    return out.to(torch.bfloat16), fin


def _run_from(run, seg: Dict[str, torch.Tensor], state: torch.Tensor
              ) -> Tuple[torch.Tensor, torch.Tensor]:
    """A segment's run from `state`; an empty segment leaves the state as it is."""
    if seg["q"].shape[0] == 0:
        out = torch.empty((0,) + tuple(seg["v"].shape[1:]), dtype=torch.bfloat16,
                          device=seg["v"].device)
        return out, state
    return run(seg, state, False)


def chain_start(As: Sequence[torch.Tensor], Bs: Sequence[torch.Tensor], r: int) -> torch.Tensor:
    """S_start(r) = S_start(r-1) A_{r-1} + B_{r-1} from S_start(1) = B_0 (r >= 1), in fp32."""
    S = Bs[0][0]
    for m in range(1, r):
        S = torch.baddbmm(Bs[m][0], S, As[m][0])
    return S.unsqueeze(0)


def segment_assemble(maps: torch.Tensor, rank: int, o_id: torch.Tensor, o_zero: torch.Tensor,
                     out: torch.Tensor = None, final: torch.Tensor = None
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Segment `rank`'s (>= 1) outputs and final state from every segment's map, `maps`
    [world, 2, HV, 128, 128] (A then B; the first segment's entry is (unused, its final
    state)), and its two runs' outputs o^I, o^0.  On the GPU: two kernels of the library
    (gdn_segment_chain_launch: the chained start state and the final state in fp32;
    gdn_segment_outputs_launch: the outputs); on the CPU the same algebra in torch.
    `out` / `final` (contiguous, of the result's shape) receive the results when given."""
    if not maps.is_cuda:
        As, Bs = [m[0:1] for m in maps], [m[1:2] for m in maps]
        o, f = segment_finish(chain_start(As, Bs, rank), maps[rank, 0:1], maps[rank, 1:2],
                              o_id, o_zero)
        if out is not None:
            o = out.copy_(o)
        if final is not None:
            f = final.copy_(f)
        return o, f
    from ._checks import stream_handle
    from ._lib import LIB, check
    maps = maps.contiguous()
    W, _, HV, D, _ = maps.shape
    start = torch.empty(1, HV, D, D, dtype=torch.float32, device=maps.device)
    fin = final if final is not None else torch.empty_like(start)
    stream = stream_handle(maps.device)
    check("gdn_segment_chain_launch", LIB.gdn_segment_chain_launch(
        maps.data_ptr(), W, rank, start.data_ptr(), fin.data_ptr(), HV, D, stream))
    out = out if out is not None else torch.empty_like(o_zero)
    o_id, o_zero = o_id.contiguous(), o_zero.contiguous()
    check("gdn_segment_outputs_launch", LIB.gdn_segment_outputs_launch(
        o_id.data_ptr(), o_zero.data_ptr(), start.data_ptr(), out.data_ptr(),
        o_id.shape[0], HV, D, stream))
    return out, fin


def segment_scan_rank(run, inp: Dict[str, torch.Tensor], world: int, rank: int, all_gather
                      ) -> Tuple[torch.Tensor, torch.Tensor]:
    """This rank's part of the segment scan.  `all_gather(t)` returns the list of every
    rank's `t` (rank order).  Returns (output of this rank's tokens, final state after
    them); the last rank's final state is the sequence's."""
    T = inp["q"].shape[0]
    lo, hi = segment_bounds(T, world)[rank]
    seg = segment_inputs(inp, lo, hi)
    HV = inp["v"].shape[1]
    if rank == 0:
        state = inp.get("state")
        if state is None:
            state = torch.zeros(1, HV, 128, 128, dtype=torch.float32, device=inp["v"].device)
        out, fin = _run_from(run, seg, state)
        A, B = torch.zeros_like(fin), fin
    else:
        A, B, o_id, o_zero = segment_map(run, seg)
    parts = all_gather(torch.cat([A, B], dim=0).contiguous())
    if rank == 0:
        return out, fin
    return segment_assemble(torch.stack(list(parts)), rank, o_id, o_zero)


def segment_scan_local(run, inp: Dict[str, torch.Tensor], world: int
                       ) -> Tuple[torch.Tensor, torch.Tensor]:
    """The whole segment scan in one process (every rank's work in turn): the
    sequence's output and final state."""
    T = inp["q"].shape[0]
    parts = []
    maps = []
    for r, (lo, hi) in enumerate(segment_bounds(T, world)):
        seg = segment_inputs(inp, lo, hi)
        if r == 0:
            HV = inp["v"].shape[1]
            state = inp.get("state")
            if state is None:
                state = torch.zeros(1, HV, 128, 128, dtype=torch.float32, device=inp["v"].device)
            out, fin = _run_from(run, seg, state)
            maps.append((torch.zeros_like(fin), fin, None, None))
            parts.append(out)
        else:
            maps.append(segment_map(run, seg))
    stacked = torch.stack([torch.cat([m[0], m[1]], dim=0) for m in maps])
    for r in range(1, world):
        out, fin = segment_assemble(stacked, r, maps[r][2], maps[r][3])
        parts.append(out)
    return torch.cat(parts, dim=0), fin


# --------------------------------------------------------------------------------------
# The same scan inside ONE call, for a single sequence whose (v-head) work leaves most SMs
# idle (few heads per GPU, e.g. one sequence sharded by q/k-head group over 4 or 8 GPUs):
# the segments run side by side as the sequences of one prefill call (segment 0 from the
# initial state, every later segment twice: from the identity with v = 0 and from zero),
# and the maps are chained on the same GPU afterwards.  No collective: the serial chain
# falls from the whole sequence to one segment, paid for with twice the work on SMs that
# would otherwise be idle.


def segmented_layout(total_tokens: int, segments: int, device, bounds: List[int] = None
                     ) -> Tuple[List[Tuple[int, int]], torch.Tensor]:
    """For one sequence of `total_tokens` tokens in `segments` equal segments (on 64-token
    chunk boundaries), or at the token offsets `bounds` = [0, b_1, .., total_tokens] when
    given: (bounds, cu_seqlens int32 of the 2 S - 1 runs of one call).  Run 0 is segment
    0; runs 2 s - 1 and 2 s are segment s from the identity (v = 0) and from zero.
    `segments` is capped at the number of chunks, so that no segment is empty (an empty
    run would return a zero state, not the identity map)."""
    if bounds is None:
        segments = max(1, min(segments, (total_tokens + 63) // 64))
        bounds = segment_bounds(total_tokens, segments, first_weight=1)
    else:
        bounds = [(int(bounds[i]), int(bounds[i + 1])) for i in range(len(bounds) - 1)]
    cu = [0]
    for s, (lo, hi) in enumerate(bounds):
        for _ in range(1 if s == 0 else 2):
            cu.append(cu[-1] + hi - lo)
    return bounds, torch.tensor(cu, dtype=torch.int32, device=device)


def segmented_inputs(inp: Dict[str, torch.Tensor], layout, template: torch.Tensor = None
                     ) -> Dict[str, torch.Tensor]:
    """The one-call problem of `layout` (segmented_layout) built from a one-sequence
    problem: q, k, a, b of every run, v of every run with zeros for the identity runs, and
    the initial states [state or 0; I; 0; I; 0; ...] -- one concatenation per tensor.
    `template` may hold the constant part [0; I; 0; I; 0; ...] (2 S - 1 states; its first
    entry is overwritten by nothing and only used when there is no initial state)."""
    bounds, cu = layout
    HV = inp["v"].shape[1]
    dev = inp["v"].device
    runs = [(lo, hi, s > 0 and r == 0) for s, (lo, hi) in enumerate(bounds)
            for r in range(1 if s == 0 else 2)]
    out = dict(inp)
    for key in ("q", "k", "a", "b"):
        x = inp[key]
        out[key] = torch.cat([x[lo:hi] for lo, hi, _ in runs])
    v = inp["v"]
    longest = max(hi - lo for lo, hi in bounds)
    zero_v = v.new_zeros((longest,) + tuple(v.shape[1:]))
    out["v"] = torch.cat([zero_v[:hi - lo] if ident else v[lo:hi] for lo, hi, ident in runs])
    if template is None:
        template = state_template(len(bounds), HV, dev)
    if inp.get("state") is None:
        out["state"] = template
    else:
        out["state"] = torch.cat([inp["state"][0:1], template[1:]])
    out["cu_seqlens"] = cu
    return out


def state_template(segments: int, num_v_heads: int, device) -> torch.Tensor:
    """Initial states [0; I; 0; I; 0; ...] of the 2 S - 1 runs of a segmented call."""
    t = torch.zeros(2 * segments - 1, num_v_heads, 128, 128, dtype=torch.float32,
                    device=device)
    t[1::2] = torch.eye(128, dtype=torch.float32, device=device)
    return t


def segmented_finish(layout, out_runs: torch.Tensor, fin_runs: torch.Tensor,
                     output: torch.Tensor = None, final: torch.Tensor = None,
                     maps: torch.Tensor = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """The sequence's output [T, HV, 128] and final state [1, HV, 128, 128] from the one
    call's outputs and final states: segment 0's as they are, every later segment's from
    its chained start state.  On the GPU: one pass of the library's chain kernel for every
    start state (gdn_segment_chain_all_launch) and its output kernel per segment; on the
    CPU the same algebra in torch.  `maps` may be the [S, 2, HV, 128, 128] tensor whose
    flattened entries 1 .. 2 S - 1 are fin_runs (the call wrote its final states there):
    then the maps need no copy."""
    bounds = layout[0]
    n = len(bounds)
    starts = [0]
    for s, (lo, hi) in enumerate(bounds):
        for _ in range(1 if s == 0 else 2):
            starts.append(starts[-1] + hi - lo)
    T = bounds[-1][1]
    HV = out_runs.shape[1]
    if output is None:
        output = torch.empty((T,) + tuple(out_runs.shape[1:]), dtype=out_runs.dtype,
                             device=out_runs.device)
    lo0, hi0 = bounds[0]
    output[lo0:hi0].copy_(out_runs[starts[0]:starts[1]])
    if n == 1:
        fin = fin_runs[0:1]
        return output, (final.copy_(fin) if final is not None else fin)
    if maps is None:
        maps = torch.empty((n, 2) + tuple(fin_runs.shape[1:]), dtype=torch.float32,
                           device=fin_runs.device)
        maps.view(2 * n, *fin_runs.shape[1:])[1:].copy_(fin_runs)
    runs = [(out_runs[starts[2 * s - 1]:starts[2 * s]], out_runs[starts[2 * s]:starts[2 * s + 1]])
            for s in range(1, n)]
    if not maps.is_cuda:
        maps = maps.clone()
        maps[0, 0].zero_()
        fin = None
        for s in range(1, n):
            lo, hi = bounds[s]
            _, fin = segment_assemble(maps, s, runs[s - 1][0], runs[s - 1][1],
                                      out=output[lo:hi])
        return output, (final.copy_(fin) if final is not None else fin)
    from ._checks import stream_handle
    from ._lib import LIB, check
    stream = stream_handle(maps.device)
    st = torch.empty((n - 1, HV, 128, 128), dtype=torch.float32, device=maps.device)
    fin = final if final is not None else torch.empty(1, HV, 128, 128, dtype=torch.float32,
                                                      device=maps.device)
    check("gdn_segment_chain_all_launch", LIB.gdn_segment_chain_all_launch(
        maps.data_ptr(), n, st.data_ptr(), fin.data_ptr(), HV, 128, stream))
    for s in range(1, n):
        lo, hi = bounds[s]
        o_id, o_zero = runs[s - 1]
        check("gdn_segment_outputs_launch", LIB.gdn_segment_outputs_launch(
            o_id.data_ptr(), o_zero.data_ptr(), st[s - 1].data_ptr(), output[lo:hi].data_ptr(),
            hi - lo, HV, 128, stream))
    return output, fin
