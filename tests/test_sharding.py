"""CPU: multi-GPU partitioning plans (batch ranges, longest-first sequence packing)
and the shard -> unshard round trip, checked with the oracle on small problems."""
import pytest
import torch

from conftest import load_pkg
from oracle import gdn_oracle as O


def test_batch_ranges_cover_exactly():
    S = load_pkg().sharding
    for batch in (0, 1, 7, 128, 1024):
        for world in (1, 2, 3, 8):
            rs = [S.batch_range(batch, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [hi - lo for lo, hi in rs]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        S.batch_range(4, 2, 2)


def test_lpt_assign_partition_and_balance():
    pkg = load_pkg()
    S, W = pkg.sharding, pkg.workloads
    cfg = W.PREFILL_CONFIGS["P3"]
    lens = W.draw_seqlens(cfg.n, cfg.lo, cfg.hi, 0)
    for world in (1, 2, 4, 8):
        plan = S.lpt_assign(lens, world)
        flat = sorted(i for b in plan for i in b)
        assert flat == list(range(len(lens)))
        loads = [sum(lens[i] for i in b) for b in plan]
        # LPT bound: max load <= mean + longest item
        assert max(loads) <= sum(lens) / world + max(lens)
    assert S.lpt_assign([5, 0, 9], 2) == S.lpt_assign([5, 0, 9], 2)  # deterministic


def test_prefill_shard_roundtrip_matches_unsharded_oracle():
    pkg = load_pkg()
    S, W = pkg.sharding, pkg.workloads
    lens = [5, 0, 9, 3, 12]
    inp = W.prefill_inputs(lens, hq=1, hv=2, seed=3)
    full_o, full_s = O.prefill(O.l2norm(inp["q"]), O.l2norm(inp["k"]), inp["v"], inp["state"],
                               inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                               inp["cu_seqlens"], inp["scale"])
    plan = S.lpt_assign(lens, 3)
    outs, states = [], []
    for ids in plan:
        sh = S.prefill_shard(inp, ids)
        assert int(sh["cu_seqlens"][-1]) == sh["q"].shape[0] == sum(lens[i] for i in ids)
        o, s = O.prefill(O.l2norm(sh["q"]), O.l2norm(sh["k"]), sh["v"], sh["state"],
                         sh["A_log"], sh["a"], sh["dt_bias"], sh["b"], sh["cu_seqlens"],
                         sh["scale"])
        outs.append(o)
        states.append(s)
    o, s = S.prefill_unshard(sum(lens), len(lens), inp["cu_seqlens"], plan, outs, states)
    assert torch.equal(o, full_o)
    # same recurrence per sequence; the batched einsum may only reorder fp32 sums
    assert O.state_rel_err(s, full_s) < 1e-6


def test_head_ranges_and_shard_roundtrip_matches_unsharded_oracle():
    pkg = load_pkg()
    S, W = pkg.sharding, pkg.workloads
    lens = [9, 0, 70]
    inp = W.prefill_inputs(lens, hq=4, hv=8, seed=5)
    full_o, full_s = O.prefill(O.l2norm(inp["q"]), O.l2norm(inp["k"]), inp["v"], inp["state"],
                               inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                               inp["cu_seqlens"], inp["scale"])
    for world in (1, 2, 3, 4):
        rs = [S.head_range(4, world, r) for r in range(world)]
        assert rs[0][0] == 0 and rs[-1][1] == 4
        outs, states = [], []
        for lo, hi in rs:
            sh = S.prefill_head_shard(inp, lo, hi)
            assert sh["q"].shape[1] == hi - lo and sh["v"].shape[1] == 2 * (hi - lo)
            assert sh["q"].is_contiguous() and sh["state"].is_contiguous()
            o, s = O.prefill(O.l2norm(sh["q"]), O.l2norm(sh["k"]), sh["v"], sh["state"],
                             sh["A_log"], sh["a"], sh["dt_bias"], sh["b"], sh["cu_seqlens"],
                             sh["scale"])
            outs.append(o)
            states.append(s)
        o, s = S.prefill_head_unshard(outs, states)
        assert torch.equal(o, full_o)
        assert O.state_rel_err(s, full_s) < 1e-6
    with pytest.raises(ValueError):
        S.prefill_head_shard(inp, 2, 2)
    with pytest.raises(ValueError):
        S.prefill_head_shard(W.prefill_inputs([3], hq=2, hv=3, seed=1), 0, 1)


def _oracle_run(seg, state, zero_v):
    """The prefill call of one segment, on the CPU oracle (normalised q/k)."""
    v = torch.zeros_like(seg["v"]) if zero_v else seg["v"]
    return O.prefill(O.l2norm(seg["q"]), O.l2norm(seg["k"]), v, state, seg["A_log"], seg["a"],
                     seg["dt_bias"], seg["b"], seg["cu_seqlens"], seg["scale"])


def test_segment_bounds():
    S = load_pkg().sharding
    # 512 chunks, the first segment two shares of nine
    assert S.segment_bounds(32768, 8) == [(0, 7232), (7232, 10880), (10880, 14528),
                                          (14528, 18176), (18176, 21824), (21824, 25472),
                                          (25472, 29120), (29120, 32768)]
    assert S.segment_bounds(32768, 8, first_weight=1)[1] == (4096, 8192)
    assert S.segment_bounds(130, 4) == [(0, 64), (64, 64), (64, 128), (128, 130)]
    for T, w in [(1, 3), (640, 4), (1000, 7)]:
        b = S.segment_bounds(T, w)
        assert b[0][0] == 0 and b[-1][1] == T
        assert all(b[i][1] == b[i + 1][0] for i in range(w - 1))
        assert all(lo % 64 == 0 or lo == T for lo, _ in b)


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_segment_scan_matches_unsegmented_oracle(world):
    """One sequence split into segments, each segment's (A, B) state map chained: the
    output and final state of the unsplit sequence (also with an empty segment)."""
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs([300], hq=2, hv=4, seed=81)
    ro, rs = _oracle_run(inp, inp["state"], False)
    out, fin = pkg.sharding.segment_scan_local(_oracle_run, inp, world)
    ok, frac, _, _ = O.flashinfer_allclose(out, ro, 2e-2, 2e-2)
    assert ok, frac
    assert O.state_rel_err(fin, rs) < 1e-5
    # a short sequence leaves a segment empty
    short = pkg.workloads.prefill_inputs([70], hq=1, hv=2, seed=82)
    ro, rs = _oracle_run(short, short["state"], False)
    out, fin = pkg.sharding.segment_scan_local(_oracle_run, short, 3)
    assert out.shape == ro.shape
    assert O.state_rel_err(fin, rs) < 1e-5


@pytest.mark.parametrize("T,segments", [(200, 3), (130, 2), (64, 4), (1000, 5)])
def test_one_call_segmented_scan_matches_unsplit(T, segments):
    """One sequence laid out as the 2 S - 1 runs of one call (segment 0 from the initial
    state; every later segment from the identity with v = 0 and from zero), run by the
    oracle as one multi-sequence call and assembled: the unsplit result."""
    pkg = load_pkg()
    S = pkg.sharding
    from oracle import gdn_oracle as O
    inp = pkg.workloads.prefill_inputs([T], hq=2, hv=4, seed=T + segments)
    q, k = O.l2norm(inp["q"]), O.l2norm(inp["k"])
    ro, rs = O.prefill(q, k, inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                       inp["b"], inp["cu_seqlens"], inp["scale"])
    layout = S.segmented_layout(T, segments, "cpu")
    assert len(layout[0]) == min(segments, (T + 63) // 64)
    run = S.segmented_inputs(dict(inp, q=q, k=k), layout)
    assert run["cu_seqlens"].numel() == 2 * len(layout[0])
    o_runs, f_runs = O.prefill(run["q"], run["k"], run["v"], run["state"], inp["A_log"],
                               run["a"], inp["dt_bias"], run["b"], run["cu_seqlens"],
                               inp["scale"])
    out, fin = S.segmented_finish(layout, o_runs, f_runs)
    ok, frac, mabs, _ = O.flashinfer_allclose(out, ro, 2e-2, 2e-2)
    assert ok, (frac, mabs)
    assert O.state_rel_err(fin, rs) < 1e-5


def test_segment_plans_of_the_library():
    """The segmented call's plans (gdn_prefill_segment_plan, host-only): explicit counts
    are the equal shares of sharding.segment_bounds; the automatic plan for B200's 148 SMs
    keeps one segment where the runs cannot spread (32 v-heads), and otherwise a long
    segment 0 with equal later segments."""
    pkg = load_pkg()
    S = pkg.sharding
    plan = pkg.prefill.segment_plan
    for T, n in ((32768, 5), (5000, 3), (200, 9), (130, 2), (1, 4)):
        b = plan(T, 4, n)
        assert [(b[i], b[i + 1]) for i in range(len(b) - 1)] == \
            S.segment_bounds(T, min(n, (T + 63) // 64), first_weight=1)
    assert plan(32768, 32, 0, sms=148) == [0, 32768]
    for hv, count in ((16, 4), (8, 8), (4, 5)):
        b = plan(32768, hv, 0, sms=148)
        assert len(b) == count + 1 and b[0] == 0 and b[-1] == 32768
        assert all(x % 64 == 0 for x in b[:-1])
        later = [b[i + 1] - b[i] for i in range(1, count)]
        assert b[1] >= max(later) and max(later) - min(later) <= 64
    assert plan(0, 4, 0, sms=148) == [0, 0]
