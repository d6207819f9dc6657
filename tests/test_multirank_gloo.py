"""CPU, world_size 2 over gloo: the one-process-per-GPU driver's host logic.

* sharded decode and prefill (by sequence and by q/k-head group; oracle as the
  per-rank compute) reassemble into
  the unsharded result, and the max-over-ranks timing reduction works;
* one sequence split into segments over 2 and 3 ranks (segment-level scan, the segments'
  state maps exchanged with all_gather) gives the unsplit result;
* failure detection on the host: a rank that dies before the barrier, or whose step
  raises, makes the surviving rank's next collective end with an error within the
  process group's short timeout instead of hanging; the same through bench.py's own
  driver (barrier, max-over-ranks timing reduction).
"""
import datetime
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_NAME, REPO


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_sharded(rank, world, port, q):
    try:
        sys.path.insert(0, str(REPO))
        import importlib
        pkg = importlib.import_module(PKG_NAME)
        from oracle import gdn_oracle as O
        _init(rank, world, port, 60)
        S, W = pkg.sharding, pkg.workloads
        # decode: batch-sharded
        inp = W.decode_inputs(5, hq=1, hv=2, seed=7)
        lo, hi = S.batch_range(5, world, rank)
        o, s = O.decode(inp["q"][lo:hi], inp["k"][lo:hi], inp["v"][lo:hi], inp["state"][lo:hi],
                        inp["A_log"], inp["a"][lo:hi], inp["dt_bias"], inp["b"][lo:hi],
                        inp["scale"])
        dec = [None] * world
        dist.all_gather_object(dec, (o, s))
        # prefill: longest-first sequence sharding
        lens = [4, 11, 0, 7, 2]
        pinp = W.prefill_inputs(lens, hq=1, hv=2, seed=8)
        plan = S.lpt_assign(lens, world)
        sh = S.prefill_shard(pinp, plan[rank])
        po, ps = O.prefill(sh["q"], sh["k"], sh["v"], sh["state"], sh["A_log"], sh["a"],
                           sh["dt_bias"], sh["b"], sh["cu_seqlens"], sh["scale"])
        pre = [None] * world
        dist.all_gather_object(pre, (po, ps))
        # prefill, one sequence: q/k-head-group sharding
        hinp = W.prefill_inputs([37], hq=2, hv=4, seed=9)
        hlo, hhi = S.head_range(2, world, rank)
        hs = S.prefill_head_shard(hinp, hlo, hhi)
        ho, hst = O.prefill(hs["q"], hs["k"], hs["v"], hs["state"], hs["A_log"], hs["a"],
                            hs["dt_bias"], hs["b"], hs["cu_seqlens"], hs["scale"])
        heads = [None] * world
        dist.all_gather_object(heads, (ho, hst))
        # max-over-ranks reduction used for the bench timing
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full_o, full_s = O.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                                      inp["a"], inp["dt_bias"], inp["b"], inp["scale"])
            ok_dec = torch.equal(torch.cat([d[0] for d in dec]), full_o) and \
                O.state_rel_err(torch.cat([d[1] for d in dec]), full_s) < 1e-6
            ro, rs = O.prefill(pinp["q"], pinp["k"], pinp["v"], pinp["state"], pinp["A_log"],
                               pinp["a"], pinp["dt_bias"], pinp["b"], pinp["cu_seqlens"],
                               pinp["scale"])
            uo, us = S.prefill_unshard(sum(lens), len(lens), pinp["cu_seqlens"], plan,
                                       [x[0] for x in pre], [x[1] for x in pre])
            ok_pre = torch.equal(uo, ro) and O.state_rel_err(us, rs) < 1e-6
            fo, fs = O.prefill(hinp["q"], hinp["k"], hinp["v"], hinp["state"], hinp["A_log"],
                               hinp["a"], hinp["dt_bias"], hinp["b"], hinp["cu_seqlens"],
                               hinp["scale"])
            ho_all, hs_all = S.prefill_head_unshard([x[0] for x in heads], [x[1] for x in heads])
            ok_pre = ok_pre and torch.equal(ho_all, fo) and O.state_rel_err(hs_all, fs) < 1e-6
            q.put(("ok", ok_dec, ok_pre, float(t.item())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(("error", traceback.format_exc()))


def _worker_segments(rank, world, port, q):
    """One sequence split into `world` segments: the (A, B) state maps are exchanged with
    all_gather and the last rank's final state is the unsplit sequence's."""
    try:
        sys.path.insert(0, str(REPO))
        import importlib
        pkg = importlib.import_module(PKG_NAME)
        from oracle import gdn_oracle as O
        _init(rank, world, port, 60)
        inp = pkg.workloads.prefill_inputs([200], hq=2, hv=4, seed=83)

        def run(seg, state, zero_v):
            v = torch.zeros_like(seg["v"]) if zero_v else seg["v"]
            return O.prefill(O.l2norm(seg["q"]), O.l2norm(seg["k"]), v, state, seg["A_log"],
                             seg["a"], seg["dt_bias"], seg["b"], seg["cu_seqlens"],
                             seg["scale"])

        def all_gather(t):
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            return parts

        out, fin = pkg.sharding.segment_scan_rank(run, inp, world, rank, all_gather)
        outs = [None] * world
        dist.all_gather_object(outs, (out, fin))
        if rank == 0:
            ro, rs = run(inp, inp["state"], False)
            full = torch.cat([o for o, _ in outs], dim=0)
            ok_o, _, _, _ = O.flashinfer_allclose(full, ro, 2e-2, 2e-2)
            q.put(("ok", bool(ok_o), float(O.state_rel_err(outs[-1][1], rs))))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(("error", traceback.format_exc()))


def _worker_failing(rank, world, port, q):
    try:
        _init(rank, world, port, 3)
        if rank == 1:
            os._exit(0)  # leaves between steps, without joining the next collective
        try:
            dist.barrier()
            q.put(("no-error",))
        except Exception as e:  # the surviving rank learns of it on the host
            q.put(("detected", type(e).__name__))
    except Exception:
        q.put(("error", traceback.format_exc()))


def _worker_raising(rank, world, port, q):
    """Rank 1 raises inside its step (before the step's collective) and leaves; rank 0's
    collective ends with an error within the short timeout."""
    try:
        _init(rank, world, port, 3)
        try:
            if rank == 1:
                raise RuntimeError("step failed on rank 1")
            t = torch.ones(4)
            dist.all_reduce(t)
            q.put(("no-error",))
        except RuntimeError as e:
            if rank == 1:
                q.put(("raised", str(e)))
                q.close()
                q.join_thread()  # the message is out before the process leaves
                os._exit(0)
            q.put(("detected", type(e).__name__))
    except Exception:
        q.put(("error", traceback.format_exc()))


def _worker_bench_dist(rank, world, port, q):
    """bench.py's own driver plumbing on gloo: barrier and the max-over-ranks reduction,
    then, with rank 1 gone, its barrier ends with an error instead of hanging."""
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                          MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import importlib.util
        spec = importlib.util.spec_from_file_location("_bench_dist", REPO / "bench.py")
        B = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = B
        spec.loader.exec_module(B)
        d = B.Dist()
        d.init("gloo", timeout_s=3)
        d.barrier()
        m = d.max(1.5 * (rank + 1))
        if rank == 1:
            q.put(("max", m))
            q.close()
            q.join_thread()  # the message is out before the process leaves
            os._exit(0)
        try:
            d.barrier()
            q.put(("no-error", m))
        except Exception as e:
            q.put(("detected", m, type(e).__name__))
    except Exception:
        q.put(("error", traceback.format_exc()))


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("worker did not finish")
    items = []
    while not q.empty():
        items.append(q.get())
    return items


def test_two_rank_sharded_results_match_unsharded():
    items = _run(_worker_sharded)
    assert items, "no result from rank 0"
    assert all(i[0] == "ok" for i in items), items
    _, ok_dec, ok_pre, tmax = items[0]
    assert ok_dec and ok_pre
    assert tmax == 2.0


def test_dead_rank_is_detected_not_hung():
    items = _run(_worker_failing)
    assert ("detected",) == items[0][:1], items


@pytest.mark.parametrize("world", [2, 3])
def test_segment_scan_over_ranks_matches_unsplit(world):
    items = _run(_worker_segments, world)
    assert items and all(i[0] == "ok" for i in items), items
    _, ok_out, err = items[0]
    assert ok_out and err < 1e-5


def test_rank_that_raises_is_detected_not_hung():
    items = _run(_worker_raising)
    kinds = sorted(i[0] for i in items)
    assert kinds == ["detected", "raised"], items


def test_bench_driver_barrier_max_and_dead_rank():
    items = _run(_worker_bench_dist)
    by = {i[0]: i for i in items}
    assert "max" in by and by["max"][1] == 3.0, items
    assert "detected" in by and by["detected"][1] == 3.0, items
