"""GPU: decode and multi-token decode launched from a captured CUDA graph (the way serving
loops launch decode, and the way bench.py times them) give bitwise the eager results."""
import pytest
import torch

from conftest import load_pkg
from gpu_util import to

pytestmark = pytest.mark.gpu


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # first calls (one-time kernel set-up) outside the capture
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


@pytest.mark.parametrize("batch,bf16", [(128, False), (32, True), (4, False)])
def test_decode_graph_replay_equals_eager(cuda, batch, bf16):
    pkg = load_pkg()
    d = to(pkg.workloads.decode_inputs(batch, seed=71), cuda)
    if bf16:  # B=32 x 32 v-heads: the streaming kernel
        d["state"] = d["state"].to(torch.bfloat16)
    args = [d[x] for x in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")]
    out = torch.empty_like(d["v"])
    ns = torch.empty_like(d["state"])
    g = _capture(lambda: pkg.gdn_decode(*args, d["scale"], out, ns, use_qk_l2norm=True))
    out.zero_()
    ns.zero_()
    g.replay()
    torch.cuda.synchronize()
    ro, rs = pkg.gdn_decode(*args, d["scale"], use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert torch.equal(out, ro) and torch.equal(ns, rs)
    assert pkg.device_error() == 0


def test_mtp_graph_replay_equals_eager(cuda):
    pkg = load_pkg()
    B, T = 16, 4
    d = to(pkg.workloads.mtp_inputs(B, T, B, seed=72), cuda)
    names = ("q", "k", "v", "state", "state_indices", "A_log", "a", "dt_bias", "b")

    def run(pool, out, inter):
        return pkg.gdn_mtp(*[pool if x == "state" else d[x] for x in names], d["scale"], out,
                           None, inter, use_qk_l2norm=True)

    pool0 = d["state"].clone()
    out = torch.empty_like(d["v"])
    inter = torch.empty((B, T) + tuple(pool0.shape[1:]), device=cuda)
    pool = pool0.clone()
    g = _capture(lambda: run(pool, out, inter))
    pool.copy_(pool0)  # the capture's warm-up call updated the pool in place
    g.replay()
    torch.cuda.synchronize()
    ref_pool = pool0.clone()
    ref_out = torch.empty_like(out)
    ref_inter = torch.empty_like(inter)
    run(ref_pool, ref_out, ref_inter)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(pool, ref_pool)
    assert torch.equal(inter, ref_inter)


@pytest.mark.parametrize("kind", ["fused", "split", "segmented"])
def test_prefill_graph_replay_equals_eager(cuda, kind):
    """Prefill launched from a captured CUDA graph (how bench.py replays prefill steps):
    the fused and split kernel families, and the one-call segmented scan of one sequence
    (its input concatenations, the call, the chain and output kernels), bitwise the eager
    results."""
    pkg = load_pkg()
    if kind == "segmented":
        d = to(pkg.workloads.prefill_inputs([3000], hq=2, hv=4, seed=72), cuda)
        args = [d[x] for x in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")]
        out = torch.empty(3000, 4, 128, dtype=torch.bfloat16, device=cuda)
        ns = torch.empty(1, 4, 128, 128, device=cuda)

        def call(o=out, s=ns):
            return pkg.gdn_prefill_segmented(*args, d["scale"], o, s, use_qk_l2norm=True)
    else:
        d = to(pkg.workloads.prefill_inputs([70, 0, 129, 300], seed=73), cuda)
        args = [d[x] for x in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b",
                               "cu_seqlens")]
        out = torch.empty_like(d["v"])
        ns = torch.empty_like(d["state"])

        def call(o=out, s=ns):
            return pkg.gdn_prefill(*args, d["scale"], o, s, use_qk_l2norm=True, kernel=kind)
    g = _capture(call)
    out.zero_()
    ns.zero_()
    g.replay()
    torch.cuda.synchronize()
    ro, rs = call(torch.empty_like(out), torch.empty_like(ns))
    torch.cuda.synchronize()
    assert torch.equal(out, ro) and torch.equal(ns, rs)
    assert pkg.device_error() == 0
