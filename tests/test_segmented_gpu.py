"""GPU: the native segmented prefill of one sequence (gdn_prefill_segmented_launch: the
runs read the tokens in place through virtual rows, one chain pass, one output pass)
against the same algebra composed from separate calls on concatenated inputs
(sharding.segmented_inputs -> gdn_prefill -> sharding.segmented_finish), bit for bit, and
against the CPU oracle."""
import pytest
import torch

from conftest import load_pkg
from gpu_util import assert_parity, oracle_prefill, to

pytestmark = pytest.mark.gpu


def composed(pkg, d, segments, bounds=None):
    """The segmented scan built from a split-kernel call on concatenated runs."""
    S = pkg.sharding
    T, HV = d["q"].shape[0], d["v"].shape[1]
    layout = S.segmented_layout(T, segments, d["q"].device, bounds)
    run = S.segmented_inputs(d, layout)
    n = len(layout[0])
    o_runs, f_runs = pkg.gdn_prefill(run["q"], run["k"], run["v"], run["state"], d["A_log"],
                                     run["a"], d["dt_bias"], run["b"], run["cu_seqlens"],
                                     d["scale"], use_qk_l2norm=True, kernel="split")
    maps = torch.empty(n, 2, HV, 128, 128, dtype=torch.float32, device=d["q"].device)
    maps.view(2 * n, HV, 128, 128)[1:].copy_(f_runs)
    return S.segmented_finish(layout, o_runs, f_runs, maps=maps)


def native(pkg, d, segments, **kw):
    return pkg.gdn_prefill_segmented(d["q"], d["k"], d["v"], d.get("state"), d["A_log"], d["a"],
                                     d["dt_bias"], d["b"], d["scale"], segments=segments,
                                     use_qk_l2norm=True, **kw)


@pytest.mark.parametrize("T,hv,segments,with_state", [
    (6000, 4, 5, True),      # ragged last chunk
    (4096, 8, 2, True),
    (3000, 4, 3, False),     # no initial state
    (200, 4, 9, True),       # capped at the 4 chunks
])
def test_native_equals_composed_and_oracle(cuda, T, hv, segments, with_state):
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs([T], hq=hv // 2, hv=hv, seed=T + hv)
    if not with_state:
        inp["state"] = None
    d = to(inp, cuda)
    o, s = native(pkg, d, segments)
    co, cs = composed(pkg, d, segments)
    torch.cuda.synchronize()
    assert pkg.device_error() == 0
    assert torch.equal(o, co) and torch.equal(s, cs)
    ro, rs = oracle_prefill(inp, True)
    assert_parity(o, s, ro, rs, what=f"segmented T={T} x{segments}")


@pytest.mark.parametrize("hv", [16, 8])
def test_planned_uneven_segments_equal_composed(cuda, hv):
    """segments = 0 with the library's plan for a head share of 2 or 4 GPUs (a long
    segment 0, shorter equal later segments; P2's length), against the composition with
    the same bounds, bit for bit, and the unsplit call within the bounds."""
    pkg = load_pkg()
    T = 32768
    bounds = pkg.prefill.segment_plan(T, hv)
    later = [bounds[i + 1] - bounds[i] for i in range(1, len(bounds) - 1)]
    assert len(bounds) > 3 and bounds[1] > max(later)
    inp = pkg.workloads.prefill_inputs([T], hq=hv // 2, hv=hv, seed=hv)
    d = to(inp, cuda)
    o, s = native(pkg, d, 0)
    o2, s2 = native(pkg, d, 0, bounds=bounds)   # the same plan given explicitly
    co, cs = composed(pkg, d, 0, bounds)
    ro, rs = pkg.gdn_prefill(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                             d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"],
                             use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert pkg.device_error() == 0
    assert torch.equal(o, co) and torch.equal(s, cs)
    assert torch.equal(o2, o) and torch.equal(s2, s)
    assert_parity(o, s, ro.cpu(), rs.cpu(), what=f"planned segments hv={hv}")


def test_one_segment_is_the_split_call(cuda):
    pkg = load_pkg()
    d = to(pkg.workloads.prefill_inputs([1000], hq=2, hv=4, seed=71), cuda)
    o, s = native(pkg, d, 1)
    ro, rs = pkg.gdn_prefill(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                             d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"],
                             use_qk_l2norm=True, kernel="split")
    torch.cuda.synchronize()
    assert torch.equal(o, ro) and torch.equal(s, rs)


def test_strided_views_in_place_state_and_auto_count(cuda):
    """q, k, v, a, b as slices of fused projections (read in place), the state updated in
    place, segments = 0 (the device's own count): the dense call's results."""
    pkg = load_pkg()
    from test_strided_gpu import fused_views
    d = to(pkg.workloads.prefill_inputs([5000], hq=2, hv=4, seed=72), cuda)
    S = pkg.prefill.segments_auto(5000, 4)
    assert S == len(pkg.prefill.segment_plan(5000, 4)) - 1 and S > 1
    o, s = native(pkg, d, 0)
    sv = fused_views(d, (5000,))
    st = d["state"].clone()
    out = torch.full_like(o, float("nan"))
    o2, s2 = pkg.gdn_prefill_segmented(sv["q"], sv["k"], sv["v"], st, d["A_log"], sv["a"],
                                       d["dt_bias"], sv["b"], d["scale"], out, st,
                                       use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert o2 is out and s2 is st
    assert torch.equal(o2, o) and torch.equal(s2, s)


def test_empty_sequence_gives_zero_state(cuda):
    pkg = load_pkg()
    d = to(pkg.workloads.prefill_inputs([0], hq=2, hv=4, seed=73), cuda)
    ns = torch.full((1, 4, 128, 128), float("nan"), device=cuda)
    o, s = pkg.gdn_prefill_segmented(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                     d["dt_bias"], d["b"], d["scale"], None, ns,
                                     use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert o.shape == (0, 4, 128) and s is ns and torch.count_nonzero(s) == 0


def test_c_abi_rejections(cuda):
    """Arguments the C entry point refuses before any launch."""
    pkg = load_pkg()
    L = pkg.LIB
    d = to(pkg.workloads.prefill_inputs([256], hq=2, hv=4, seed=74), cuda)
    out = torch.empty(256, 4, 128, dtype=torch.bfloat16, device=cuda)
    ns = torch.empty(1, 4, 128, 128, device=cuda)
    nbytes = L.gdn_prefill_segmented_workspace_size(256, 4, 2, None)
    ws = torch.empty(nbytes + 2048, dtype=torch.uint8, device=cuda)
    base = (ws.data_ptr() + 1023) // 1024 * 1024

    def call(out_ptr=out.data_ptr(), ws_ptr=base, ws_len=nbytes, hk=2, segments=2, qs=256):
        return L.gdn_prefill_segmented_launch(
            d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["state"].data_ptr(),
            d["A_log"].data_ptr(), d["a"].data_ptr(), d["dt_bias"].data_ptr(),
            d["b"].data_ptr(), 0.0, out_ptr, ns.data_ptr(), 256, 2, hk, 4, 128, 1, segments,
            None, qs, 256, 512, 4, 4, ws_ptr, ws_len, torch.cuda.current_stream().cuda_stream)
    name = lambda st: L.gdn_status_string(st).decode()  # noqa: E731
    assert name(call(ws_len=nbytes - 1)) == "GDN_ERR_WORKSPACE"
    assert name(call(ws_ptr=base + 16)) == "GDN_ERR_INVALID_ARGUMENT"   # not 1024-aligned
    assert name(call(hk=4)) == "GDN_ERR_UNSUPPORTED"
    assert name(call(segments=-1)) == "GDN_ERR_INVALID_ARGUMENT"
    assert name(call(qs=128)) == "GDN_ERR_INVALID_ARGUMENT"            # overlapping q rows
    assert name(call(out_ptr=out.data_ptr() + 8)) == "GDN_ERR_UNSUPPORTED"  # output unaligned
    assert call() == 0
    torch.cuda.synchronize()
    ro, rs = native(pkg, d, 2)
    torch.cuda.synchronize()
    assert torch.equal(out, ro) and torch.equal(ns, rs)
