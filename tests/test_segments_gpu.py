"""GPU: one long sequence as consecutive segments chained through their affine state maps
(the multi-GPU plan for a single sequence, run here segment after segment on one GPU)
gives the output and final state of the unsplit call."""
import pytest
import torch

from conftest import load_pkg
from gpu_util import assert_parity, to

pytestmark = pytest.mark.gpu


def _kernel_run(pkg):
    def run(seg, state, zero_v):
        v = torch.zeros_like(seg["v"]) if zero_v else seg["v"]
        return pkg.gdn_prefill(seg["q"], seg["k"], v, state, seg["A_log"], seg["a"],
                               seg["dt_bias"], seg["b"], seg["cu_seqlens"], seg["scale"],
                               use_qk_l2norm=True)
    return run


@pytest.mark.parametrize("world", [2, 8])
def test_p2_segment_scan_equals_unsplit(cuda, world):
    pkg = load_pkg()
    d = to(pkg.workloads.prefill_config_inputs("P2", seed=0), cuda)
    run = _kernel_run(pkg)
    ro, rs = run(d, d["state"], False)
    out, fin = pkg.sharding.segment_scan_local(run, d, world)
    torch.cuda.synchronize()
    assert out.shape == ro.shape
    assert_parity(out, fin, ro.cpu(), rs.cpu(), what=f"P2 in {world} segments")
    assert pkg.device_error() == 0


def test_segment_scan_short_sequence_with_empty_segment(cuda):
    pkg = load_pkg()
    d = to(pkg.workloads.prefill_inputs([130], hq=2, hv=4, seed=84), cuda)
    run = _kernel_run(pkg)
    ro, rs = run(d, d["state"], False)
    out, fin = pkg.sharding.segment_scan_local(run, d, 4)  # the second segment is empty
    torch.cuda.synchronize()
    assert_parity(out, fin, ro.cpu(), rs.cpu(), what="130 tokens in 4 segments")


@pytest.mark.parametrize("L,hv", [(1, 1), (130, 4), (3648, 32)])
def test_segment_outputs_kernel_vs_fp64(cuda, L, hv):
    """gdn_segment_outputs_launch: out = S o^I + o^0 per v-head against an fp64 product of
    the same bf16 inputs (ragged last tile, one token, P2's eight-way segment length)."""
    pkg = load_pkg()
    g = torch.Generator().manual_seed(L + hv)
    o_id = (torch.randn(L, hv, 128, generator=g) * 0.1).bfloat16()
    o_zero = (torch.randn(L, hv, 128, generator=g) * 0.1).bfloat16()
    start = torch.randn(1, hv, 128, 128, generator=g) * 0.05
    A = torch.randn(1, hv, 128, 128, generator=g) * 0.05
    B = torch.randn(1, hv, 128, 128, generator=g) * 0.05
    out, fin = pkg.sharding.segment_finish(start.to(cuda), A.to(cuda), B.to(cuda),
                                           o_id.to(cuda), o_zero.to(cuda))
    torch.cuda.synchronize()
    ref = torch.einsum("thj,hvj->thv", o_id.double(), start[0].double()) + o_zero.double()
    err = (out.cpu().double() - ref).abs()
    # the bf16 rounding of the result, plus the residual of S = hi + lo (below 2^-15 of |S|)
    # over the summed terms: bounded by the magnitude of the terms, not of their sum
    mag = torch.einsum("thj,hvj->thv", o_id.double().abs(), start[0].double().abs())
    assert (err <= 2.0 ** -8 * ref.abs() + 2.0 ** -14 * mag + 1e-7).all(), err.max().item()
    ref_fin = torch.matmul(start.double(), A.double()) + B.double()
    assert torch.allclose(fin.cpu().double(), ref_fin, rtol=1e-5, atol=1e-6)


def test_segment_outputs_kernel_rejects_bad_arguments(cuda):
    pkg = load_pkg()
    from importlib import import_module
    lib = import_module(pkg.__name__ + "._lib").LIB
    t = torch.zeros(4, 2, 128, dtype=torch.bfloat16, device=cuda)
    s = torch.zeros(2, 128, 128, device=cuda)
    assert lib.gdn_segment_outputs_launch(t.data_ptr(), t.data_ptr(), s.data_ptr(), t.data_ptr(),
                                          4, 2, 64, None) == -2          # head_size
    assert lib.gdn_segment_outputs_launch(None, t.data_ptr(), s.data_ptr(), t.data_ptr(),
                                          4, 2, 128, None) == -1         # null input
    assert lib.gdn_segment_outputs_launch(t.data_ptr() + 8, t.data_ptr(), s.data_ptr(),
                                          t.data_ptr(), 3, 2, 128, None) == -1  # unaligned
    assert lib.gdn_segment_outputs_launch(None, None, None, None, 0, 2, 128, None) == 0


@pytest.mark.parametrize("world,hv", [(2, 1), (4, 3), (8, 32)])
def test_segment_chain_kernel_vs_fp64(cuda, world, hv):
    """gdn_segment_chain_launch: every rank's chained start state and final state against
    an fp64 chain of the same maps (maps scaled like contracting state maps)."""
    pkg = load_pkg()
    g = torch.Generator().manual_seed(world * 100 + hv)
    maps = torch.randn(world, 2, hv, 128, 128, generator=g) * 0.05
    maps[:, 0] += torch.eye(128) * 0.5  # A_m near a scaled identity, as decaying segments give
    # o^I[t][h][j] = (t == j): the outputs then read back the start state, out[t][h][v] =
    # bf16(start[h][v][t])
    eye = torch.eye(128).unsqueeze(1).expand(128, hv, 128).bfloat16().contiguous()
    zero = torch.zeros(128, hv, 128, dtype=torch.bfloat16)
    md = maps.double()
    for r in range(1, world):
        S = md[0, 1]
        for m in range(1, r):
            S = torch.matmul(S, md[m, 0]) + md[m, 1]
        ref_fin = torch.matmul(S, md[r, 0]) + md[r, 1]
        out, fin = pkg.sharding.segment_assemble(maps.to(cuda), r, eye.to(cuda), zero.to(cuda))
        torch.cuda.synchronize()
        assert torch.allclose(fin.cpu()[0].double(), ref_fin, rtol=1e-5, atol=1e-6), r
        start_read = out.cpu().double().permute(1, 2, 0)  # [h][v][t]
        # one bf16 rounding of S carried as hi + lo (2^-15): at most half an ulp plus that
        assert ((start_read - S).abs() <= (2.0 ** -8 + 2.0 ** -13) * S.abs() + 1e-7).all(), r


def test_segment_chain_kernel_rejects_bad_arguments(cuda):
    pkg = load_pkg()
    from importlib import import_module
    lib = import_module(pkg.__name__ + "._lib").LIB
    m = torch.zeros(2, 2, 1, 128, 128, device=cuda)
    s = torch.zeros(1, 128, 128, device=cuda)
    p = (m.data_ptr(), s.data_ptr(), s.data_ptr())
    assert lib.gdn_segment_chain_launch(p[0], 2, 0, p[1], p[2], 1, 128, None) == -1  # rank 0
    assert lib.gdn_segment_chain_launch(p[0], 2, 2, p[1], p[2], 1, 128, None) == -1  # rank >= maps
    assert lib.gdn_segment_chain_launch(p[0], 2, 1, p[1], p[2], 1, 64, None) == -2   # head_size
    assert lib.gdn_segment_chain_launch(p[0] + 4, 2, 1, p[1], p[2], 1, 128, None) == -1


@pytest.mark.parametrize("maps_n,hv", [(2, 3), (5, 4), (8, 32)])
def test_segment_chain_all_matches_per_segment_chains(cuda, maps_n, hv):
    """gdn_segment_chain_all_launch (every segment's start state in one pass) against one
    gdn_segment_chain_launch per segment: the same fp32 arithmetic, bit for bit."""
    pkg = load_pkg()
    from importlib import import_module
    lib = import_module(pkg.__name__ + "._lib").LIB
    g = torch.Generator().manual_seed(maps_n * 10 + hv)
    maps = (torch.randn(maps_n, 2, hv, 128, 128, generator=g) * 0.05).to(cuda)
    maps[:, 0] += torch.eye(128, device=cuda) * 0.5
    starts = torch.empty(maps_n - 1, hv, 128, 128, device=cuda)
    fin = torch.empty(1, hv, 128, 128, device=cuda)
    assert lib.gdn_segment_chain_all_launch(maps.data_ptr(), maps_n, starts.data_ptr(),
                                            fin.data_ptr(), hv, 128, None) == 0
    for r in range(1, maps_n):
        st = torch.empty(1, hv, 128, 128, device=cuda)
        fr = torch.empty(1, hv, 128, 128, device=cuda)
        assert lib.gdn_segment_chain_launch(maps.data_ptr(), maps_n, r, st.data_ptr(),
                                            fr.data_ptr(), hv, 128, None) == 0
        torch.cuda.synchronize()
        assert torch.equal(st[0], starts[r - 1]), r
        if r == maps_n - 1:
            assert torch.equal(fr, fin)
    assert lib.gdn_segment_chain_all_launch(maps.data_ptr(), 1, starts.data_ptr(),
                                            fin.data_ptr(), hv, 128, None) == -1
