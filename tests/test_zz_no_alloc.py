"""GPU: the allocation-free prefill entry point (gdn_prefill_launch_noalloc).

That entry point exists for callers that cannot allocate device memory where
they launch (allocator or memory-pool callbacks, runtimes whose device memory
is fully pre-reserved, plugin hosts that pass only inputs and outputs): it
uses a fixed scratch array inside the library instead of a caller workspace.
These tests call it through the C ABI twice in a row and check both results
against the CPU oracle and against the regular entry point (gdn_prefill_launch
with a workspace), with the same tolerances as the other prefill tests; run it
on buffers only 8 bytes past a 16-byte boundary right after a tensor-core call
has left its contents in the scratch array (that call takes the token-serial
kernel); and check that a request beyond its fixed capacity is refused
without launching anything.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
import pytest
import torch

from conftest import load_pkg
from gpu_util import OUT_ATOL, STATE_REL, assert_parity, oracle_prefill
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

LENS = [70, 5, 129, 0, 64, 200, 1]  # several sequences: the scratch order is used


def _noalloc(pkg, d, out, ns, l2):
    T, HQ, D = d["q"].shape
    HV = d["v"].shape[1]
    N = d["cu_seqlens"].numel() - 1
    return pkg.LIB.gdn_prefill_launch_noalloc(
        d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["state"].data_ptr(),
        d["A_log"].data_ptr(), d["a"].data_ptr(), d["dt_bias"].data_ptr(), d["b"].data_ptr(),
        d["cu_seqlens"].data_ptr(), 0, d["scale"], out.data_ptr(), ns.data_ptr(), T, N, HQ, HQ,
        HV, D, int(l2), torch.cuda.current_stream().cuda_stream)


def _shifted(t, dev):
    """A copy of `t` whose data starts 8 bytes past a 16-byte boundary."""
    buf = torch.empty(t.numel() + 4, dtype=t.dtype, device=dev)
    view = buf[4:].view(t.shape)
    view.copy_(t)
    assert view.data_ptr() % 16 == 8
    return view


def test_noalloc_matches_oracle_and_workspace_entry_point_twice(cuda):
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs(LENS, seed=41)
    ro, rs = oracle_prefill(inp, True)
    d = {k: (v.to(cuda) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    ref_o, ref_s = pkg.gdn_prefill(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                   d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"],
                                   use_qk_l2norm=True)
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        out = torch.full_like(ref_o, float("nan"))
        ns = torch.full_like(ref_s, float("nan"))
        status = _noalloc(pkg, d, out, ns, True)
        assert status == 0, pkg.LIB.gdn_status_string(status)
        torch.cuda.synchronize()
        assert_parity(out, ns, ro, rs, what="no-alloc vs oracle")
        ok, frac, mabs, _ = O.flashinfer_allclose(out.cpu(), ref_o.cpu(), OUT_ATOL, OUT_ATOL)
        assert ok, (frac, mabs)
        assert O.state_rel_err(ns.cpu(), ref_s.cpu()) <= STATE_REL
    assert pkg.device_error() == 0


def test_noalloc_unaligned_buffers_after_a_tensor_core_call(cuda):
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs(LENS, seed=43)
    ro, rs = oracle_prefill(inp, True)
    d = {k: (v.to(cuda) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    out = torch.empty(d["v"].shape, dtype=torch.bfloat16, device=cuda)
    ns = torch.empty_like(d["state"])
    assert _noalloc(pkg, d, out, ns, True) == 0  # aligned: the tensor-core kernel
    torch.cuda.synchronize()
    assert_parity(out, ns, ro, rs, what="no-alloc aligned")
    sh = dict(d)
    for key in ("q", "k", "v"):
        sh[key] = _shifted(d[key], cuda)
    out2 = _shifted(torch.full_like(out, float("nan")), cuda)
    ns2 = torch.full_like(ns, float("nan"))
    assert _noalloc(pkg, sh, out2, ns2, True) == 0  # 8-byte aligned: token-serial kernel
    torch.cuda.synchronize()
    assert_parity(out2, ns2, ro, rs, what="no-alloc unaligned")
    assert pkg.device_error() == 0


def test_noalloc_refuses_more_sequences_than_its_scratch_holds(cuda):
    pkg = load_pkg()
    lens = [1] * 4097
    inp = pkg.workloads.prefill_inputs(lens, hq=1, hv=1, seed=42, with_state=True)
    d = {k: (v.to(cuda) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    out = torch.zeros_like(d["v"])
    ns = torch.zeros_like(d["state"])
    status = _noalloc(pkg, d, out, ns, True)
    torch.cuda.synchronize()
    assert pkg.LIB.gdn_status_string(status) == b"GDN_ERR_TOO_LARGE"
    assert out.abs().max().item() == 0.0  # nothing was launched
