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
