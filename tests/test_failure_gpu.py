"""GPU: the bounded-wait path that keeps a lost arrival from hanging the GPU, exercised
without any fault.  A wait on a barrier nothing arrives on gives up after its iteration
limit, records its bit in the device error word and returns; the context stays usable
(a decode call afterwards matches the oracle)."""
import pytest
import torch

from conftest import load_pkg
from gpu_util import assert_parity, oracle_decode, to

pytestmark = pytest.mark.gpu


def _selftest(pkg, limit, arrive, dev):
    res = torch.full((1,), -1, dtype=torch.int32, device=dev)
    status = pkg.LIB.gdn_selftest_bounded_wait(limit, arrive, res.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream)
    assert status == 0, pkg.LIB.gdn_status_string(status)
    torch.cuda.synchronize()
    return int(res.item())


def test_wait_that_is_satisfied_sets_no_error(cuda):
    pkg = load_pkg()
    assert pkg.device_error() == 0
    assert _selftest(pkg, 1 << 12, 1, cuda) == 1
    assert pkg.device_error() == 0


def test_wait_that_runs_out_reports_and_returns(cuda):
    pkg = load_pkg()
    assert pkg.device_error() == 0
    assert _selftest(pkg, 1 << 12, 0, cuda) == 0          # nothing arrived: gave up
    assert pkg.device_error(clear=False) == 16            # reported, not cleared yet
    assert pkg.device_error() == 16                       # read and cleared
    assert pkg.device_error() == 0
    # the context is still usable
    inp = pkg.workloads.decode_inputs(3, hq=2, hv=4, seed=97)
    d = to(inp, cuda)
    o, s = pkg.gdn_decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                          d["dt_bias"], d["b"], d["scale"], use_qk_l2norm=True)
    torch.cuda.synchronize()
    ro, rs = oracle_decode(inp, True)
    assert_parity(o, s, ro, rs, what="decode after the self-test")


def test_selftest_rejects_bad_arguments(cuda):
    pkg = load_pkg()
    assert pkg.LIB.gdn_selftest_bounded_wait(0, 0, None, None) == -1
    assert pkg.LIB.gdn_selftest_bounded_wait((1 << 24) + 1, 0, None, None) == -1
    buf = torch.zeros(2, dtype=torch.int32, device=cuda)
    assert pkg.LIB.gdn_selftest_bounded_wait(16, 1, buf.data_ptr() + 2, None) == -1
