"""GPU: the pipelined one-sequence prefill (two pieces, the second piece's preparation on
the SMs the first piece's state kernel leaves idle) when the sequence does not cover the
token rows exactly: cu_seqlens starting after row 0, and a sequence that ends inside the
first piece (the second piece is then empty and passes the state through).  Each must give,
bit for bit, the call on just the sequence's tokens, and leave the rows outside it alone."""
import pytest
import torch

from conftest import load_pkg
from gpu_util import to

pytestmark = pytest.mark.gpu

ARGS = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale")


def trimmed(d, lo, hi):
    """The one-sequence problem of rows [lo, hi) as its own dense call."""
    out = dict(d)
    for key in ("q", "k", "v", "a", "b"):
        out[key] = d[key][lo:hi].contiguous()
    out["cu_seqlens"] = torch.tensor([0, hi - lo], dtype=torch.int32, device=d["q"].device)
    return out


@pytest.mark.parametrize("lo,hi", [(0, 32768), (1000, 32768), (0, 9000), (130, 20130)])
def test_sequence_inside_the_rows(cuda, lo, hi):
    pkg = load_pkg()
    d = to(pkg.workloads.prefill_inputs([32768], hq=16, hv=32, seed=55), cuda)
    d["cu_seqlens"] = torch.tensor([lo, hi], dtype=torch.int32, device=cuda)
    out = torch.full((32768, 32, 128), 7.0, dtype=torch.bfloat16, device=cuda)
    o, s = pkg.gdn_prefill(*[d[k] for k in ARGS], out, None, use_qk_l2norm=True, kernel="split")
    t = trimmed(d, lo, hi)
    ro, rs = pkg.gdn_prefill(*[t[k] for k in ARGS], use_qk_l2norm=True, kernel="split")
    torch.cuda.synchronize()
    assert pkg.device_error() == 0
    assert torch.equal(o[lo:hi], ro) and torch.equal(s, rs)
    assert bool((o[:lo] == 7.0).all()) and bool((o[hi:] == 7.0).all())


def test_int64_offsets_and_in_place_state(cuda):
    pkg = load_pkg()
    d = to(pkg.workloads.prefill_inputs([20000], hq=16, hv=32, seed=56), cuda)
    o, s = pkg.gdn_prefill(*[d[k] for k in ARGS], use_qk_l2norm=True, kernel="split")
    e = dict(d, cu_seqlens=d["cu_seqlens"].to(torch.int64), state=d["state"].clone())
    o2, s2 = pkg.gdn_prefill(*[e[k] for k in ARGS], None, e["state"], use_qk_l2norm=True,
                             kernel="split")
    torch.cuda.synchronize()
    assert s2.data_ptr() == e["state"].data_ptr()
    assert torch.equal(o2, o) and torch.equal(s2, s)
