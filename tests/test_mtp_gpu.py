"""GPU parity: the sm_100a multi-token decode (gdn_mtp_launch) vs the CPU oracle."""
import pytest
import torch

from conftest import load_golden, load_pkg
from gpu_util import OUT_ATOL, STATE_REL, assert_parity, to
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


def oracle_mtp(inp, l2, inter=False):
    q, k = (O.l2norm(inp["q"]), O.l2norm(inp["k"])) if l2 else (inp["q"], inp["k"])
    return O.mtp(q, k, inp["v"], inp["state"], inp["state_indices"], inp["A_log"], inp["a"],
                 inp["dt_bias"], inp["b"], inp.get("scale"), intermediate=inter)


def run(pkg, inp, l2, dev, *, inter=False, inplace=True):
    d = to(inp, dev)
    P, HV = d["state"].shape[:2]
    B, T = d["q"].shape[:2]
    buf = torch.full((P, T, HV, 128, 128), 0.0, device=dev) if inter else None
    fin = None if inplace else torch.full_like(d["state"], float("nan"))
    o, s = pkg.gdn_mtp(d["q"], d["k"], d["v"], d["state"], d["state_indices"], d["A_log"],
                       d["a"], d["dt_bias"], d["b"], d.get("scale"), None, fin, buf,
                       use_qk_l2norm=l2)
    torch.cuda.synchronize()
    if inplace:
        assert s.data_ptr() == d["state"].data_ptr()
    return o, s, buf


@pytest.mark.parametrize("name,l2,inter", [("mtp_gva_inter", False, True), ("mtp_l2", True, False)])
def test_golden(cuda, name, l2, inter):
    pkg = load_pkg()
    d, m = load_golden(name)
    d["scale"] = float(m["scale"])
    o, s, it = run(pkg, d, l2, cuda, inter=inter)
    assert_parity(o, s, d["out"], d["final_state"], what=name)
    if inter:
        assert O.state_rel_err(it.cpu(), d["intermediate"]) <= STATE_REL


@pytest.mark.parametrize("l2", [True, False])
@pytest.mark.parametrize("inplace", [True, False])
def test_pool_padding_and_rollback_buffer(cuda, l2, inplace):
    pkg = load_pkg()
    # rows 1 and 4 are padding (-1 and an index past the pool)
    inp = pkg.workloads.mtp_inputs(5, 3, 8, hq=2, hv=4, seed=31, indices=[6, -1, 0, 3, 8])
    ro, rs, rit = oracle_mtp(inp, l2, inter=True)
    o, s, it = run(pkg, inp, l2, cuda, inter=True, inplace=inplace)
    assert_parity(o, s, ro, rs, what=f"pool l2={l2} inplace={inplace}")
    assert O.state_rel_err(it.cpu(), rit) <= STATE_REL
    assert o[1].abs().max().item() == 0.0 and o[4].abs().max().item() == 0.0
    untouched = [1, 2, 4, 5, 7]
    assert torch.equal(s.cpu()[untouched], inp["state"][untouched])


def test_int64_indices_and_long_draft(cuda):
    pkg = load_pkg()
    inp = pkg.workloads.mtp_inputs(4, 8, 6, hq=4, hv=8, seed=32, index_dtype=torch.int64)
    ro, rs, _ = oracle_mtp(inp, True)
    o, s, _ = run(pkg, inp, True, cuda)
    assert_parity(o, s, ro, rs, what="int64 T=8")


def test_full_size_equals_successive_decode_steps_bitwise(cuda):
    """B=128 rows, T=4 tokens, 16/32 heads: the multi-token kernel applies exactly the
    decode kernel's per-token arithmetic, so it equals four gdn_decode launches bit for
    bit (outputs, final states and the state after every token)."""
    pkg = load_pkg()
    B, T, P = 128, 4, 160
    inp = to(pkg.workloads.mtp_inputs(B, T, P, seed=33), cuda)
    pool0 = inp["state"].clone()
    buf = torch.zeros(P, T, 32, 128, 128, device=cuda)
    o, s = pkg.gdn_mtp(inp["q"], inp["k"], inp["v"], inp["state"], inp["state_indices"],
                       inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["scale"],
                       intermediate_states_buffer=buf, use_qk_l2norm=True)
    idx = inp["state_indices"].long()
    st = pool0[idx].contiguous()
    for t in range(T):
        sl = slice(t, t + 1)
        od, st = pkg.gdn_decode(inp["q"][:, sl].contiguous(), inp["k"][:, sl].contiguous(),
                                inp["v"][:, sl].contiguous(), st, inp["A_log"],
                                inp["a"][:, sl].contiguous(), inp["dt_bias"],
                                inp["b"][:, sl].contiguous(), inp["scale"],
                                use_qk_l2norm=True)
        assert torch.equal(o[:, t], od[:, 0])
        assert torch.equal(buf[idx, t], st)
    assert torch.equal(s[idx], st)
    others = torch.ones(P, dtype=torch.bool, device=cuda)
    others[idx] = False
    assert torch.equal(s[others], pool0[others])


def test_dps_kernel_arity_and_errors(cuda):
    pkg = load_pkg()
    import inspect
    assert len(inspect.signature(pkg.mtp_kernel).parameters) == 13
    inp = to(pkg.workloads.mtp_inputs(2, 2, 3, hq=1, hv=2, seed=34), cuda)
    with pytest.raises(TypeError):
        pkg.gdn_mtp(inp["q"], inp["k"], inp["v"], inp["state"],
                    inp["state_indices"].float(), inp["A_log"], inp["a"], inp["dt_bias"],
                    inp["b"], inp["scale"])
    with pytest.raises(ValueError):
        pkg.gdn_mtp(inp["q"], inp["k"], inp["v"][:, :1].contiguous(), inp["state"],
                    inp["state_indices"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                    inp["scale"])
    fin = torch.empty_like(inp["state"])
    o, s = pkg.mtp_kernel(inp["q"], inp["k"], inp["v"], inp["state"], inp["state_indices"],
                          inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["scale"], None,
                          torch.empty(2, 2, 2, 128, dtype=torch.bfloat16, device=cuda), fin)
    torch.cuda.synchronize()
    ro, rs, _ = oracle_mtp({k_: (v_.cpu() if isinstance(v_, torch.Tensor) else v_)
                            for k_, v_ in inp.items()}, False)
    assert_parity(o, s, ro, rs, what="dps")


@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("inplace", [True, False])
def test_rollback_buffer_leaves_results_unchanged_bitwise(cuda, state_dtype, inplace):
    """With enough (row, v-head) pairs for the largest CTAs, a call with the rollback
    buffer and one without agree bit for bit (outputs and final pools, padding rows
    included), in place and out of place, for fp32 and bf16 pools; the buffer's last
    token holds the final state."""
    pkg = load_pkg()
    B, T, P = 40, 3, 48
    idx = list(range(3, 43))
    idx[5], idx[17] = -1, P + 2  # padding rows
    inp = to(pkg.workloads.mtp_inputs(B, T, P, seed=35, indices=idx), cuda)
    inp["state"] = inp["state"].to(state_dtype)
    args = lambda pool: (inp["q"], inp["k"], inp["v"], pool, inp["state_indices"],  # noqa: E731
                         inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["scale"])
    pool_a = inp["state"].clone()
    o_a, s_a = pkg.gdn_mtp(*args(pool_a), use_qk_l2norm=True)
    pool_b = inp["state"].clone()
    buf = torch.zeros((P, T) + tuple(pool_b.shape[1:]), dtype=state_dtype, device=cuda)
    fin = None if inplace else torch.full_like(pool_b, float("nan"))
    o_b, s_b = pkg.gdn_mtp(*args(pool_b), None, fin, buf, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert pkg.device_error() == 0
    assert torch.equal(o_a, o_b) and torch.equal(s_a, s_b)
    rows = torch.tensor([i for i in idx if 0 <= i < P], device=cuda)
    assert torch.equal(buf[rows, T - 1], s_b[rows])
    assert o_b[5].abs().max().item() == 0.0 and o_b[17].abs().max().item() == 0.0
    ro, rs, _ = oracle_mtp({k_: (v_.cpu() if isinstance(v_, torch.Tensor) else v_)
                            for k_, v_ in inp.items()}, True)
    assert_parity(o_b, s_b.float(), ro, rs.float(), what=f"rollback {state_dtype}")
