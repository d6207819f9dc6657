"""GPU parity: bf16 state storage (gdn_decode_launch_bf16state, gdn_mtp_launch_bf16state)
vs the CPU oracle with the same storage semantics (widen on load, fp32 update, round to
nearest bf16 on store)."""
import pytest
import torch

from conftest import load_pkg
from gpu_util import STATE_REL, assert_parity, to
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


def bf16_state(inp, key="state"):
    inp = dict(inp)
    inp[key] = inp[key].to(torch.bfloat16)
    return inp


@pytest.mark.parametrize("l2", [True, False])
def test_decode_bf16_state_vs_oracle(cuda, l2):
    pkg = load_pkg()
    inp = bf16_state(pkg.workloads.decode_inputs(7, hq=4, hv=8, seed=61))
    q, k = (O.l2norm(inp["q"]), O.l2norm(inp["k"])) if l2 else (inp["q"], inp["k"])
    ro, rs = O.decode(q, k, inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                      inp["b"], inp["scale"])
    assert rs.dtype == torch.bfloat16
    d = to(inp, cuda)
    o, s = pkg.gdn_decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                          d["b"], d["scale"], use_qk_l2norm=l2)
    torch.cuda.synchronize()
    assert s.dtype == torch.bfloat16
    assert_parity(o, s.float(), ro, rs.float(), what=f"bf16 state l2={l2}")
    # both sides round the same fp32 values: all but rare ties land on the same bf16
    assert (s.cpu() == rs).float().mean().item() > 0.999


def test_decode_bf16_state_many_heads_vs_oracle(cuda):
    """B=32 x 32 v-heads (1024 heads: the largest-CTA configuration of the kernel)."""
    pkg = load_pkg()
    inp = bf16_state(pkg.workloads.decode_inputs(32, seed=65))
    ro, rs = O.decode(O.l2norm(inp["q"]), O.l2norm(inp["k"]), inp["v"], inp["state"],
                      inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["scale"])
    d = to(inp, cuda)
    o, s = pkg.gdn_decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                          d["b"], d["scale"], use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert_parity(o, s.float(), ro, rs.float(), what="bf16 B=32")
    assert (s.cpu() == rs).float().mean().item() > 0.999


def test_decode_bf16_state_b1024_equals_shards_bitwise(cuda):
    pkg = load_pkg()
    inp = to(bf16_state(pkg.workloads.decode_inputs(1024, seed=62)), cuda)
    args = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")
    o, s = pkg.gdn_decode(*[inp[x] for x in args], inp["scale"], use_qk_l2norm=True)
    for r in range(8):
        sl = slice(128 * r, 128 * (r + 1))
        part = {x: (inp[x][sl].contiguous() if x not in ("A_log", "dt_bias") else inp[x])
                for x in args}
        po, ps = pkg.gdn_decode(*[part[x] for x in args], inp["scale"], use_qk_l2norm=True)
        assert torch.equal(po, o[sl]) and torch.equal(ps, s[sl])


def test_decode_bf16_streaming_equals_one_shot_bitwise(cuda):
    """B=32 (1024 heads) takes the streaming kernel, B=4 slices the one-shot kernel: the
    per-row arithmetic is the same, so the results are bitwise equal; also in place."""
    pkg = load_pkg()
    inp = to(bf16_state(pkg.workloads.decode_inputs(32, seed=66)), cuda)
    args = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")
    o, s = pkg.gdn_decode(*[inp[x] for x in args], inp["scale"], use_qk_l2norm=True)
    for r in range(8):
        sl = slice(4 * r, 4 * (r + 1))
        part = {x: (inp[x][sl].contiguous() if x not in ("A_log", "dt_bias") else inp[x])
                for x in args}
        po, ps = pkg.gdn_decode(*[part[x] for x in args], inp["scale"], use_qk_l2norm=True)
        assert torch.equal(po, o[sl]) and torch.equal(ps, s[sl])
    st = inp["state"].clone()
    o2, s2 = pkg.gdn_decode(*[inp[x] if x != "state" else st for x in args], inp["scale"], None, st,
                            use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert s2.data_ptr() == st.data_ptr()
    assert torch.equal(o2, o) and torch.equal(st, s)
    assert pkg.device_error() == 0


def test_decode_bf16_unaligned_qkv_takes_one_shot_path(cuda):
    """q/k/v only 8-byte aligned: the streaming kernel's bulk copies need 16 bytes, so the
    call runs the one-shot kernel; the results are the same bits."""
    pkg = load_pkg()
    inp = to(bf16_state(pkg.workloads.decode_inputs(32, seed=67)), cuda)
    args = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")
    o, s = pkg.gdn_decode(*[inp[x] for x in args], inp["scale"], use_qk_l2norm=True)
    shifted = dict(inp)
    for x in ("q", "k", "v"):
        t = inp[x]
        buf = torch.empty(t.numel() + 4, dtype=t.dtype, device=cuda)
        view = buf[4:].view(t.shape)  # 8 bytes past a 16-byte boundary
        view.copy_(t)
        assert view.data_ptr() % 16 == 8
        shifted[x] = view
    o2, s2 = pkg.gdn_decode(*[shifted[x] for x in args], inp["scale"], use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert torch.equal(o2, o) and torch.equal(s2, s)


def test_decode_bf16_zero_state(cuda):
    pkg = load_pkg()
    inp = pkg.workloads.decode_inputs(3, hq=1, hv=2, seed=63, with_state=False)
    ro, rs = O.decode(O.l2norm(inp["q"]), O.l2norm(inp["k"]), inp["v"], None, inp["A_log"],
                      inp["a"], inp["dt_bias"], inp["b"], inp["scale"])
    d = to(inp, cuda)
    ns = torch.empty(3, 2, 128, 128, dtype=torch.bfloat16, device=cuda)
    o, s = pkg.gdn_decode(d["q"], d["k"], d["v"], None, d["A_log"], d["a"], d["dt_bias"], d["b"],
                          d["scale"], None, ns, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert s.data_ptr() == ns.data_ptr()
    assert_parity(o, s.float(), ro, rs.to(torch.bfloat16).float(), what="bf16 zero state")


@pytest.mark.parametrize("l2", [True, False])
def test_mtp_bf16_pool_vs_oracle(cuda, l2):
    pkg = load_pkg()
    inp = bf16_state(pkg.workloads.mtp_inputs(5, 4, 8, hq=2, hv=4, seed=64,
                                              indices=[6, -1, 0, 3, 2]))
    q, k = (O.l2norm(inp["q"]), O.l2norm(inp["k"])) if l2 else (inp["q"], inp["k"])
    ro, rs, rit = O.mtp(q, k, inp["v"], inp["state"], inp["state_indices"], inp["A_log"],
                        inp["a"], inp["dt_bias"], inp["b"], inp["scale"], intermediate=True)
    d = to(inp, cuda)
    buf = torch.zeros(8, 4, 4, 128, 128, dtype=torch.bfloat16, device=cuda)
    o, s = pkg.gdn_mtp(d["q"], d["k"], d["v"], d["state"], d["state_indices"], d["A_log"],
                       d["a"], d["dt_bias"], d["b"], d["scale"], None, None, buf,
                       use_qk_l2norm=l2)
    torch.cuda.synchronize()
    assert s.dtype == torch.bfloat16 and s.data_ptr() == d["state"].data_ptr()
    assert_parity(o, s.float(), ro, rs.float(), what=f"mtp bf16 l2={l2}")
    assert O.state_rel_err(buf.cpu().float(), rit.float()) <= STATE_REL
    assert o[1].abs().max().item() == 0.0
