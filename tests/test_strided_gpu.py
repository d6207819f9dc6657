"""GPU: q, k, v, a, b and the output as strided views, the way a model hands them over
(slices of one fused projection per token), as the reference's wrappers allow by passing
every stride to their kernels (gdn_decode/solution/triton/kernel.py:255-264,
gdn_prefill/solution/triton/kernel.py:318-325).  Strided rows go to the kernels as they
are (no copy): results equal the dense call bit for bit and match the oracle."""
import pytest
import torch

from conftest import load_pkg
from gpu_util import assert_parity, oracle_decode, oracle_prefill, to

pytestmark = pytest.mark.gpu

ARGS_P = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale")
ARGS_D = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale")


def fused_views(d, lead, pad=0):
    """q, k, v as slices of one [*lead, 2 HQ 128 + HV 128 + pad] tensor and a, b as
    slices of one [*lead, 2 HV + pad] tensor, holding the values of d's tensors."""
    HQ, HV = d["q"].shape[-2], d["v"].shape[-2]
    dev = d["q"].device
    qkv = torch.zeros(*lead, (2 * HQ + HV) * 128 + pad, dtype=torch.bfloat16, device=dev)
    ab = torch.zeros(*lead, 2 * HV + pad, dtype=torch.bfloat16, device=dev)
    out = dict(d)
    n = HQ * 128
    out["q"] = qkv[..., :n].unflatten(-1, (HQ, 128))
    out["k"] = qkv[..., n:2 * n].unflatten(-1, (HQ, 128))
    out["v"] = qkv[..., 2 * n:2 * n + HV * 128].unflatten(-1, (HV, 128))
    out["a"] = ab[..., :HV]
    out["b"] = ab[..., HV:2 * HV]
    for key in ("q", "k", "v", "a", "b"):
        out[key].copy_(d[key])
        assert not out[key].is_contiguous()
    return out


def strided_output(shape, dev, pad=64):
    """An output view whose rows are `pad` elements longer than dense."""
    rows = shape[0]
    inner = 1
    for s in shape[1:]:
        inner *= s
    buf = torch.full((rows, inner + pad), float("nan"), dtype=torch.bfloat16, device=dev)
    return buf[:, :inner].view(shape)


@pytest.mark.parametrize("kernel", ["auto", "split", "fused", "recurrent"])
def test_prefill_fused_projection_views(cuda, kernel):
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs([70, 0, 129, 5], seed=91)
    d = to(inp, cuda)
    fn = pkg.gdn_prefill_recurrent if kernel == "recurrent" else \
        (lambda *a, **k: pkg.gdn_prefill(*a, kernel=kernel, **k))
    o, s = fn(*[d[x] for x in ARGS_P], use_qk_l2norm=True)
    sv = fused_views(d, (d["q"].shape[0],))
    out = strided_output(tuple(o.shape), cuda)
    o2, s2 = fn(*[sv[x] for x in ARGS_P], out, None, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert o2.data_ptr() == out.data_ptr()
    assert torch.equal(o2, o) and torch.equal(s2, s)
    ro, rs = oracle_prefill(inp, True)
    assert_parity(o2, s2, ro, rs, what=f"strided prefill {kernel}")
    assert pkg.device_error() == 0


def test_prefill_rows_not_16_byte_aligned(cuda):
    """Token rows 8 bytes longer than a multiple of 16: the tensor-core kernels read rows
    by TMA and need 16-byte rows.  Through the C ABI such views run the token-serial
    kernel (and an explicit tensor-core variant is refused); the Python entry point copies
    them into dense tensors first, so it gets the tensor-core result of the dense call."""
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs([33, 100], hq=4, hv=8, seed=92)
    d = to(inp, cuda)
    sv = fused_views(d, (d["q"].shape[0],), pad=4)
    assert sv["q"].stride(0) % 8 == 4
    T, N = d["q"].shape[0], 2
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device=cuda)
    ns = torch.empty(N, 8, 128, 128, device=cuda)

    wsb = pkg.LIB.gdn_prefill_workspace_size_variant(0, T, N, 4, 8, 128)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=cuda)

    def abi(variant):
        return pkg.LIB.gdn_prefill_launch_strided(
            variant, sv["q"].data_ptr(), sv["k"].data_ptr(), sv["v"].data_ptr(),
            d["state"].data_ptr(), d["A_log"].data_ptr(), sv["a"].data_ptr(),
            d["dt_bias"].data_ptr(), sv["b"].data_ptr(), d["cu_seqlens"].data_ptr(), 0,
            d["scale"], out.data_ptr(), ns.data_ptr(), T, N, 4, 4, 8, 128, 1,
            sv["q"].stride(0), sv["k"].stride(0), sv["v"].stride(0), sv["a"].stride(0),
            sv["b"].stride(0), out.stride(0), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream().cuda_stream)
    assert abi(0) == 0                                   # AUTO: token-serial kernel
    torch.cuda.synchronize()
    o_rec, s_rec = pkg.gdn_prefill_recurrent(*[d[x] for x in ARGS_P], use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert torch.equal(out, o_rec) and torch.equal(ns, s_rec)
    assert pkg.LIB.gdn_status_string(abi(2)) == b"GDN_ERR_UNSUPPORTED"  # FUSED refused
    o, s = pkg.gdn_prefill(*[sv[x] for x in ARGS_P], use_qk_l2norm=True, kernel="fused")
    o_d, s_d = pkg.gdn_prefill(*[d[x] for x in ARGS_P], use_qk_l2norm=True, kernel="fused")
    torch.cuda.synchronize()
    assert torch.equal(o, o_d) and torch.equal(s, s_d)


def test_prefill_other_layouts_are_copied(cuda):
    """A layout whose heads are not dense (here q with its two inner dims transposed in
    memory) is copied into a dense tensor first; non-dense output and new_state are
    written through temporaries."""
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs([64, 17], hq=2, hv=4, seed=93)
    d = to(inp, cuda)
    o, s = pkg.gdn_prefill(*[d[x] for x in ARGS_P], use_qk_l2norm=True)
    e = dict(d)
    e["q"] = d["q"].transpose(1, 2).contiguous().transpose(1, 2)
    assert not e["q"].is_contiguous()
    out = torch.empty(o.shape[1], o.shape[0], 128, dtype=torch.bfloat16,
                      device=cuda).transpose(0, 1)
    ns = torch.empty(s.shape[1], s.shape[0], 128, 128, device=cuda).transpose(0, 1)
    o2, s2 = pkg.gdn_prefill(*[e[x] for x in ARGS_P], out, ns, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert o2 is out and s2 is ns
    assert torch.equal(o2, o) and torch.equal(s2, s)


@pytest.mark.parametrize("batch", [3, 128])
def test_decode_fused_projection_views(cuda, batch):
    pkg = load_pkg()
    inp = pkg.workloads.decode_inputs(batch, seed=94)
    d = to(inp, cuda)
    o, s = pkg.gdn_decode(*[d[x] for x in ARGS_D], use_qk_l2norm=True)
    sv = fused_views(d, (batch, 1))
    out = strided_output(tuple(o.shape), cuda)
    o2, s2 = pkg.gdn_decode(*[sv[x] for x in ARGS_D], out, None, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert o2.data_ptr() == out.data_ptr()
    assert torch.equal(o2, o) and torch.equal(s2, s)
    ro, rs = oracle_decode(inp, True)
    assert_parity(o2, s2, ro, rs, what=f"strided decode B={batch}")


def test_decode_bf16_state_with_strided_views(cuda):
    """bf16 state: the strided views are copied into dense tensors (no strided bf16-state
    entry point); the result is the dense call's."""
    pkg = load_pkg()
    inp = pkg.workloads.decode_inputs(8, seed=95)
    inp["state"] = inp["state"].to(torch.bfloat16)
    d = to(inp, cuda)
    o, s = pkg.gdn_decode(*[d[x] for x in ARGS_D], use_qk_l2norm=True)
    sv = fused_views(d, (8, 1))
    o2, s2 = pkg.gdn_decode(*[sv[x] for x in ARGS_D], use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert torch.equal(o2, o) and torch.equal(s2, s)


def test_dps_kernel_entry_points_take_views(cuda):
    """The 11/12-parameter flashinfer-bench entry points accept the same views."""
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs([40, 3], hq=2, hv=4, seed=96)
    d = to(inp, cuda)
    o, s = pkg.prefill_kernel(*[d[x] for x in ARGS_P], torch.empty_like(d["v"]),
                              torch.empty_like(d["state"]))
    sv = fused_views(d, (d["q"].shape[0],))
    o2, s2 = pkg.prefill_kernel(*[sv[x] for x in ARGS_P], torch.empty_like(d["v"]),
                                torch.empty_like(d["state"]))
    torch.cuda.synchronize()
    assert torch.equal(o2, o) and torch.equal(s2, s)


def test_misaligned_first_elements_are_copied(cuda):
    """q/k/v views starting 2 bytes past an aligned address (a layout the kernels' vector
    loads cannot take): the Python entry points copy them into aligned dense tensors, so
    decode and prefill still give the dense calls' results."""
    pkg = load_pkg()

    def offset(t):
        buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=cuda)
        view = buf[1:].view(t.shape)
        view.copy_(t)
        assert view.data_ptr() % 4 == 2
        return view
    dinp = to(pkg.workloads.decode_inputs(5, hq=2, hv=4, seed=98), cuda)
    o, s = pkg.gdn_decode(*[dinp[x] for x in ARGS_D], use_qk_l2norm=True)
    e = dict(dinp, q=offset(dinp["q"]), k=offset(dinp["k"]), v=offset(dinp["v"]))
    o2, s2 = pkg.gdn_decode(*[e[x] for x in ARGS_D], use_qk_l2norm=True)
    pinp = to(pkg.workloads.prefill_inputs([70, 9], hq=2, hv=4, seed=99), cuda)
    po, ps = pkg.gdn_prefill(*[pinp[x] for x in ARGS_P], use_qk_l2norm=True)
    f = dict(pinp, q=offset(pinp["q"]), k=offset(pinp["k"]), v=offset(pinp["v"]))
    out = offset(torch.zeros_like(po))
    po2, ps2 = pkg.gdn_prefill(*[f[x] for x in ARGS_P], out, None, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert torch.equal(o2, o) and torch.equal(s2, s)
    assert po2 is out and torch.equal(po2, po) and torch.equal(ps2, ps)
