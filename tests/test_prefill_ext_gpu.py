"""GPU parity: prefill with precomputed gates and state checkpoints (the options of
FlashInfer's chunk_gated_delta_rule) on every prefill kernel family vs the CPU oracle."""
import pytest
import torch

from conftest import load_golden, load_pkg
from gpu_util import STATE_REL, assert_parity, to
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

KERNELS = ["auto", "split", "fused", "recurrent"]


def call(pkg, d, alpha, beta, l2, kernel, **kw):
    o, s = pkg.chunk_gated_delta_rule(d["q"], d["k"], d["v"], alpha, beta, d.get("scale"),
                                      d.get("state"), True, d["cu_seqlens"],
                                      use_qk_l2norm_in_kernel=l2, kernel=kernel, **kw)
    torch.cuda.synchronize()
    return o, s


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("name,l2", [("prefill_varlen_l2", True), ("prefill_nostate_raw", False)])
def test_precomputed_gates_reproduce_golden(cuda, name, l2, kernel):
    """alpha = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b) computed on the host
    and passed in: the definition-pinned golden outputs are reproduced."""
    pkg = load_pkg()
    d, m = load_golden(name)
    d["scale"] = float(m["scale"])
    g, beta = O.gates(d["A_log"], d["a"], d["dt_bias"], d["b"])
    dd = to(d, cuda)
    if kernel == "fused" and not l2:
        with pytest.raises(pkg.GDNError):
            call(pkg, dd, g.to(cuda), beta.to(cuda), l2, kernel)
        return
    o, s = call(pkg, dd, g.to(cuda), beta.to(cuda), l2, kernel)
    assert_parity(o, s, d["out"], d["new_state"], what=f"{name} {kernel}")


@pytest.mark.parametrize("kernel", ["split", "fused", "recurrent"])
def test_default_gates_are_ones(cuda, kernel):
    pkg = load_pkg()
    inp = pkg.workloads.prefill_inputs([70, 5, 129], hq=2, hv=4, seed=51)
    ro, rs, _ = O.prefill_gated(O.l2norm(inp["q"]), O.l2norm(inp["k"]), inp["v"], inp["state"],
                                None, None, inp["cu_seqlens"], inp["scale"])
    o, s = call(pkg, to(inp, cuda), None, None, True, kernel)
    assert_parity(o, s, ro, rs, what=f"ones {kernel}")


@pytest.mark.parametrize("kernel", ["split", "fused", "recurrent"])
@pytest.mark.parametrize("every", [64, 128])
def test_checkpoints_vs_oracle_and_capacity(cuda, kernel, every):
    pkg = load_pkg()
    lens = [64, 200, 0, 128, 300, 5]
    inp = pkg.workloads.prefill_inputs(lens, hq=2, hv=4, seed=52)
    g, beta = O.gates(inp["A_log"], inp["a"], inp["dt_bias"], inp["b"])
    ro, rs, rck = O.prefill_gated(O.l2norm(inp["q"]), O.l2norm(inp["k"]), inp["v"],
                                  inp["state"], g, beta, inp["cu_seqlens"], inp["scale"],
                                  checkpoint_every=every)
    counts = [n // every for n in lens]
    starts = torch.tensor([0] + list(torch.tensor(counts).cumsum(0).tolist()), dtype=torch.int64)
    total = int(starts[-1])
    d = to(inp, cuda)
    # one slot short: the last checkpoint must not be written (canary stays NaN)
    big = torch.full((total, 4, 128, 128), float("nan"), device=cuda)
    o, s = call(pkg, d, g.to(cuda), beta.to(cuda), True, kernel, state_checkpoints=big[:total - 1],
                checkpoint_cu_starts=starts.to(cuda), checkpoint_every_n_tokens=every)
    assert_parity(o, s, ro, rs, what=f"ckpt {kernel} {every}")
    ck = big.cpu()
    for i in range(total - 1):
        assert O.state_rel_err(ck[i], rck[i]) <= STATE_REL, (kernel, every, i)
    assert torch.isnan(ck[total - 1]).all()


def test_p2_checkpoints_equal_prefix_final_states_bitwise(cuda):
    """P2 (32768 tokens, initial state) with a checkpoint every 4096 tokens: checkpoint j
    equals, bit for bit, the final state of the same call on the first (j + 1) * 4096
    tokens (the chunked scan is deterministic and chunk-aligned)."""
    pkg = load_pkg()
    inp = pkg.workloads.prefill_config_inputs("P2", seed=0, device="cuda")
    g, beta = O.gates(inp["A_log"].cpu(), inp["a"].cpu(), inp["dt_bias"].cpu(), inp["b"].cpu())
    g, beta = g.cuda(), beta.cuda()
    ck = torch.empty(8, 32, 128, 128, device="cuda")
    starts = torch.tensor([0, 8], dtype=torch.int64, device="cuda")
    o, s = call(pkg, inp, g, beta, True, "auto", state_checkpoints=ck,
                checkpoint_cu_starts=starts, checkpoint_every_n_tokens=4096)
    assert torch.equal(ck[7], s[0])
    for j in (0, 3):
        n = (j + 1) * 4096
        sub = {"q": inp["q"][:n], "k": inp["k"][:n], "v": inp["v"][:n], "state": inp["state"],
               "scale": inp["scale"],
               "cu_seqlens": torch.tensor([0, n], dtype=torch.int32, device="cuda")}
        _, sj = call(pkg, sub, g[:n].contiguous(), beta[:n].contiguous(), True, "auto")
        assert torch.equal(ck[j], sj[0]), j
    assert pkg.device_error() == 0
