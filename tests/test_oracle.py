"""CPU: the oracle reproduces the reference's golden vectors (no GPU needed)."""
import pytest
import torch

from conftest import load_golden
from oracle import gdn_oracle as O

pytestmark = pytest.mark.filterwarnings("ignore")


def test_decode_matches_definition_and_reference_triton():
    d, m = load_golden("decode_gva")
    o, s = O.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                    d["b"], m["scale"])
    # definition reference (flashinfer) -- fp32 on both sides
    assert O.state_rel_err(s, d["new_state"]) < 1e-6
    assert (s - d["new_state"]).abs().max().item() < 1e-5
    assert (o.float() - d["out"].float()).abs().max().item() <= 0.0 + 1e-6
    # the reference repository's own Triton kernel (run by the Triton interpreter)
    assert O.state_rel_err(s, d["new_state_triton"]) < 1e-6
    ok, frac, _, _ = O.flashinfer_allclose(o, d["out_triton"], 1e-2, 1e-2)
    assert ok and frac == 1.0


def test_decode_defaults_and_l2norm():
    d, m = load_golden("decode_nostate_l2")
    q = O.l2norm(d["q"])
    k = O.l2norm(d["k"])
    o, s = O.decode(q, k, d["v"], None, d["A_log"], d["a"], d["dt_bias"], d["b"], m["scale"])
    assert m["scale"] == 0.0  # exercised the 1/sqrt(D) default
    assert O.state_rel_err(s, d["new_state"]) < 1e-6
    assert (o.float() - d["out"].float()).abs().max().item() < 1e-6


def test_prefill_varlen_with_empty_sequence():
    d, m = load_golden("prefill_varlen_l2")
    o, s = O.prefill(O.l2norm(d["q"]), O.l2norm(d["k"]), d["v"], d["state"], d["A_log"], d["a"],
                     d["dt_bias"], d["b"], d["cu_seqlens"], m["scale"])
    assert O.state_rel_err(s, d["new_state"]) < 1e-6
    ok, frac, _, _ = O.flashinfer_allclose(o, d["out"], 1e-3, 1e-3)
    assert ok
    # the empty middle sequence leaves a zero state slice (definition semantics)
    assert d["cu_seqlens"][1] == d["cu_seqlens"][2]
    assert s[1].abs().max().item() == 0.0 and d["new_state"][1].abs().max().item() == 0.0


def test_prefill_zero_state_raw_qk():
    d, m = load_golden("prefill_nostate_raw")
    o, s = O.prefill(d["q"], d["k"], d["v"], None, d["A_log"], d["a"], d["dt_bias"], d["b"],
                     d["cu_seqlens"], None)
    assert O.state_rel_err(s, d["new_state"]) < 1e-5
    ok, _, _, _ = O.flashinfer_allclose(o, d["out"], 1e-2, 1e-2)
    assert ok


@pytest.mark.parametrize("name,l2,inter", [("mtp_gva_inter", False, True), ("mtp_l2", True, False)])
def test_mtp_matches_definition(name, l2, inter):
    """Multi-token decode (pool slots, rollback buffer) against _gdn_mtp_reference."""
    d, m = load_golden(name)
    q, k = (O.l2norm(d["q"]), O.l2norm(d["k"])) if l2 else (d["q"], d["k"])
    o, s, it = O.mtp(q, k, d["v"], d["state"], d["state_indices"], d["A_log"], d["a"],
                     d["dt_bias"], d["b"], float(m["scale"]), intermediate=inter)
    assert torch.equal(o, d["out"])
    assert O.state_rel_err(s, d["final_state"]) < 1e-6
    if inter:
        assert O.state_rel_err(it, d["intermediate"]) < 1e-6
        # slots no row references stay zero in the rollback buffer and initial in the pool
        assert it[1].abs().max().item() == 0.0
        assert torch.equal(s[1], d["state"][1])


def test_mtp_padding_rows_and_single_token_equals_decode():
    W = __import__("conftest").load_pkg().workloads
    inp = W.mtp_inputs(3, 1, 4, hq=1, hv=2, seed=21, indices=[2, -1, 7])
    o, s, _ = O.mtp(inp["q"], inp["k"], inp["v"], inp["state"], inp["state_indices"],
                    inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["scale"])
    assert o[1].abs().max().item() == 0.0 and o[2].abs().max().item() == 0.0
    assert torch.equal(s[[0, 1, 3]], inp["state"][[0, 1, 3]])  # padding rows touch nothing
    od, sd = O.decode(inp["q"][:1], inp["k"][:1], inp["v"][:1], inp["state"][2:3], inp["A_log"],
                      inp["a"][:1], inp["dt_bias"], inp["b"][:1], inp["scale"])
    assert torch.equal(o[:1], od) and torch.equal(s[2:3], sd)


def test_prefill_gated_and_checkpoints_restate_prefill():
    """Precomputed gates (the definition's g, beta) reproduce prefill exactly, and each
    checkpoint is the final state of the matching prefix."""
    W = __import__("conftest").load_pkg().workloads
    lens = [130, 0, 64, 70]
    inp = W.prefill_inputs(lens, hq=1, hv=2, seed=22)
    q, k = O.l2norm(inp["q"]), O.l2norm(inp["k"])
    o, s = O.prefill(q, k, inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                     inp["b"], inp["cu_seqlens"], inp["scale"])
    g, beta = O.gates(inp["A_log"], inp["a"], inp["dt_bias"], inp["b"])
    og, sg, ck = O.prefill_gated(q, k, inp["v"], inp["state"], g, beta, inp["cu_seqlens"],
                                 inp["scale"], checkpoint_every=64)
    assert torch.equal(o, og) and torch.equal(s, sg)
    assert ck.shape[0] == sum(n // 64 for n in lens) == 4
    # checkpoint 1 = state of sequence 0 after 128 tokens
    cu = torch.tensor([0, 128], dtype=torch.int32)
    _, s128 = O.prefill(q[:128], k[:128], inp["v"][:128], inp["state"][:1], inp["A_log"],
                        inp["a"][:128], inp["dt_bias"], inp["b"][:128], cu, inp["scale"])
    assert torch.equal(ck[1], s128[0])
    _, _, none_ck = O.prefill_gated(q, k, inp["v"], None, None, None, inp["cu_seqlens"], 0.0)
    assert none_ck is None


def test_oracle_fp32_vs_fp64():
    """The fp32 oracle is itself accurate: compare with its float64 evaluation."""
    d, m = load_golden("prefill_varlen_l2")
    args = (O.l2norm(d["q"]), O.l2norm(d["k"]), d["v"], d["state"], d["A_log"], d["a"],
            d["dt_bias"], d["b"], d["cu_seqlens"], m["scale"])
    o32, s32 = O.prefill(*args)
    o64, s64 = O.prefill(*args, dtype=torch.float64)
    assert O.state_rel_err(s32, s64) < 1e-6


def test_tolerance_rule_semantics():
    """flashinfer rule: fail only if BOTH abs and rel error exceed their bounds."""
    ref = torch.tensor([1.0, 100.0, 0.001])
    act = torch.tensor([1.015, 101.0, 0.0105])
    ok, frac, _, _ = O.flashinfer_allclose(act, ref, 1e-2, 1e-2)
    # 1.015: abs .015>.01 and rel .015>.01 -> fail; 101: rel .01 ok; .0105: abs ok
    assert not ok and abs(frac - 2 / 3) < 1e-6


def test_planted_mistake_is_caught():
    """A deliberately wrong gate (planted in a copy of the oracle's inputs) fails the check."""
    d, m = load_golden("decode_gva")
    wrong_dt = d["dt_bias"] + 0.5
    o, s = O.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], wrong_dt, d["b"],
                    m["scale"])
    assert O.state_rel_err(s, d["new_state"]) > 1e-3
