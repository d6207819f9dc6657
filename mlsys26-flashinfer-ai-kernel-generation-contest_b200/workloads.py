"""Seeded synthetic inputs for the GDN decode / prefill workloads.

The reference is benchmarked on flashinfer-bench dataset workloads (safetensors
blobs) that are not available offline; these generators stand in for them with
the shapes and value distributions of the configurations this package is
measured on:

* q, k, v ~ N(0, 1) bf16; a, b ~ N(0, 1) bf16
* state ~ N(0, 0.02^2) fp32 in k-last layout [.., HV, V=D, K=D]
* A_log = log(U(1, 16)) fp32 [HV]; dt_bias ~ N(0, 0.5^2) fp32 [HV]
* scale = 1/sqrt(D)

Draw order is fixed (prefill sequence lengths first, then q, k, v, state,
A_log, dt_bias, a, b) from one ``torch.Generator`` seeded with ``seed``, so a
given (config, seed) always produces the same tensors on the CPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

HQ = 16
HV = 32
D = 128


def _randn(shape, g, dtype, device, std=1.0):
    x = torch.randn(shape, generator=g, dtype=torch.float32, device=device)
    if std != 1.0:
        x.mul_(std)
    return x.to(dtype)


def decode_inputs(batch: int, *, hq: int = HQ, hv: int = HV, d: int = D, seed: int = 0,
                  with_state: bool = True, device: str = "cpu") -> Dict[str, torch.Tensor]:
    """Inputs of one decode step (seq_len 1).  Generated on ``device`` with a
    generator of that device (CPU values are the reproducible ones)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = {
        "q": _randn((batch, 1, hq, d), g, torch.bfloat16, device),
        "k": _randn((batch, 1, hq, d), g, torch.bfloat16, device),
        "v": _randn((batch, 1, hv, d), g, torch.bfloat16, device),
    }
    state = _randn((batch, hv, d, d), g, torch.float32, device, std=0.02)
    out["state"] = state if with_state else None
    u = torch.rand((hv,), generator=g, dtype=torch.float32, device=device)
    out["A_log"] = torch.log(1.0 + 15.0 * u)
    out["dt_bias"] = _randn((hv,), g, torch.float32, device, std=0.5)
    out["a"] = _randn((batch, 1, hv), g, torch.bfloat16, device)
    out["b"] = _randn((batch, 1, hv), g, torch.bfloat16, device)
    out["scale"] = 1.0 / math.sqrt(d)
    return out


def mtp_inputs(batch: int, seq_len: int, pool_size: int, *, hq: int = HQ, hv: int = HV,
               d: int = D, seed: int = 0, indices: Optional[Sequence[int]] = None,
               index_dtype: torch.dtype = torch.int32,
               device: str = "cpu") -> Dict[str, torch.Tensor]:
    """Inputs of one multi-token decode (speculative verification) call: T tokens per
    batch row and a k-last state pool [pool_size, HV, D, D].  ``indices`` maps batch rows
    to pool slots (default: a seeded permutation of distinct slots, pool_size >= batch)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = {
        "q": _randn((batch, seq_len, hq, d), g, torch.bfloat16, device),
        "k": _randn((batch, seq_len, hq, d), g, torch.bfloat16, device),
        "v": _randn((batch, seq_len, hv, d), g, torch.bfloat16, device),
        "state": _randn((pool_size, hv, d, d), g, torch.float32, device, std=0.02),
    }
    u = torch.rand((hv,), generator=g, dtype=torch.float32, device=device)
    out["A_log"] = torch.log(1.0 + 15.0 * u)
    out["dt_bias"] = _randn((hv,), g, torch.float32, device, std=0.5)
    out["a"] = _randn((batch, seq_len, hv), g, torch.bfloat16, device)
    out["b"] = _randn((batch, seq_len, hv), g, torch.bfloat16, device)
    if indices is None:
        if pool_size < batch:
            raise ValueError("default indices need pool_size >= batch")
        perm = torch.randperm(pool_size, generator=torch.Generator().manual_seed(seed + 1))
        indices = perm[:batch].tolist()
    out["state_indices"] = torch.tensor(list(indices), dtype=index_dtype).to(device)
    out["scale"] = 1.0 / math.sqrt(d)
    return out


def mtp_state_bytes(batch: int, seq_len: int, hv: int = HV, d: int = D,
                    intermediate: bool = False) -> int:
    """State bytes one multi-token decode call moves: each slot read and written once,
    plus one state write per token with the intermediate-state buffer."""
    per = hv * d * d * 4
    return batch * per * (2 + (seq_len if intermediate else 0))


def draw_seqlens(n: int, lo: int, hi: int, seed: int = 0) -> List[int]:
    """Sequence lengths ~ U[lo, hi] (inclusive), the first draw of a prefill config."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def prefill_inputs(seqlens: Sequence[int], *, hq: int = HQ, hv: int = HV, d: int = D,
                   seed: int = 0, with_state: bool = True, device: str = "cpu",
                   generator: Optional[torch.Generator] = None) -> Dict[str, torch.Tensor]:
    """Inputs of one varlen prefill call with the given sequence lengths."""
    g = generator or torch.Generator(device=device).manual_seed(seed)
    n = len(seqlens)
    t = int(sum(seqlens))
    cu = torch.zeros(n + 1, dtype=torch.int32)
    if n:
        cu[1:] = torch.tensor(list(seqlens), dtype=torch.int64).cumsum(0).to(torch.int32)
    out = {
        "q": _randn((t, hq, d), g, torch.bfloat16, device),
        "k": _randn((t, hq, d), g, torch.bfloat16, device),
        "v": _randn((t, hv, d), g, torch.bfloat16, device),
    }
    state = _randn((n, hv, d, d), g, torch.float32, device, std=0.02)
    out["state"] = state if with_state else None
    u = torch.rand((hv,), generator=g, dtype=torch.float32, device=device)
    out["A_log"] = torch.log(1.0 + 15.0 * u)
    out["dt_bias"] = _randn((hv,), g, torch.float32, device, std=0.5)
    out["a"] = _randn((t, hv), g, torch.bfloat16, device)
    out["b"] = _randn((t, hv), g, torch.bfloat16, device)
    out["cu_seqlens"] = cu.to(device)
    out["scale"] = 1.0 / math.sqrt(d)
    return out


@dataclass(frozen=True)
class PrefillConfig:
    name: str
    n: int
    lo: int
    hi: int
    with_state: bool


# The measured configurations (decode batch sizes; prefill sequence-length laws).
DECODE_CONFIGS = {"D1": 4, "D2": 128, "D3": 1024}
PREFILL_CONFIGS = {
    "P1": PrefillConfig("P1", 8, 256, 4096, False),
    "P2": PrefillConfig("P2", 1, 32768, 32768, True),
    "P3": PrefillConfig("P3", 64, 512, 8192, False),
}


def prefill_config_inputs(name: str, seed: int = 0, device: str = "cpu"):
    cfg = PREFILL_CONFIGS[name]
    lens = draw_seqlens(cfg.n, cfg.lo, cfg.hi, seed)
    g = torch.Generator(device=device).manual_seed(seed)
    if device == "cpu":
        # sequence lengths were the first draw of the same CPU stream
        torch.randint(cfg.lo, cfg.hi + 1, (cfg.n,), generator=g)
    return prefill_inputs(lens, seed=seed, with_state=cfg.with_state, device=device,
                          generator=g)


# Algorithmic work units (per-unit figures used for the rooflines).
def decode_state_bytes(batch: int, hv: int = HV, d: int = D) -> int:
    """State bytes one decode step must move: read + write of B*HV*D*D fp32."""
    return batch * hv * d * d * 4 * 2


def decode_io_bytes(batch: int, hq: int = HQ, hv: int = HV, d: int = D) -> int:
    """q, k, v, o (bf16) + a, b (bf16) per decode step."""
    return batch * ((2 * hq + 2 * hv) * d * 2 + 2 * hv * 2)


def prefill_flops_per_token(hq: int = HQ, hv: int = HV, d: int = D, chunk: int = 64) -> int:
    """GEMM FLOPs per token of the chunked form: HV*(6d^2 + 4Cd) + HQ*4Cd."""
    return hv * (6 * d * d + 4 * chunk * d) + hq * 4 * chunk * d
