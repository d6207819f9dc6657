"""Benchmark of the GDN decode / prefill hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode_b128|decode_b4|decode_b1024|prefill_p1|prefill_p2|prefill_p3|
                                mtp_b128_t4|decode_b128_bf16state]

Prints ONE JSON line (rank 0).  Default workload: one GDN decode step over
batch 128 (state 128 x 32 x 128 x 128 fp32 = 268 MB read + 268 MB written per
step), the single-GPU configuration the headline metric is quoted on.  The
line also carries a ``prefill`` object with the P1 (8 varlen sequences) and P2
(one 32768-token sequence) prefill measurements.

N > 1 (torchrun, one process per GPU): weak scaling -- every rank runs the
same per-GPU workload on its own data (decode: 128 sequences per GPU, so N=8
is the 1024-sequence configuration sharded by batch); the prefill extras are
strong scaling: P2 (one sequence) and P3 (64 sequences) sharded by q/k-head
group, with P3 by sequence (longest-first packing) and P2 by the token-segment
scan (its one all-gather) as separate lines.  Decode has
no collective on the data path.  Time is the max over ranks of the device time.

Timing: W untimed warm-up steps, then exactly K steps between CUDA events on
the launching stream, barrier + synchronize on both sides.  Inputs are larger
than L2 (126 MB) and decode ping-pongs its state between two buffers.
``--impl reference`` times the CPU restatement of the reference's algorithm
(the oracle port; the reference itself is Triton-only and has no CPU path) on
the host's cores, on the same workload, metric, config and step count, with
the flashinfer-bench definition reference timed beside it on a small sample;
it never imports the package or loads its CUDA library.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
PKG_NAME = "mlsys26-flashinfer-ai-kernel-generation-contest_b200"
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
E2E_SLICES = 8  # batch slices of the pipelined end-to-end decode step
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# --------------------------------------------------------------------------- helpers
def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def ncu_traffic(workload: str):
    """Per-launch DRAM bytes (read + write) of the dominant kernel from the committed
    ncu summary (profiles/ncu_traffic.txt: lines 'workload bytes ...')."""
    p = REPO / "profiles" / "ncu_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == workload and not line.startswith("#"):
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons = [], set()
        self.period = period_s
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            # map the torch device to its NVML handle through the GPU UUID
            self.h = None
            uuid = getattr(torch.cuda.get_device_properties(device_index), "uuid", None)
            if uuid is not None:
                try:
                    self.h = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}".encode())
                except Exception:
                    self.h = None
            if self.h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[device_index]) if vis else device_index
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _sample(self):
        nv = self.nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        try:
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        for bit, name in self.REASONS.items():
            if r & bit:
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        busy = [s for s in self.samples if s > 0]
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend="nccl", timeout_s=120):
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            if backend == "nccl":
                torch.cuda.set_device(self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
            self.pg = dist

    def barrier(self):
        if self.pg:
            if torch.cuda.is_available() and self.pg.get_backend() == "nccl":
                self.pg.barrier(device_ids=[self.local])
            else:
                self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        dev = torch.device("cuda", self.local) if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# --------------------------------------------------------------------------- workloads
class DecodeWork:
    """One decode step over `batch` sequences; state ping-pongs between two buffers
    (fp32, or bf16 with `state_bf16`)."""

    def __init__(self, pkg, batch, dev, seed, state_bf16=False):
        W = pkg.workloads
        self.pkg, self.batch, self.dev = pkg, batch, dev
        inp = W.decode_inputs(batch, seed=seed, device=str(dev))
        if state_bf16:
            inp["state"] = inp["state"].to(torch.bfloat16)
        self.inp = inp
        self.s = [inp["state"], torch.empty_like(inp["state"])]
        self.out = torch.empty_like(inp["v"])
        self.i = 0
        # algorithmic bytes per step (state read + write)
        self.units = W.decode_state_bytes(batch) // (2 if state_bf16 else 1)
        self.io_bytes = W.decode_io_bytes(batch)
        self.launches = 1

    def step(self):
        d = self.inp
        src, dst = self.s[self.i], self.s[1 - self.i]
        self.pkg.gdn_decode(d["q"], d["k"], d["v"], src, d["A_log"], d["a"], d["dt_bias"],
                            d["b"], d["scale"], self.out, dst, use_qk_l2norm=True)
        self.i ^= 1

    def host_copies(self):
        """Pinned host copies for the end-to-end leg."""
        d = self.inp
        self.h = {k: d[k].cpu().pin_memory() for k in ("q", "k", "v", "state", "a", "b")}
        self.h_out = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h_ns = torch.empty(d["state"].shape, dtype=d["state"].dtype).pin_memory()
        self.d_in = {k: torch.empty_like(d[k]) for k in self.h}
        self.d_ns = torch.empty_like(d["state"])
        h2d = sum(t.numel() * t.element_size() for t in self.h.values())
        d2h = self.h_out.numel() * 2 + self.h_ns.numel() * self.h_ns.element_size()
        return h2d, d2h

    def e2e_step(self):
        """Host inputs -> device -> the C-ABI entry point (gdn_decode_launch, same flags as
        the device-timed step) -> host outputs, pipelined over slices of the batch: slice
        i + 1 goes up while slice i is computed and slice i - 1 comes back (PCIe is full
        duplex), on two copy streams besides the compute stream."""
        cur = torch.cuda.current_stream()
        if not hasattr(self, "s_up"):
            self.s_up, self.s_down = torch.cuda.Stream(), torch.cuda.Stream()
        n = E2E_SLICES if self.batch % E2E_SLICES == 0 else 1
        n = getattr(self, "slices", n)
        rows = self.batch // n
        di, d = self.d_in, self.inp
        self.s_up.wait_stream(cur)  # inputs of the previous step are consumed
        for i in range(n):
            sl = slice(i * rows, (i + 1) * rows)
            with torch.cuda.stream(self.s_up):
                for k_, t in self.h.items():
                    di[k_][sl].copy_(t[sl], non_blocking=True)
            cur.wait_stream(self.s_up)
            self.pkg.gdn_decode(di["q"][sl], di["k"][sl], di["v"][sl], di["state"][sl],
                                d["A_log"], di["a"][sl], d["dt_bias"], di["b"][sl], d["scale"],
                                self.out[sl], self.d_ns[sl], use_qk_l2norm=True)
            self.s_down.wait_stream(cur)
            with torch.cuda.stream(self.s_down):
                self.h_out[sl].copy_(self.out[sl], non_blocking=True)
                self.h_ns[sl].copy_(self.d_ns[sl], non_blocking=True)
        cur.wait_stream(self.s_down)  # the step ends when its results are on the host


class MtpWork:
    """One multi-token decode call: `batch` rows of MTP_T draft tokens against a resident
    state pool (one slot per row, updated in place), with the rollback buffer that
    receives the state after every token."""

    def __init__(self, pkg, batch, dev, seed):
        W = pkg.workloads
        self.pkg, self.batch, self.dev = pkg, batch, dev
        self.inp = W.mtp_inputs(batch, MTP_T, batch, seed=seed, device=str(dev))
        d = self.inp
        self.inter = torch.empty((batch, MTP_T) + tuple(d["state"].shape[1:]),
                                 dtype=torch.float32, device=dev)
        self.out = torch.empty_like(d["v"])
        self.units = W.mtp_state_bytes(batch, MTP_T, intermediate=True)
        self.launches = 1

    def step(self):
        d = self.inp
        self.pkg.gdn_mtp(d["q"], d["k"], d["v"], d["state"], d["state_indices"], d["A_log"],
                         d["a"], d["dt_bias"], d["b"], d["scale"], self.out, None, self.inter,
                         use_qk_l2norm=True)

    def host_copies(self):
        d = self.inp
        keys = ("q", "k", "v", "state", "state_indices", "a", "b")
        self.h = {k_: d[k_].cpu().pin_memory() for k_ in keys}
        self.d_in = {k_: torch.empty_like(d[k_]) for k_ in keys}
        self.h_out = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h_state = torch.empty(d["state"].shape, dtype=torch.float32).pin_memory()
        self.h_inter = torch.empty(self.inter.shape, dtype=torch.float32).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in self.h.values())
        d2h = (self.h_out.numel() * 2 + self.h_state.numel() * 4 + self.h_inter.numel() * 4)
        return h2d, d2h

    def e2e_step(self):
        """Host inputs and pool -> device -> gdn_mtp_launch -> output, pool and rollback
        buffer back to the host."""
        di = self.d_in
        for k_, t in self.h.items():
            di[k_].copy_(t, non_blocking=True)
        d = self.inp
        self.pkg.gdn_mtp(di["q"], di["k"], di["v"], di["state"], di["state_indices"],
                         d["A_log"], di["a"], d["dt_bias"], di["b"], d["scale"], self.out, None,
                         self.inter, use_qk_l2norm=True)
        self.h_out.copy_(self.out, non_blocking=True)
        self.h_state.copy_(di["state"], non_blocking=True)
        self.h_inter.copy_(self.inter, non_blocking=True)


MTP_T = 4  # draft tokens verified per row (speculative decoding)


def plan_kind(W, name, world, force="auto"):
    """How prefill config `name` is split over `world` GPUs: None (one GPU), "heads" (every
    GPU runs all sequences for its q/k-head group and the v-heads that read them), "seqs"
    (whole sequences, longest-first packing) or "segments" (one sequence as consecutive
    token segments chained through their state maps, one all-gather per call).  Neither of
    the first two has a collective.  The default is head groups whenever the q/k heads
    divide evenly: every GPU then gets the same mix of sequence lengths, so the ranks
    finish together (P3, each rank's share timed on one B200: 0.797 ms at N = 8 against
    0.853 ms for sequence packing).  `force` picks "heads", "seqs" or "segments" (one
    sequence only) instead."""
    if world == 1:
        return None
    cfg = W.PREFILL_CONFIGS[name]
    if force == "segments" and cfg.n == 1:
        return "segments"
    if force == "seqs" and cfg.n >= world:
        return "seqs"
    if force == "heads" or W.HQ % world == 0 or cfg.n < world:
        return "heads"
    return "seqs"


def prefill_plan(pkg, name, dist, force="auto"):
    """This rank's part of prefill config `name` (see plan_kind)."""
    W = pkg.workloads
    kind = plan_kind(W, name, dist.world, force)
    if kind is None:
        return None
    if kind == "seqs":
        cfg = W.PREFILL_CONFIGS[name]
        lens = W.draw_seqlens(cfg.n, cfg.lo, cfg.hi, 0)
        return ("seqs", pkg.sharding.lpt_assign(lens, dist.world)[dist.rank])
    if kind == "segments":
        return ("segments", dist.world, dist.rank)
    return ("heads",) + tuple(pkg.sharding.head_range(W.HQ, dist.world, dist.rank))


def plan_text(plan, world):
    kind = plan if (plan is None or isinstance(plan, str)) else plan[0]
    if kind is None:
        return "single GPU"
    if kind == "seqs":
        return f"sequence-sharded x{world} (LPT), no collective"
    if kind == "segments":
        return (f"token-segment scan x{world} (one all-gather of the segments' state maps per "
                f"call: departs from the no-collective v-head plan)")
    return f"q/k-head-group-sharded x{world}, no collective"


class PrefillWork:
    def __init__(self, pkg, cfg_name, dev, seed, shard=None, dist=None):
        W = pkg.workloads
        self.pkg, self.dev = pkg, dev
        inp = W.prefill_config_inputs(cfg_name, seed=seed, device="cpu")
        self.segments = shard is not None and shard[0] == "segments"
        self.local_segments = 1
        if self.segments:
            self._init_segment(inp, shard[1], shard[2], dist)
            return
        head_frac = 1.0
        if shard is not None and shard[0] == "seqs":  # this rank's sequences, re-packed
            inp = pkg.sharding.prefill_shard(inp, shard[1])
        elif shard is not None:  # this rank's q/k heads and their v-heads
            inp = pkg.sharding.prefill_head_shard(inp, shard[1], shard[2])
            head_frac = inp["v"].shape[1] / W.HV
        lens = pkg.sharding.seqlens_from_cu(inp["cu_seqlens"])
        self.lens = lens
        self.inp = {k_: (v_.to(dev) if isinstance(v_, torch.Tensor) else v_) for k_, v_ in inp.items()}
        self.cpu_inp = inp
        T = self.inp["q"].shape[0]
        N = len(lens)
        # one sequence whose v-heads leave most SMs idle (a head group of a multi-GPU plan):
        # its token segments run side by side in one call (gdn_prefill_segmented)
        self.local_segments = pkg.prefill.segments_auto(T, self.inp["v"].shape[1]) \
            if (shard is not None and N == 1) else 1
        self.out = torch.empty(T, self.inp["v"].shape[1], 128, dtype=torch.bfloat16, device=dev)
        self.ns = torch.empty(N, self.inp["v"].shape[1], 128, 128, dtype=torch.float32, device=dev)
        # whole-sequence tokens this rank completes (a head group does a share of each)
        self.tokens = T * head_frac
        self.flops = T * W.prefill_flops_per_token(inp["q"].shape[1], inp["v"].shape[1])
        self.launches = pkg.prefill.launches_per_call(T, N, self.inp["q"].shape[1], self.inp["v"].shape[1])
        if self.local_segments > 1:  # the call of 2 S - 1 runs, one chain pass, one output pass
            self.launches = pkg.prefill.segmented_launches(self.local_segments)

    def _init_segment(self, inp, world, rank, dist):
        """Segment `rank` of the single sequence.  Rank 0 runs it from the initial state;
        every other rank runs, in one call of two sequences, the segment from the identity
        with v = 0 and from a zero state (its state map A, B and the two runs' outputs: the
        doubled input is a layout prepared once), then, after the all-gather of every
        rank's (A, B), assembles its outputs and final state from its chained start state
        with fp32 matrix products."""
        S, W = self.pkg.sharding, self.pkg.workloads
        self.world, self.rank, self.dist = world, rank, dist
        lo, hi = S.segment_bounds(inp["q"].shape[0], world)[rank]
        seg = S.segment_inputs(inp, lo, hi)
        L, HQ, HV = hi - lo, inp["q"].shape[1], inp["v"].shape[1]
        dev = self.dev
        self.inp = {k_: (v_.to(dev) if isinstance(v_, torch.Tensor) else v_)
                    for k_, v_ in seg.items()}
        if rank == 0:
            if self.inp.get("state") is None:
                self.inp["state"] = torch.zeros(1, HV, 128, 128, device=dev)
        else:
            eye = torch.eye(128).expand(1, HV, 128, 128)
            dbl = dict(seg)
            for key in ("q", "k", "a", "b"):
                dbl[key] = torch.cat([seg[key], seg[key]], dim=0)
            dbl["v"] = torch.cat([torch.zeros_like(seg["v"]), seg["v"]], dim=0)
            dbl["state"] = torch.cat([eye, torch.zeros(1, HV, 128, 128)], dim=0).contiguous()
            dbl["cu_seqlens"] = torch.tensor([0, L, 2 * L], dtype=seg["cu_seqlens"].dtype)
            self.dbl = {k_: (v_.to(dev) if isinstance(v_, torch.Tensor) else v_)
                        for k_, v_ in dbl.items()}
            self.dbl_out = torch.empty(2 * L, HV, 128, dtype=torch.bfloat16, device=dev)
            self.dbl_ns = torch.empty(2, HV, 128, 128, device=dev)
        self.out = torch.empty(L, HV, 128, dtype=torch.bfloat16, device=dev)
        self.ns = torch.empty(1, HV, 128, 128, device=dev)
        self.A = torch.zeros(1, HV, 128, 128, device=dev)
        self.maps = torch.empty(world, 2, HV, 128, 128, device=dev)
        self.lens = [L]
        self.cpu_inp = seg
        self.tokens = L
        self.flops = L * W.prefill_flops_per_token(HQ, HV)
        per = self.pkg.prefill.launches_per_call
        # rank > 0: the two-sequence call, then the chain and output kernels
        self.launches = per(L, 1, HQ, HV) if rank == 0 else per(2 * L, 2, HQ, HV) + 2

    def _segment_step(self, d):
        P = self.pkg
        if self.rank == 0:
            P.gdn_prefill(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                          d["b"], d["cu_seqlens"], d["scale"], self.out, self.ns,
                          use_qk_l2norm=True)
            mine = torch.cat([self.A, self.ns], dim=0)
        else:
            e = self.dbl
            P.gdn_prefill(e["q"], e["k"], e["v"], e["state"], e["A_log"], e["a"], e["dt_bias"],
                          e["b"], e["cu_seqlens"], e["scale"], self.dbl_out, self.dbl_ns,
                          use_qk_l2norm=True)
            mine = self.dbl_ns
        self.dist.pg.all_gather_into_tensor(self.maps, mine)
        if self.rank > 0:
            L = self.out.shape[0]
            self.pkg.sharding.segment_assemble(self.maps, self.rank, self.dbl_out[:L],
                                               self.dbl_out[L:], out=self.out, final=self.ns)

    def _call(self, d):
        if self.local_segments > 1:
            self.pkg.gdn_prefill_segmented(d["q"], d["k"], d["v"], d.get("state"), d["A_log"],
                                           d["a"], d["dt_bias"], d["b"], d["scale"], self.out,
                                           self.ns, use_qk_l2norm=True)  # the library's plan
            return
        self.pkg.gdn_prefill(d["q"], d["k"], d["v"], d.get("state"), d["A_log"], d["a"],
                             d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"], self.out, self.ns,
                             use_qk_l2norm=True)

    def step(self):
        d = self.inp
        if self.segments:
            self._segment_step(d)
            return
        self._call(d)

    def host_copies(self):
        d = self.inp
        keys = [k_ for k_ in ("q", "k", "v", "state", "a", "b", "cu_seqlens") if d[k_] is not None]
        self.h = {k_: d[k_].cpu().pin_memory() for k_ in keys}
        self.d_in = {k_: torch.empty_like(d[k_]) for k_ in keys}
        self.h_out = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h_ns = torch.empty(self.ns.shape, dtype=torch.float32).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in self.h.values())
        d2h = self.h_out.numel() * 2 + self.h_ns.numel() * 4
        return h2d, d2h

    def e2e_step(self):
        """Host inputs -> device -> the C-ABI entry point (gdn_prefill_launch, same flags as
        the device-timed step) -> host outputs."""
        di = self.d_in
        for k_, t in self.h.items():
            di[k_].copy_(t, non_blocking=True)
        d = self.inp
        if self.segments:  # the segment's inputs, duplicated on the device for the maps
            if self.rank > 0:
                L = di["q"].shape[0]
                for key in ("q", "k", "a", "b"):
                    self.dbl[key][:L].copy_(di[key])
                    self.dbl[key][L:].copy_(di[key])
                self.dbl["v"][L:].copy_(di["v"])
            self._segment_step({**d, **di})
            self.h_out.copy_(self.out, non_blocking=True)
            self.h_ns.copy_(self.ns, non_blocking=True)
            return
        self._call({**d, **di})
        self.h_out.copy_(self.out, non_blocking=True)
        self.h_ns.copy_(self.ns, non_blocking=True)


# --------------------------------------------------------------------------- timing
def time_steps(fn, steps, warmup, dist, per_launch_events=True, flush=None):
    """Returns (max-over-ranks ms per step, mean kernel ms per step on this rank).
    With `flush` (workloads smaller than L2), L2 is flushed before every step outside the
    per-step events, and the step time is the mean of those events (max over ranks)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    per_launch_events = per_launch_events or flush is not None
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)] if per_launch_events else []
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        if flush is not None:
            flush()
        if per_launch_events:
            ev[i][0].record(stream)
        fn()
        if per_launch_events:
            ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    total = t0.elapsed_time(t1)
    per_kernel = (sum(a.elapsed_time(b) for a, b in ev) / steps) if ev else total / steps
    if flush is not None:
        return dist.max(per_kernel * steps) / steps, per_kernel
    return dist.max(total) / steps, per_kernel


def graph_steps(work, n_graphs):
    """CUDA graphs of `n_graphs` consecutive steps of `work`, one step per graph (decode
    ping-pongs its state between two buffers, so two graphs alternate), replayed in turn:
    the way a serving loop launches decode, without the Python wrapper's host time between
    kernels.  Returns the replay function and the graphs (kept alive by the caller)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # first calls (one-time kernel configuration) off capture
        for _ in range(n_graphs):
            work.step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graphs = []
    for _ in range(n_graphs):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            work.step()
        graphs.append(g)
    turn = [0]

    def replay():
        graphs[turn[0]].replay()
        turn[0] = (turn[0] + 1) % n_graphs
    return replay, graphs


_CPU_MODS = None


def cpu_modules():
    """(workloads, oracle) for the CPU legs, loaded from their files without importing the
    package: the package's import maps the CUDA library, which a CPU arm must not load."""
    global _CPU_MODS
    if _CPU_MODS is None:
        import importlib.util
        spec = importlib.util.spec_from_file_location("_gdn_bench_workloads",
                                                      REPO / PKG_NAME / "workloads.py")
        W = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = W
        spec.loader.exec_module(W)
        from oracle import gdn_oracle as O
        _CPU_MODS = (W, O)
    return _CPU_MODS


def host_threads():
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return n


def cpu_decode_step(batch, seed=0, state_bf16=False):
    """One full decode step of the oracle port on the host, as a callable (inputs built
    once); returns (step, state bytes per step)."""
    W, O = cpu_modules()
    inp = W.decode_inputs(batch, seed=seed)
    if state_bf16:
        inp["state"] = inp["state"].to(torch.bfloat16)
    q, k = O.l2norm(inp["q"]), O.l2norm(inp["k"])

    def step():
        O.decode(q, k, inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                 inp["scale"])
    return step, W.decode_state_bytes(batch) // (2 if state_bf16 else 1)


def cpu_mtp_step(rows, seed=0):
    W, O = cpu_modules()
    inp = W.mtp_inputs(rows, MTP_T, rows, seed=seed)
    q, k = O.l2norm(inp["q"]), O.l2norm(inp["k"])

    def step():
        O.mtp(q, k, inp["v"], inp["state"], inp["state_indices"], inp["A_log"], inp["a"],
              inp["dt_bias"], inp["b"], inp["scale"], intermediate=True)
    return step, W.mtp_state_bytes(rows, MTP_T, intermediate=True)


def cpu_prefill_step(cfg_name, budget_tokens):
    """The oracle port's prefill over the first `budget_tokens` tokens of config
    `cfg_name` (its first sequences, the last one cut), as a callable; returns (step,
    tokens per step, sample text)."""
    W, O = cpu_modules()
    inp = W.prefill_config_inputs(cfg_name, seed=0)
    cu = inp["cu_seqlens"].tolist()
    n = 1
    while n < len(cu) - 1 and cu[n] < budget_tokens:
        n += 1
    T = min(cu[n], budget_tokens)
    sub_cu = torch.tensor([min(c, T) for c in cu[:n + 1]], dtype=torch.int32)
    st = inp["state"][:n] if inp["state"] is not None else None
    q, k = O.l2norm(inp["q"][:T]), O.l2norm(inp["k"][:T])

    def step():
        O.prefill(q, k, inp["v"][:T], st, inp["A_log"], inp["a"][:T], inp["dt_bias"],
                  inp["b"][:T], sub_cu, inp["scale"])
    return step, T, f"first {T} tokens of {cfg_name} ({n} sequence(s))"


def timed_cpu(step, steps, warmup):
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    return (time.perf_counter() - t0) / steps


def definition_baseline(kind, param):
    """The flashinfer-bench definition reference itself (`_gdn_decode_reference` /
    `_gdn_prefill_reference`, the Python loops the contest's speedups divide by) on a
    bounded sample, fed host-normalised q/k like the oracle.  None when it cannot be
    imported."""
    try:
        from flashinfer.trace.templates.gdn import (_gdn_decode_reference,
                                                    _gdn_prefill_reference)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    W, O = cpu_modules()
    threads = host_threads()
    if kind in ("decode", "decode_bf16state", "mtp"):
        rows = 8
        inp = W.decode_inputs(rows, seed=0)
        q, k = O.l2norm(inp["q"]), O.l2norm(inp["k"])
        args = (q, k, inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                inp["scale"])
        per = timed_cpu(lambda: _gdn_decode_reference(*args), 2, 1)
        return {"value": W.decode_state_bytes(rows) / per / 1e9, "unit": "GB/s",
                "cores": threads, "kind": "definition",
                "sample": f"one fp32 decode step of {rows} rows (flashinfer-bench definition "
                          f"_gdn_decode_reference)"}
    tokens = 128
    inp = W.prefill_inputs([tokens], seed=0)
    q, k = O.l2norm(inp["q"]), O.l2norm(inp["k"])
    args = (q, k, inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
            inp["cu_seqlens"], inp["scale"])
    per = timed_cpu(lambda: _gdn_prefill_reference(*args), 1, 1)
    return {"value": tokens / per, "unit": "tokens/s", "cores": threads, "kind": "definition",
            "sample": f"{tokens} tokens of one sequence (flashinfer-bench definition "
                      f"_gdn_prefill_reference)"}


def cpu_baseline(kind, param, budget_s=10.0):
    """The oracle port on the host cores, bounded sample (rank 0, N = 1 only)."""
    threads = host_threads()
    if kind in ("decode", "decode_bf16state"):
        step, units = cpu_decode_step(param, state_bf16=kind == "decode_bf16state")
        reps = max(1, min(5, int(budget_s / max(timed_cpu(step, 1, 0), 1e-3))))
        per = timed_cpu(step, reps, 0)
        res = {"value": units / per / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{reps} full decode step(s) of batch {param} (oracle, fp32 torch CPU)"}
    elif kind == "mtp":
        rows = min(param, 16)
        step, units = cpu_mtp_step(rows)
        per = timed_cpu(step, 2, 1)
        res = {"value": units / per / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{rows} rows x {MTP_T} tokens of the same workload (oracle, fp32 "
                         f"torch CPU)"}
    else:
        step, T, sample = cpu_prefill_step(param, 4096)
        per = timed_cpu(step, 1, 0)
        res = {"value": T / per, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": sample + " (oracle, fp32 torch CPU)"}
    res["definition"] = definition_baseline(kind, param)
    return res


# --------------------------------------------------------------------------- arms
def l2_flusher(units, dev):
    """None when a step moves more than L2 holds; else a function that overwrites L2."""
    if units > L2_BYTES:
        return None
    buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    return lambda: buf.fill_(1.0)


def copy_reference(units, dev, reps=20):
    """GB/s of a device-to-device copy that moves the same bytes as one step (units / 2
    read, units / 2 written; two buffer pairs alternate so the source is not in L2): the
    HBM rate a plain copy reaches at this size, beside the roofline's fixed denominator."""
    n = max(1, units // 2 // 4)
    bufs = [(torch.ones(n, device=dev), torch.empty(n, device=dev)) for _ in range(2)]
    for i in range(4):
        bufs[i & 1][1].copy_(bufs[i & 1][0])
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(reps):
        bufs[i & 1][1].copy_(bufs[i & 1][0])
    t1.record()
    torch.cuda.synchronize()
    return 2 * n * 4 * reps / (t0.elapsed_time(t1) * 1e-3) / 1e9


def pcie_reference(h2d, d2h, dev, reps=3):
    """GB/s (both directions together) of one pinned host->device copy of `h2d` bytes
    running beside one device->host copy of `d2h` bytes on a second stream: the PCIe rate
    the end-to-end step's copies can reach, beside its measured rate."""
    hu = torch.empty(max(1, h2d), dtype=torch.uint8).pin_memory()
    hd = torch.empty(max(1, d2h), dtype=torch.uint8).pin_memory()
    du = torch.empty(hu.numel(), dtype=torch.uint8, device=dev)
    dd = torch.empty(hd.numel(), dtype=torch.uint8, device=dev)
    s_up, s_dn = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def both():
        with torch.cuda.stream(s_up):
            du.copy_(hu, non_blocking=True)
        with torch.cuda.stream(s_dn):
            hd.copy_(dd, non_blocking=True)
    both()
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        both()
    torch.cuda.synchronize()
    return (h2d + d2h) * reps / (time.perf_counter() - t) / 1e9


def measure_decode(pkg, dist, batch, steps, warmup, dev, with_e2e=True, state_bf16=False,
                   graphs=True, e2e_slices=0):
    w = DecodeWork(pkg, batch, dev, seed=dist.rank, state_bf16=state_bf16)
    if e2e_slices > 0 and batch % e2e_slices == 0:
        w.slices = e2e_slices
    fn, keep = graph_steps(w, 2) if graphs else (w.step, None)
    flush = l2_flusher(w.units, dev)
    with ClockSampler(dev.index) as clk:
        ms, kern_ms = time_steps(fn, steps, warmup, dist, flush=flush)
    del keep
    total_bytes = w.units * dist.world
    res = {"ms": ms, "kern_ms": kern_ms, "value": total_bytes / (ms * 1e-3) / 1e9,
           "achieved": w.units / (kern_ms * 1e-3) / 1e9, "clocks": clk.summary(),
           "launches": w.launches * steps, "units": w.units}
    if with_e2e:
        h2d, d2h = w.host_copies()
        e2e_steps = max(3, min(steps, 20))
        e_ms, _ = time_steps(w.e2e_step, e2e_steps, 2, dist, per_launch_events=False)
        pcie = pcie_reference(h2d, d2h, dev)
        res["e2e"] = {"value": total_bytes / (e_ms * 1e-3) / 1e9, "unit": "GB/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "ms_per_step": e_ms, "steps": e2e_steps,
                      "pcie_same_bytes_gbs": round(pcie, 1),
                      "frac_of_pcie": round((h2d + d2h) / (e_ms * 1e-3) / 1e9 / pcie, 4)}
    return res


def measure_mtp(pkg, dist, batch, steps, warmup, dev, with_e2e=True, graphs=True):
    w = MtpWork(pkg, batch, dev, seed=dist.rank)
    fn, keep = graph_steps(w, 1) if graphs else (w.step, None)
    flush = l2_flusher(w.units, dev)
    with ClockSampler(dev.index) as clk:
        ms, kern_ms = time_steps(fn, steps, warmup, dist, flush=flush)
    del keep
    total_bytes = w.units * dist.world
    res = {"ms": ms, "kern_ms": kern_ms, "value": total_bytes / (ms * 1e-3) / 1e9,
           "achieved": w.units / (kern_ms * 1e-3) / 1e9, "clocks": clk.summary(),
           "launches": w.launches * steps, "units": w.units}
    if with_e2e:
        h2d, d2h = w.host_copies()
        e2e_steps = max(3, min(steps, 10))
        e_ms, _ = time_steps(w.e2e_step, e2e_steps, 2, dist, per_launch_events=False)
        res["e2e"] = {"value": total_bytes / (e_ms * 1e-3) / 1e9, "unit": "GB/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "ms_per_step": e_ms, "steps": e2e_steps}
    return res


def measure_prefill(pkg, dist, cfg_name, steps, warmup, dev, shard=None, with_e2e=True,
                    graphs=True):
    w = PrefillWork(pkg, cfg_name, dev, seed=0, shard=shard, dist=dist)
    # replayed from a CUDA graph like decode (the cross-GPU segment scan, whose step holds
    # an NCCL all-gather, runs eagerly)
    fn, keep = graph_steps(w, 1) if (graphs and not w.segments) else (w.step, None)
    with ClockSampler(dev.index) as clk:
        ms, kern_ms = time_steps(fn, steps, warmup, dist)
    del keep
    tokens_all = w.tokens
    if dist.pg:
        t = torch.tensor([w.tokens], dtype=torch.float64, device=dev)
        dist.pg.all_reduce(t)
        tokens_all = int(round(t.item()))
    res = {"ms": ms, "kern_ms": kern_ms, "value": tokens_all / (ms * 1e-3),
           "tflops": tokens_all * pkg.workloads.prefill_flops_per_token() / (ms * 1e-3) / 1e12,
           "achieved": w.flops / (kern_ms * 1e-3) / 1e12, "clocks": clk.summary(),
           "launches": w.launches * steps, "tokens": w.tokens, "tokens_all": tokens_all,
           "local_segments": w.local_segments}
    if with_e2e:
        h2d, d2h = w.host_copies()
        e2e_steps = max(2, min(steps, 5))
        e_ms, _ = time_steps(w.e2e_step, e2e_steps, 1, dist, per_launch_events=False)
        res["e2e"] = {"value": tokens_all / (e_ms * 1e-3), "unit": "tokens/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "ms_per_step": e_ms, "steps": e2e_steps}
    return res


def roofline(bound, achieved, workload, pk, src):
    if bound == "hbm":
        peak, unit = pk["hbm_gbs"], "GB/s"
    else:
        peak, unit = pk["bf16_tflops"], "TFLOP/s"
    return {"bound": bound, "achieved": round(achieved, 3), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": ncu_traffic(workload),
            "peak_source": f"{src} (burst; MEASURED_PEAKS.json)" if src == "measured"
            else "fallback (no MEASURED_PEAKS.json)"}


WORKLOADS = {
    "decode_b4": ("decode", 4), "decode_b128": ("decode", 128), "decode_b1024": ("decode", 1024),
    "prefill_p1": ("prefill", "P1"), "prefill_p2": ("prefill", "P2"),
    "prefill_p3": ("prefill", "P3"),
    "mtp_b128_t4": ("mtp", 128),
    "decode_b128_bf16state": ("decode_bf16state", 128),
}


def workload_config(W, kind, param, world, args):
    """`config` of the JSON line (the same dict for both arms): what one step is."""
    launch = "CUDA graph replay" if not args.no_graphs else "eager"
    if kind in ("decode", "decode_bf16state"):
        bf = kind == "decode_bf16state"
        units = W.decode_state_bytes(param) // (2 if bf else 1)
        return {"workload": f"GDN decode, batch {param} per GPU, 16 q/k + 32 v heads, "
                            f"head_dim 128, {'bf16' if bf else 'fp32'} k-last state, "
                            f"q/k L2-normalised in-kernel",
                "batch_per_gpu": param, "global_batch": param * world,
                "parallelism": f"batch-sharded x{world}, no collective",
                "l2": (f"inputs > L2: {units / 1e6:.0f} MB state traffic per step, state "
                       f"ping-pong" if units > L2_BYTES else
                       f"L2 flushed before every step ({units / 1e6:.1f} MB state traffic "
                       f"per step)"),
                "launch": launch}
    if kind == "mtp":
        units = W.mtp_state_bytes(param, MTP_T, intermediate=True)
        return {"workload": f"GDN multi-token decode, {param} rows x {MTP_T} tokens per GPU, "
                            f"16 q/k + 32 v heads, fp32 k-last state pool updated in place, "
                            f"rollback buffer written per token, q/k L2-normalised in-kernel",
                "batch_per_gpu": param, "draft_tokens": MTP_T,
                "parallelism": f"batch-sharded x{world}, no collective",
                "l2": f"inputs > L2: {units / 1e9:.2f} GB state traffic per step",
                "launch": launch}
    cfg = W.PREFILL_CONFIGS[param]
    lens = W.draw_seqlens(cfg.n, cfg.lo, cfg.hi, 0)
    return {"workload": f"GDN prefill {param}", "tokens": int(sum(lens)),
            "parallelism": plan_text(plan_kind(W, param, world, args.prefill_plan), world),
            "l2": "inputs > L2",
            "launch": launch if plan_kind(W, param, world, args.prefill_plan) != "segments"
            else "eager"}


def metric_of(kind):
    if kind in ("decode", "decode_bf16state"):
        return "decode state-traffic GB/s", "GB/s"
    if kind == "mtp":
        return "mtp state-traffic GB/s", "GB/s"
    return "prefill tokens/s", "tokens/s"


def dtype_of(kind):
    return {"decode": "fp32", "decode_bf16state": "fp32 compute, bf16 state",
            "mtp": "fp32"}.get(kind, "bf16")


def run_ours(args, dist):
    pkg = importlib.import_module(PKG_NAME)
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    pk, src = peaks()
    kind, param = WORKLOADS[args.workload]
    metric, unit = metric_of(kind)
    line = {"impl": "ours", "metric": metric}
    cfg = workload_config(pkg.workloads, kind, param, dist.world, args)
    if kind in ("decode", "decode_bf16state", "mtp"):
        if kind == "mtp":
            r = measure_mtp(pkg, dist, param, args.steps, args.warmup, dev,
                            graphs=not args.no_graphs)
        else:
            r = measure_decode(pkg, dist, param, args.steps, args.warmup, dev,
                               state_bf16=kind == "decode_bf16state", graphs=not args.no_graphs,
                               e2e_slices=args.e2e_slices)
        value, bound, scaling = round(r["value"], 2), "hbm", "weak"
    else:
        shard = prefill_plan(pkg, param, dist, args.prefill_plan)
        r = measure_prefill(pkg, dist, param, args.steps, args.warmup, dev, shard=shard,
                            graphs=not args.no_graphs)
        value, bound = round(r["value"], 1), "tensor"
        scaling = "strong" if dist.world > 1 else "weak"
    line.update({
        "value": value, "unit": unit, "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(r["ms"], 5), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": dtype_of(kind),
        "data": "synthetic (seeded)", "config": cfg,
        "roofline": roofline(bound, r["achieved"],
                             args.workload if (bound == "hbm" or dist.world == 1) else "",
                             pk, src),
        "e2e": r["e2e"], "gpu_launches": r["launches"], "clocks": r["clocks"],
        "kernel_ms": round(r["kern_ms"], 5),
    })
    if bound == "hbm":  # context: what a plain copy of the step's bytes reaches at this size
        cr = copy_reference(r["units"], dev)
        line["roofline"]["copy_same_bytes_gbs"] = round(cr, 1)
        line["roofline"]["frac_of_copy_same_bytes"] = round(r["achieved"] / cr, 4)
    if bound == "tensor":
        line["tflops"] = round(r["tflops"], 2)
    # secondary: the latency-bound decode config and the prefill configurations
    if kind == "decode" and not args.no_prefill_extra:
        d1 = measure_decode(pkg, dist, 4, max(20, min(args.steps, 100)), 5, dev, with_e2e=False)
        line["decode_b4"] = {
            "us_per_step": round(d1["ms"] * 1e3, 2),  # CUDA events around each graph replay
            "state_gb_per_s": round(d1["value"], 1), "launch": cfg["launch"],
            "l2": "L2 overwritten before every step (16.8 MB state traffic per step per GPU)",
            "global_batch": 4 * dist.world}
        extra = {}
        names = [("P1", "auto"), ("P2", "auto")] if dist.world == 1 else \
            [("P2", "heads"), ("P2_segment_scan", "segments"), ("P3", "heads"),
             ("P3_by_sequence", "seqs")]
        for label, force in names:
            nm = label.split("_")[0]
            shard = prefill_plan(pkg, nm, dist, force)
            r = measure_prefill(pkg, dist, nm, max(3, min(args.steps, 10)), 3, dev, shard=shard,
                                with_e2e=False, graphs=not args.no_graphs)
            extra[label] = {"tokens_per_s": round(r["value"], 1), "ms_per_step": round(r["ms"], 4),
                            "tflops": round(r["tflops"], 2), "tokens": r["tokens_all"],
                            "parallelism": plan_text(shard, dist.world)
                            + (f"; the sequence in {r['local_segments']} token segments side "
                               f"by side in one call per rank" if r["local_segments"] > 1
                               else ""),
                            # the committed traffic capture is of the unsharded call
                            "roofline": roofline("tensor", r["achieved"],
                                                 "prefill_" + nm.lower() if shard is None else "",
                                                 pk, src)}
        line["prefill"] = extra
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(kind, param)
    return line


def run_reference(args, dist):
    """The reference's CPU path on the host cores: the reference itself is Triton-only, so
    the CPU restatement of its algorithm (the oracle port) is timed, with every host thread,
    on the same workload, metric and config as the GPU arm, for exactly `steps` steps after
    `warmup` untimed ones (decode and multi-token decode: whole steps of the global batch
    up to 256 rows, each further row costing the same; prefill: a bounded sample of 1024
    tokens per step).  Only rank 0 runs; the package (and so the CUDA library) is never
    imported."""
    if dist.rank != 0:
        return None
    W, _ = cpu_modules()
    threads = host_threads()
    kind, param = WORKLOADS[args.workload]
    metric, unit = metric_of(kind)
    cfg = workload_config(W, kind, param, dist.world, args)
    if kind in ("decode", "decode_bf16state"):
        rows = min(param * dist.world, 256)
        step, units = cpu_decode_step(rows, state_bf16=kind == "decode_bf16state")
        per = timed_cpu(step, args.steps, args.warmup)
        value = units / per / 1e9
        sample = f"full decode steps of {rows} rows (oracle, fp32 torch CPU)"
    elif kind == "mtp":
        rows = min(param * dist.world, 16)
        step, units = cpu_mtp_step(rows)
        per = timed_cpu(step, args.steps, args.warmup)
        value = units / per / 1e9
        sample = f"{rows} rows x {MTP_T} tokens per step (oracle, fp32 torch CPU)"
    else:
        step, T, sample = cpu_prefill_step(param, 1024)
        per = timed_cpu(step, args.steps, args.warmup)
        value = T / per
        sample += " per step (oracle, fp32 torch CPU)"
    cb = {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample,
          "definition": definition_baseline(kind, param)}
    return {"impl": "reference", "metric": metric, "value": round(value, 4), "unit": unit,
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per * 1e3, 4), "higher_is_better": True,
            "scaling": "strong" if (kind == "prefill" and dist.world > 1) else "weak",
            "vs_baseline": None, "dtype": dtype_of(kind), "data": "synthetic (seeded)",
            "config": cfg, "cpu_baseline": cb,
            "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


class RankOnOneGpu:
    """The slice of Dist a prefill share needs, for rank `rank` of `world` emulated on one
    GPU (no process group: barriers and the max-over-ranks reduction are local)."""

    def __init__(self, world, rank):
        self.world, self.rank, self.local, self.pg = world, rank, 0, None

    def barrier(self):
        pass

    def max(self, x):
        return x


def run_emulated_ranks(args):
    """Each rank's share of a prefill config under the chosen multi-GPU plan, run on this
    one GPU in turn (`--emulate-world N`, optionally `--emulate-rank r`): per-rank device
    time, and the slowest rank's, which is the step a real N-GPU run would take without its
    launch skew.  The cross-GPU segment plan needs its collective and is not emulated."""
    pkg = importlib.import_module(PKG_NAME)
    dev = torch.device("cuda", 0)
    kind, param = WORKLOADS[args.workload]
    if kind != "prefill":
        raise SystemExit("--emulate-world applies to the prefill workloads")
    world = args.emulate_world
    ranks = [args.emulate_rank] if args.emulate_rank >= 0 else list(range(world))
    per = {}
    for r in ranks:
        d = RankOnOneGpu(world, r)
        shard = prefill_plan(pkg, param, d, args.prefill_plan)
        if shard is not None and shard[0] == "segments":
            raise SystemExit("the cross-GPU segment plan needs its all-gather: not emulated")
        w = PrefillWork(pkg, param, dev, seed=0, shard=shard, dist=d)
        fn, keep = graph_steps(w, 1) if not args.no_graphs else (w.step, None)
        ms, _ = time_steps(fn, args.steps, args.warmup, d)
        del keep
        per[r] = {"ms_per_step": round(ms, 4), "local_segments": w.local_segments}
    worst = max(v["ms_per_step"] for v in per.values())
    return {"impl": "ours", "metric": "prefill ms per rank (ranks emulated on one GPU)",
            "value": worst, "unit": "ms", "higher_is_better": False,
            "emulated_world": world, "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": f"GDN prefill {param}",
                       "parallelism": plan_text(plan_kind(pkg.workloads, param, world,
                                                          args.prefill_plan), world),
                       "launch": "eager" if args.no_graphs else "CUDA graph replay"},
            "ranks": per}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode_b128")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill-extra", action="store_true")
    ap.add_argument("--prefill-plan", choices=["auto", "heads", "seqs", "segments"],
                    default="auto",
                    help="multi-GPU split of a prefill config (default: q/k-head groups when "
                         "the heads divide evenly, no collective; 'seqs': whole sequences by "
                         "longest-first packing; 'segments': token-segment scan of one "
                         "sequence, one all-gather per call)")
    ap.add_argument("--e2e-slices", type=int, default=0,
                    help="batch slices of the pipelined end-to-end decode step (default %d)"
                         % E2E_SLICES)
    ap.add_argument("--no-graphs", action="store_true",
                    help="launch decode, multi-token decode and prefill steps eagerly (default: "
                         "CUDA graph replay)")
    ap.add_argument("--emulate-world", type=int, default=0,
                    help="prefill workloads: run each rank's share of an N-GPU plan on this "
                         "one GPU in turn and report per-rank times (not a bench line)")
    ap.add_argument("--emulate-rank", type=int, default=-1,
                    help="with --emulate-world: only this rank's share")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3  # timing rule: at least 3 warm-up steps
    dist = Dist()
    if args.impl == "reference":
        line = run_reference(args, dist)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "ours", "error": "no CUDA device"}), flush=True)
        sys.exit(1)
    if args.emulate_world > 1:
        print(json.dumps(run_emulated_ranks(args)), flush=True)
        return
    dist.init("nccl")
    try:
        line = run_ours(args, dist)
        if dist.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
