#!/usr/bin/env python
"""Benchmark of the B200-native fused FP8 MoE layer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (config 1 of the benchmark, the single-B200 decode path):
one call of the layer on T=64 tokens, 32 local experts, seeded synthetic
inputs with the benchmark distributions
(flashinfer-bench-avengers_b200/workloads.py). With N>1 GPUs (torchrun)
every rank owns a different 32-expert shard of the 256 experts
(local_expert_offset = 32*rank) over the same tokens; the library's NVLink
combine (moe_b200_ep_combine_shards, buffers shared through CUDA IPC) forms
the summed bf16 output on every rank: expert parallelism with fixed work
per GPU ("weak" scaling). At N>1 the line carries `ep_check`: every rank's
status word, and the fused output against the fp32 sum of independent
runs of every rank's shard (operator tolerance), identical on all ranks.

A step is one layer call. Timing: W untimed warm-up steps, then K steps
bracketed by a barrier and device synchronisation; the reported time is the
max over ranks. `value` is microseconds per call. L2: a call whose active
experts' weights exceed twice the 126 MB L2 (705 MB at T=64) cannot find
any weight byte in L2 from the previous call, so those calls run back to
back ("inputs larger than L2"); smaller calls get a 256 MB write flush
before each timed call. The headline line also reports the same call after
a 256 MB write flush (`value_l2_write_flushed`).

Extra points:
* every N: `ep_t8192` (config 3: T=8192, all 256 experts as 8 shards of 32
  spread over the N ranks, 8/N shards per rank, NVLink combine; fixed total
  work, "strong" scaling) and `stress` (config 4: T=16384 with Zipf(1.2)
  expert popularity, the same 8-shard layout; per-shard and per-rank times,
  the per-rank maximum is the figure). Both carry their own ep_check.
  `token_parallel_t8192`: the same T=8192 batch split over the ranks (each
  rank its own 8192/N tokens), all-to-all dispatch and combine
  (TokenParallelEP), checked against the expert-parallel sum of every
  shard's independent run.
* N=1 only: the decode sweep T in {1,4,16,64} (config 1; T=1 uses the first
  seed >= 1234 whose token picks a local expert, stated in the point), the
  prefill point (config 2, T=4096 with 4 hot experts), the reference
  solution's own CUDA kernel timed on the same box and inputs at each of
  those points (`reference_kernel`, built unchanged from its sources by
  baseline/build_reference.py; "unavailable" when not built) and the CPU
  baselines (the oracle over all active experts, median of 3 runs, for the
  headline and for config 0).

`--impl reference` times the reference algorithm on the host CPU (the
reference solution has no CPU implementation, so its CPU restatement in
oracle/ stands in for it) on the same workload and prints the same line
with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "flashinfer-bench-avengers_b200")
sys.path.insert(0, PKG)

import workloads  # noqa: E402

METRIC = "fused-MoE µs/call and TFLOPS vs FP8/HBM roofline, T=1..16384, 1/2/4/8 B200"
UNIT = "us/call"
SEED = 1234
# name -> (T, routing variant, description); "decode" is the default headline.
WORKLOADS = {
    "decode": (64, "uniform", "config1 decode: one MoE layer call, T=64"),
    "prefill": (4096, "hot", "config2 prefill: one MoE layer call, T=4096, 4 hot local experts"),
}
NUM_SHARDS = 8
DATA = ("synthetic, seeded (contest dataset unavailable); N(0,1) logits, N(0,0.1) bf16 bias, "
        "e4m3 1x128 / 128x128 block-scaled N(0,1) activations and N(0,0.02) weights")
REL_TOL = 1e-2
MATCH_FRAC = 0.999

# Algorithmic sizes (bytes, FLOPs) of the operator.
W13_BYTES = 2 * 2048 * 7168 + 32 * 56 * 4          # per active expert, weights + scales
W2_BYTES = 7168 * 2048 + 56 * 16 * 4
ACT_IN_BYTES = 7168 + 56 * 4                        # one gathered token row + its scales
C_BYTES = 2 * 2048 + 16 * 4                         # hi/lo operand row + scales
LAYER_BYTES_PER_EXPERT = 44_050_944
LAYER_BYTES_PER_TOKEN = 22_752
FLOP_PER_ASSIGNMENT_G1 = 2 * 7168 * 4096
FLOP_PER_ASSIGNMENT_G2 = 2 * 2048 * 7168

# Published reference latencies: the reference kernel on a Modal B200, from
# the summary of its scripts/run_modal.py in the reference's Trace_Summary.png.
PUBLISHED_US = {1: 551.0, 7: 1034.0, 14: 1609.0, 15: 850.0, 16: 1727.0, 32: 2803.0, 80: 3620.0,
                901: 4545.0, 11948: 11731.0, 14107: 15650.0}

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) from
# the ncu captures summarised in profiles/, keyed by (kernel, T) of the bench
# workloads; None when no capture of that launch exists.
NCU_TRAFFIC_BYTES = {("gemm1", 64): 472_752_896 + 9_058_048, ("gemm1", 4096): 860_626_688 + 72_598_016}


def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and throttle reasons of this rank's GPU during the timed region.

    With NVML (nvidia-ml-py) samples are kept only while the sampler is armed,
    which `time_step` does around its timed loop (a few milliseconds): a
    background thread polls every 0.25 ms when it gets the interpreter, and
    the timing loop itself samples once all timed calls are queued, until
    the last one ends. Without NVML, nvidia-smi samples every 200 ms for the
    whole block instead."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    POLL_S = 0.00025
    # NVML clock-event reason bits
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: torch.device):
        self.dev = device
        self.proc = None
        self.lines: list[str] = []
        self.thread = None
        self.nvml = None
        self.handle = None
        self.armed = False
        self.stop = False
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None

    def _uuid(self) -> str | None:
        try:
            uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            return uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            return None

    def __enter__(self):
        uuid = self._uuid()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.handle = (pynvml.nvmlDeviceGetHandleByUUID(uuid) if uuid is not None
                           else pynvml.nvmlDeviceGetHandleByIndex(self.dev.index or 0))
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            sel = uuid if uuid is not None else str(self.dev.index or 0)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", sel, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def arm(self):
        self.armed = True

    def sample_now(self):
        """One sample from the calling thread (the timing loop calls this
        once all timed calls are queued, while the GPU still runs them)."""
        if self.nvml is None:
            return
        try:
            nv = self.nvml
            self.samples.append((float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)),
                                 int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle))))
        except Exception:
            pass

    def disarm(self):
        self.armed = False

    def _poll(self):
        nv = self.nvml
        while not self.stop:
            if self.armed:
                try:
                    mhz = float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                    reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
                    self.samples.append((mhz, reasons))
                except Exception:
                    pass
            time.sleep(self.POLL_S)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop = True
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        if self.nvml is not None:
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self) -> dict:
        if self.nvml is not None:
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "source": "nvml"}
            reasons = sorted(n for n, bit in self.REASON_BITS.items() if any(r & bit for _, r in self.samples))
            return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml, timed region only"}
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": "nvidia-smi"}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 200 ms"}


# ------------------------------------------------------------------ helpers
def routing_stats(inp: dict) -> dict:
    """Active local experts and assignment counts, computed on the device
    from the layer's own routing output (no CPU oracle)."""
    import moe_host

    idx, _ = moe_host.route(inp["routing_logits"], inp["routing_bias"], inp["routed_scaling_factor"])
    le = idx.long() - int(inp["local_expert_offset"])
    local = (le >= 0) & (le < 32)
    counts = torch.bincount(le[local], minlength=32).cpu()
    return {"T": int(idx.shape[0]), "E_act": int((counts > 0).sum()), "sum_Tk": int(counts.sum()),
            "max_Tk": int(counts.max()), "tokens_touched": int(local.any(dim=1).sum())}


def kernel_bytes(st: dict) -> dict:
    e, n = st["E_act"], st["sum_Tk"]
    g1 = e * W13_BYTES + n * (ACT_IN_BYTES + C_BYTES)
    g2 = e * W2_BYTES + n * C_BYTES + st["tokens_touched"] * 7168 * 4
    return {"gemm1": g1, "gemm2": g2}


def kernel_flops(st: dict) -> dict:
    n = st["sum_Tk"]
    return {"gemm1": n * FLOP_PER_ASSIGNMENT_G1, "gemm2": n * FLOP_PER_ASSIGNMENT_G2}


def layer_bytes(st: dict) -> int:
    return st["E_act"] * LAYER_BYTES_PER_EXPERT + st["T"] * LAYER_BYTES_PER_TOKEN + 512


def layer_flops(sum_tk: int) -> int:
    return sum_tk * (FLOP_PER_ASSIGNMENT_G1 + FLOP_PER_ASSIGNMENT_G2)


L2_BYTES = 126 * 1024 * 1024


def weights_exceed_l2(st: dict) -> bool:
    """True when one call streams more than twice the L2 in expert weights."""
    return st["E_act"] * (W13_BYTES + W2_BYTES) > 2 * L2_BYTES


def headline_config(desc: str, T: int, offset: int, st: dict, world: int, back_to_back: bool) -> dict:
    """The `config` of the headline line; both arms print the same one (the
    reference arm derives `st` and the L2 policy from the same routing)."""
    return {"workload": f"{desc}, 32 local experts per GPU",
            "T": T, "local_expert_offset": offset, "E_act": st["E_act"], "sum_Tk": st["sum_Tk"],
            "parallelism": f"ep{world}" + (" + NVLink combine (peer loads/stores, one kernel)" if world > 1 else ""),
            **({"hidden": "bf16, quantised per 1x128 block inside the row copy (moe_b200_run_bf16_hidden)"}
               if BF16_HIDDEN else {}),
            "l2": ("back to back: each call streams the active experts' weights "
                   f"({st['E_act'] * (W13_BYTES + W2_BYTES) / 1e6:.0f} MB > 2 x 126 MB L2), so no "
                   "weight byte is L2-resident from the previous call; value_l2_write_flushed is the "
                   "same call after a 256 MB write flush" if back_to_back else
                   "flushed (256 MB write) before every timed call")}


# --bf16-hidden: the calls take bf16 hidden states (inp["hidden_bf16"]) and
# quantise them inside the layer (moe_b200_run_bf16_hidden), one GPU only.
BF16_HIDDEN = False


def token_keys() -> tuple:
    """The per-call activation tensors of a step."""
    return ("routing_logits", "hidden_bf16") if BF16_HIDDEN else ("routing_logits", "hidden_states",
                                                                     "hidden_states_scale")


def shard_list(inps: list) -> list:
    return [(i["gemm1_weights"], i["gemm1_weights_scale"], i["gemm2_weights"], i["gemm2_weights_scale"],
             i["local_expert_offset"]) for i in inps]


def make_step(inps: list, combiner=None, marks=None):
    """One layer call on a step's tokens into `out`: the library entry point
    (one shard, no combiner), or this rank's shards one after another and the
    NVLink combine. `marks` (external CUDA events, shards + 2 of them) are
    recorded before each shard, before the combine and after it."""
    import moe_host

    inp = inps[0]
    if BF16_HIDDEN:
        args = workloads.as_args(inp)
        return lambda tokens, out: moe_host.run_bf16_hidden(tokens["routing_logits"], inp["routing_bias"],
                                                            tokens["hidden_bf16"], *args[4:], output=out)
    if combiner is None:
        args = workloads.as_args(inp)
        return lambda tokens, out: moe_host.run_dps(tokens["routing_logits"], inp["routing_bias"],
                                                    tokens["hidden_states"], tokens["hidden_states_scale"],
                                                    *args[4:], out)
    shards = shard_list(inps)

    def step(tokens, out):
        tok = {"routing_logits": tokens["routing_logits"], "routing_bias": inp["routing_bias"],
               "hidden_states": tokens["hidden_states"], "hidden_states_scale": tokens["hidden_states_scale"],
               "routed_scaling_factor": inp["routed_scaling_factor"]}
        for s, (w13, s13, w2, s2, off) in enumerate(shards):
            if marks is not None:
                marks[s].record()
            combiner.run_shard(s, tok, w13, s13, w2, s2, off)
        if marks is not None:
            marks[len(shards)].record()
        combiner.combine(tok["routing_logits"].shape[0], out)
        if marks is not None:
            marks[len(shards) + 1].record()
        return out
    return step


def time_step(inps: list, steps: int, warmup: int, flush: torch.Tensor, group=None,
              do_flush: bool = True, combiner=None, clocks=None, flushed_too: bool = True) -> dict:
    """Device time of `steps` calls replayed from a CUDA graph, each after a
    256 MB write flush when `do_flush` (otherwise back to back, and the
    flushed timing is then taken as well, as `call_ms_flushed`). A second
    graph of the same call gives the breakdown: with one shard the library's
    stage events, with a combiner external events around every shard and the
    combine (their nodes add a little latency, so the headline time comes
    from the graph without them)."""
    import moe_host
    import torch.distributed as dist

    inp = inps[0]
    tokens = {k: inp[k] for k in token_keys()}
    T = inp["routing_logits"].shape[0]
    dev = inp["routing_logits"].device
    out = torch.empty(T, 7168, dtype=torch.bfloat16, device=dev)
    call = make_step(inps, combiner)
    if combiner is None:
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(moe_host.NUM_STAGE_EVENTS)]
        for e in ev:
            e.record()
        staged_call = call
    else:
        ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(inps) + 2)]
        staged_call = make_step(inps, combiner, marks=ev)
    for _ in range(warmup):
        call(tokens, out)
    torch.cuda.synchronize()
    cap_stream = torch.cuda.Stream(dev)
    plain, staged = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap_stream):
        with torch.cuda.graph(plain, stream=cap_stream):
            call(tokens, out)
        if combiner is None:
            moe_host.set_stage_events(ev)
        try:
            with torch.cuda.graph(staged, stream=cap_stream):
                staged_call(tokens, out)
        finally:
            if combiner is None:
                moe_host.set_stage_events(None)
    for _ in range(warmup):
        plain.replay()
    torch.cuda.synchronize()
    if group is not None:
        dist.barrier(group=group)
    torch.cuda.synchronize()

    def timed(flushed: bool, sampler=None) -> list:
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        if sampler is not None:
            sampler.arm()   # clock samples only while the timed calls run
        for i in range(steps):
            if flushed:
                flush.zero_()
            starts[i].record()
            plain.replay()
            ends[i].record()
        if sampler is not None:
            # every timed call is queued: sample while the GPU runs them (not
            # between enqueues, which would delay this rank's calls and, with
            # the NVLink combine, make the other ranks wait inside their steps)
            while not ends[-1].query():
                sampler.sample_now()
                time.sleep(0.0002)
        torch.cuda.synchronize()
        if sampler is not None:
            sampler.disarm()
        if group is not None:
            dist.barrier(group=group)
        return [a.elapsed_time(b) for a, b in zip(starts, ends)]

    call_ms = timed(do_flush, clocks)
    call_ms_flushed = call_ms if (do_flush or not flushed_too) else timed(True)
    # the same calls once more, replaying the graph with the breakdown events
    parts: dict[str, list] = {}
    for _ in range(max(3, steps // 4)):
        if do_flush:
            flush.zero_()
        staged.replay()
        torch.cuda.synchronize()  # the events are reused every replay
        if combiner is None:
            names = moe_host.STAGE_NAMES
        else:
            names = [f"shard{s}" for s in range(len(inps))] + ["combine"]
        for j, name in enumerate(names):
            parts.setdefault(name, []).append(ev[j].elapsed_time(ev[j + 1]))
    torch.cuda.synchronize()
    if group is not None:
        dist.barrier(group=group)
    del plain, staged
    return {"call_ms": call_ms, "call_ms_flushed": call_ms_flushed,
            "stage_ms": {k: statistics.mean(v) for k, v in parts.items()}, "out": out}


def time_e2e(inps: list, steps: int, warmup: int, group=None, combiner=None) -> dict:
    """The public API call with host buffers: every step copies its
    activations host->device from pinned memory, runs the layer through
    moe_host.run_dps (with a combiner: this rank's shards and the NVLink
    combine) and copies the bf16 result device->host. Copies run on their
    own streams with two buffer sets, so step i+1's upload and step i-1's
    download overlap step i's compute; the timed region spans the first
    upload to the last download."""
    inp = inps[0]
    call = make_step(inps, combiner)
    dev = inp["routing_logits"].device
    T = inp["routing_logits"].shape[0]
    keys = token_keys()
    host_in = {k: inp[k].cpu().pin_memory() for k in keys}
    dev_in = [{k: torch.empty_like(v, device=dev) for k, v in host_in.items()} for _ in range(2)]
    out = [torch.empty(T, 7168, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    host_out = [torch.empty(T, 7168, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    d2h = host_out[0].numel() * host_out[0].element_size()
    compute = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    for b in range(2):
        computed[b].record(compute)
        downloaded[b].record(compute)

    def step(i):
        b = i % 2
        with torch.cuda.stream(up):
            up.wait_event(computed[b])           # buffer b's previous compute is done
            for k in keys:
                dev_in[b][k].copy_(host_in[k], non_blocking=True)
            uploaded[b].record(up)
        compute.wait_event(uploaded[b])
        compute.wait_event(downloaded[b])        # out[b] has been read back
        call(dev_in[b], out[b])
        computed[b].record(compute)
        with torch.cuda.stream(down):
            down.wait_event(computed[b])
            host_out[b].copy_(out[b], non_blocking=True)
            downloaded[b].record(down)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(up)
    for i in range(steps):
        step(i)
    down.wait_event(computed[(steps - 1) % 2])
    e.record(down)
    torch.cuda.synchronize()
    return {"ms": s.elapsed_time(e) / steps, "h2d": h2d, "d2h": d2h}


def ep_check(combiner, inps: list, fused: torch.Tensor, group) -> dict:
    """Correctness of the combined output of the last timed call: every
    rank's status words, the output against the fp32 sum over every shard of
    every rank of independent layer runs (moe_host.run, the regular entry
    point), within the operator tolerance, and identical on all ranks."""
    import moe_host
    import torch.distributed as dist

    status = combiner.status()
    ref = None
    for inp in inps:
        part = moe_host.run(*workloads.as_args(inp)).float()
        ref = part if ref is None else ref + part
    world = 1 if group is None else dist.get_world_size(group)
    if world > 1:
        dist.all_reduce(ref, group=group)
    err = (fused.float() - ref).abs()
    amax = float(ref.abs().max())
    matched = float((err <= REL_TOL * amax).float().mean())
    other = fused.clone()
    if world > 1:
        dist.broadcast(other, src=0, group=group)
    mine = torch.tensor([float(status), matched, float(err.max()), 1.0 if torch.equal(fused, other) else 0.0],
                        dtype=torch.float64, device=fused.device)
    allr = [torch.zeros_like(mine) for _ in range(world)]
    if world > 1:
        dist.all_gather(allr, mine, group=group)
    else:
        allr = [mine]
    st = 0
    for v in allr:
        st |= int(v[0])
    return {"status": st, "matched": round(min(float(v[1]) for v in allr), 6),
            "max_err": max(float(v[2]) for v in allr), "max_abs_ref": amax,
            "identical": all(float(v[3]) == 1.0 for v in allr),
            "reference": "fp32 sum of independent moe_b200_run outputs of every shard",
            "tolerance": f"|err| <= {REL_TOL} * max|ref| on >= {MATCH_FRAC} of elements"}


def cpu_oracle_time(inp: dict, runs: int = 3) -> dict:
    """The CPU restatement of the reference algorithm (oracle/) over the
    whole workload (every active expert) on the host cores: one warm-up run,
    then the median of `runs` runs. The inputs are copied to host memory
    first, outside the timing (only the active experts' weights)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import moe_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    small = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale")
    cpu_inp = {k: (v.cpu() if isinstance(v, torch.Tensor) and k in small else v) for k, v in inp.items()}
    active = moe_oracle.active_local_experts(cpu_inp["routing_logits"], cpu_inp["routing_bias"],
                                             inp["routed_scaling_factor"], inp["local_expert_offset"])
    for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale"):
        full = inp[k]
        host = torch.zeros(full.shape, dtype=full.dtype)
        for e in active:
            host[e].copy_(full[e].cpu())
        cpu_inp[k] = host
    cargs = workloads.as_args(cpu_inp)
    moe_oracle.moe_forward(*cargs)   # warm-up
    times, route_times = [], []
    for _ in range(runs):
        t0 = time.perf_counter()
        moe_oracle.moe_forward(*cargs)
        times.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        moe_oracle.route(cpu_inp["routing_logits"], cpu_inp["routing_bias"], inp["routed_scaling_factor"])
        route_times.append(time.perf_counter() - t0)
    T = inp["routing_logits"].shape[0]
    total_us = statistics.median(times) * 1e6
    route_us = statistics.median(route_times) * 1e6
    return {"value": round(total_us, 1), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port", "runs_s": [round(t, 3) for t in times],
            "routing_us": round(route_us, 1), "experts_us": round(total_us - route_us, 1),
            "sample": f"T={T}, all {len(active)} active experts (the whole call), median of {runs} runs "
                      f"after one warm-up"}


def roofline_entry(ms: float, nbytes: int, flops: int, peaks: dict, bound: str) -> dict:
    if bound == "hbm":
        achieved = nbytes / (ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        unit = "GB/s"
    else:
        achieved = flops / (ms * 1e-3) / 1e12
        peak = 2.0 * peaks["bf16_tflops"]  # dense e4m3 = 2x dense bf16 on the same tensor cores
        unit = "TFLOP/s"
    return {"achieved": round(achieved, 1), "peak": round(peak, 1), "unit": unit,
            "frac": round(achieved / peak, 4)}


def roofline_point(us: float, lb: int, lf: int, peaks: dict, n_gpus: int = 1) -> dict:
    t_hbm = lb / (n_gpus * peaks["hbm_gbs"] * 1e9)
    t_tc = lf / (n_gpus * 2.0 * peaks["bf16_tflops"] * 1e12)
    r = max(t_hbm, t_tc) * 1e6
    return {"roofline_us": round(r, 2), "roofline_bound": "hbm" if t_hbm >= t_tc else "tensor",
            "frac_of_roofline": round(r / us, 4) if us > 0 else None}


def first_seed_with_local_pick(T: int, device, seed: int = SEED) -> int:
    """The first seed >= `seed` whose tokens pick at least one of the 32
    local experts at offset 0 (with offset 0 a token reaches them only when
    routing group 0 is among its 4 kept groups, about half the time)."""
    import moe_host

    for s in range(seed, seed + 1000):
        r = workloads.make_routing_inputs(T, s, device)
        idx, _ = moe_host.route(r["routing_logits"], r["routing_bias"], 2.5)
        if bool(((idx >= 0) & (idx < 32)).any()):
            return s
    raise RuntimeError("no seed with a local pick")


def fixed_latency_split(p: dict, steps: int, warmup: int, flush, peaks, device) -> dict:
    """Where a decode call's time goes beyond its weight bytes: the same
    call with local_expert_offset 256, where no pick is local (routing, the
    permutation, the GEMM launches that find no unit, the zero output),
    against the call's bytes at the measured HBM peak."""
    inp = workloads.make_inputs(p["T"], p["seed"], device, "uniform")
    inp["local_expert_offset"] = 256
    r = time_step([inp], steps, warmup, flush, do_flush=True, flushed_too=False)
    empty_us = statistics.mean(r["call_ms"]) * 1e3
    del r["out"]
    bytes_us = p["roofline_us"]
    return {"empty_call_us": round(empty_us, 2), "empty_call": "same tokens, local_expert_offset 256",
            "bytes_at_hbm_peak_us": round(bytes_us, 2),
            "rest_us": round(p["us_per_call"] - empty_us - bytes_us, 2),
            "note": "us_per_call = empty_call_us (fixed latency) + bytes_at_hbm_peak_us + rest_us "
                    "(streaming below peak and the stage hand-offs)"}


def point(T: int, variant: str, steps: int, warmup: int, flush, peaks, device, seed=SEED) -> dict:
    inp = workloads.make_inputs(T, seed, device, variant)
    st = routing_stats(inp)
    r = time_step([inp], steps, warmup, flush, do_flush=not weights_exceed_l2(st))
    us = statistics.mean(r["call_ms"]) * 1e3
    lb = layer_bytes(st)
    lf = layer_flops(st["sum_Tk"])
    res = {"T": T, "variant": variant, "seed": seed, "us_per_call": round(us, 2), **st,
           "layer_GBps": round(lb / (us * 1e-6) / 1e9, 1), "layer_TFLOPs": round(lf / (us * 1e-6) / 1e12, 2),
           "stages_us": {k: round(v * 1e3, 2) for k, v in r["stage_ms"].items()},
           "l2": "back to back (weights > 2x L2)" if weights_exceed_l2(st) else "256 MB write flush",
           "us_per_call_l2_write_flushed": round(statistics.mean(r["call_ms_flushed"]) * 1e3, 2)}
    res.update(roofline_point(us, lb, lf, peaks))
    if T in PUBLISHED_US and st["sum_Tk"] > 0:
        res["published_reference_us"] = PUBLISHED_US[T]
    del r["out"]
    return res


def reference_kernel_point(T: int, variant: str, seed: int, steps: int, warmup: int, flush, device,
                           ours_us: float) -> dict:
    """The reference solution's own CUDA implementation (built unchanged from
    its solution/cuda sources by baseline/build_reference.py) on the same
    inputs as our point: device time of whole calls of its run(...) from a
    start event to an end event on the stream (its call synchronises the
    host mid-way and launches per-expert kernels from a host loop, so
    that time is part of it), with our L2 policy. Its output is compared
    with ours within the operator tolerance."""
    import moe_host

    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import build_reference

    if build_reference.built_path() is None:
        return {"T": T, "unavailable": "reference extension not built (baseline/build_reference.py)"}
    mod = build_reference.load_built()
    inp = workloads.make_inputs(T, seed, device, variant)
    st = routing_stats(inp)
    args = workloads.as_args(inp)
    do_flush = not weights_exceed_l2(st)
    for _ in range(warmup):
        out_ref = mod.run(*args)
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        if do_flush:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out_ref = mod.run(*args)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    ours = moe_host.run(*args)
    torch.cuda.synchronize()
    err = (ours.float() - out_ref.float()).abs()
    amax = float(out_ref.float().abs().max())
    us = statistics.median(times)
    return {"T": T, "variant": variant, "seed": seed, "reference_kernel_us": round(us, 2),
            "ours_us": round(ours_us, 2), "speedup": round(us / ours_us, 2) if ours_us > 0 else None,
            "E_act": st["E_act"], "sum_Tk": st["sum_Tk"],
            "ours_vs_reference_matched": round(float((err <= REL_TOL * amax).float().mean()), 6)}


def all_shard_point(T: int, variant: str, desc: str, steps: int, warmup: int, flush, peaks, device, group,
                    world: int, rank: int, shards_per_rank: int | None = None) -> dict:
    """Configs 3 and 4: the whole layer over all 256 experts as 8 shards of
    32, 8/N shards per rank (offsets 32 * (rank * 8/N + s)), each shard its
    own layer call with its combine rows kept, then one NVLink combine.
    Total work is fixed ("strong" scaling); the time is the max over ranks.
    Reports every shard's routing statistics and time, each rank's shard and
    combine times, the whole-layer roofline over N GPUs and an ep_check.
    ``shards_per_rank`` below 8/N covers only the first N x that many shards
    (a smaller case of the same calls, for profiling)."""
    import expert_parallel
    import torch.distributed as dist

    spr = NUM_SHARDS // world if shards_per_rank is None else shards_per_rank
    offsets = [32 * (rank * spr + s) for s in range(spr)]
    inps = [workloads.make_inputs(T, SEED, device, variant, off, 2.5, weight_seed=SEED + 1 + off // 32)
            for off in offsets]
    stats = [routing_stats(i) for i in inps]
    combiner = expert_parallel.NvlinkCombiner(T, device, group, shards_per_rank=spr)
    try:
        r = time_step(inps, steps, warmup, flush, group, do_flush=False, combiner=combiner, flushed_too=False)
        check = ep_check(combiner, inps, r["out"], group)
    finally:
        combiner.close()
    step_us = statistics.mean(r["call_ms"]) * 1e3
    shard_us = [r["stage_ms"][f"shard{s}"] * 1e3 for s in range(spr)]
    comb_us = r["stage_ms"]["combine"] * 1e3
    mine = torch.tensor([step_us, sum(shard_us), comb_us], dtype=torch.float64, device=device)
    rows = torch.tensor([[offsets[s], st["E_act"], st["sum_Tk"], st["max_Tk"], st["tokens_touched"], shard_us[s]]
                         for s, st in enumerate(stats)], dtype=torch.float64, device=device)
    if world > 1:
        allm = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allm, mine, group=group)
        allrows = [torch.zeros_like(rows) for _ in range(world)]
        dist.all_gather(allrows, rows, group=group)
    else:
        allm, allrows = [mine], [rows]
    per_rank = [{"rank": q, "us_per_call": round(float(v[0]), 2), "shards_us": round(float(v[1]), 2),
                 "combine_us": round(float(v[2]), 2)} for q, v in enumerate(allm)]
    shards = [{"local_expert_offset": int(x[0]), "E_act": int(x[1]), "sum_Tk": int(x[2]), "max_Tk": int(x[3]),
               "tokens_touched": int(x[4]), "us": round(float(x[5]), 2)} for rr in allrows for x in rr]
    us = max(p["us_per_call"] for p in per_rank)
    e_act = sum(s["E_act"] for s in shards)
    sum_tk = sum(s["sum_Tk"] for s in shards)
    lb = e_act * LAYER_BYTES_PER_EXPERT + T * LAYER_BYTES_PER_TOKEN + 512
    lf = layer_flops(sum_tk)
    res = {"T": T, "variant": variant, "workload": desc, "n_gpus": world, "shards_per_rank": spr,
           "scaling": "strong (all 256 experts at every N)", "us_per_call": round(us, 2),
           "E_act": e_act, "sum_Tk": sum_tk, "layer_TFLOPs": round(lf / (us * 1e-6) / 1e12, 2),
           "max_shard_us": max(s["us"] for s in shards), "per_rank": per_rank, "shards": shards,
           "l2": "back to back (weights > 2x L2)", "ep_check": check}
    res.update(roofline_point(us, lb, lf, peaks, world))
    return res


def token_parallel_point(T: int, steps: int, warmup: int, peaks, device, group, world: int, rank: int) -> dict:
    """Token-parallel expert parallelism on the batch of config 3: rank r
    holds rows [rT/N, (r+1)T/N) of the same T-token batch (each rank its own
    tokens) and owns 8/N shards; one step is routing, the all-to-all
    dispatch, the shards on the received rows and the all-to-all combine
    (TokenParallelEP), replayed from a CUDA graph; time = max over ranks.
    Checked against the expert-parallel sum of independent runs of every
    shard on the whole batch (operator tolerance), status words clear."""
    import expert_parallel
    import moe_host
    import torch.distributed as dist

    spr = NUM_SHARDS // world
    offsets = [32 * (rank * spr + s) for s in range(spr)]
    full = [workloads.make_inputs(T, SEED, device, "uniform", off, 2.5, weight_seed=SEED + 1 + off // 32)
            for off in offsets]
    lo, hi = T * rank // world, T * (rank + 1) // world
    f = full[0]
    tok = {"routing_logits": f["routing_logits"][lo:hi].contiguous(), "routing_bias": f["routing_bias"],
           "hidden_states": f["hidden_states"][lo:hi].contiguous(),
           "hidden_states_scale": f["hidden_states_scale"][:, lo:hi].contiguous(), "routed_scaling_factor": 2.5}
    shards = [(i["gemm1_weights"], i["gemm1_weights_scale"], i["gemm2_weights"], i["gemm2_weights_scale"])
              for i in full]
    Tmax = max(T * (q + 1) // world - T * q // world for q in range(world))
    tp = expert_parallel.TokenParallelEP(Tmax, device, group)
    out = torch.empty(hi - lo, 7168, dtype=torch.bfloat16, device=device)
    try:
        for _ in range(warmup):
            tp.forward(tok, shards, out)
        torch.cuda.synchronize()
        stream = torch.cuda.Stream(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                tp.forward(tok, shards, out)
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        if group is not None:
            dist.barrier(group=group)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        for i in range(steps):
            starts[i].record()
            graph.replay()
            ends[i].record()
        torch.cuda.synchronize()
        if group is not None:
            dist.barrier(group=group)
        us = statistics.mean(a.elapsed_time(b) for a, b in zip(starts, ends)) * 1e3
        status = tp.status()
        recv = tp.slab_rows()
        del graph
    finally:
        tp.close()
    # reference: every shard's independent run on the whole batch, summed over ranks
    ref = None
    for i in full:
        part = moe_host.run(*workloads.as_args(i)).float()
        ref = part if ref is None else ref + part
    if world > 1:
        dist.all_reduce(ref, group=group)
    ref = ref[lo:hi]
    err = (out.float() - ref).abs()
    amax = float(ref.abs().max())
    matched = float((err <= REL_TOL * amax).float().mean())
    mine = torch.tensor([us, float(status), matched, float(recv), float(hi - lo)], dtype=torch.float64, device=device)
    if world > 1:
        allm = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allm, mine, group=group)
    else:
        allm = [mine]
    st = 0
    for v in allm:
        st |= int(v[1])
    us_max = max(float(v[0]) for v in allm)
    lf = layer_flops(T * 8)
    return {"T": T, "variant": "uniform", "n_gpus": world, "shards_per_rank": spr,
            "workload": "token-parallel EP: each rank holds 1/N of the config-3 batch, all-to-all dispatch "
                        "and combine over NVLink",
            "scaling": "strong (all 256 experts, the same 8192 tokens at every N)", "us_per_call": round(us_max, 2),
            "layer_TFLOPs": round(lf / (us_max * 1e-6) / 1e12, 2),
            "per_rank": [{"rank": q, "us_per_call": round(float(v[0]), 2), "tokens": int(v[4]),
                          "rows_received": int(v[3])} for q, v in enumerate(allm)],
            "check": {"status": st, "matched": round(min(float(v[2]) for v in allm), 6),
                      "reference": "fp32 sum of independent moe_b200_run outputs of every shard on the whole batch",
                      "tolerance": f"|err| <= {REL_TOL} * max|ref| on >= {MATCH_FRAC} of elements"}}


# --------------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip the sweep/prefill/stress/EP points")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="decode",
                    help="headline configuration (default: config 1 decode, T=64)")
    ap.add_argument("--bf16-hidden", action="store_true",
                    help="bf16 hidden states quantised inside the layer (one GPU; the extras are skipped)")
    ap.add_argument("--ep-point", default=None, metavar="T:S",
                    help="only the expert-parallel point with T uniform tokens and S shards per rank "
                         "(a smaller case of ep_t8192 for profiling); prints that point as the line")
    args = ap.parse_args()
    warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, world, rank, warmup)
        return

    import moe_host
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        if NUM_SHARDS % world != 0:
            raise SystemExit(f"--gpus {world} must divide the {NUM_SHARDS} expert shards")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
        group = dist.group.WORLD
    moe_host.load_library()
    peaks = load_peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    if args.ep_point is not None:
        T_ep, spr = (int(x) for x in args.ep_point.split(":"))
        res = all_shard_point(T_ep, "uniform", f"expert-parallel point: T={T_ep}, {spr} shards per rank",
                              args.steps, warmup, flush, peaks, device, group, world, rank, shards_per_rank=spr)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "unit": UNIT, "value": res["us_per_call"], "n_gpus": world,
                              "steps": args.steps, "warmup": warmup, "ep_point": res}), flush=True)
        if group is not None:
            torch.cuda.synchronize()
            dist.barrier(group=group)
            dist.destroy_process_group()
        return

    HEADLINE_T, variant, desc = WORKLOADS[args.workload]
    offset = (32 * rank) % 256
    inp = workloads.make_inputs(HEADLINE_T, SEED, device, variant, offset, 2.5, weight_seed=SEED + 1 + rank)
    if args.bf16_hidden:
        if world > 1:
            raise SystemExit("--bf16-hidden runs on one GPU")
        global BF16_HIDDEN
        BF16_HIDDEN = True
        # the bf16 source of inp's e4m3 hidden states: the same tokens and routing
        inp["hidden_bf16"] = workloads.make_hidden_bf16(HEADLINE_T, SEED, device)
    st = routing_stats(inp)

    # every rank must take the same timing path (the all-reduces inside it)
    b2b = torch.tensor(1 if weights_exceed_l2(st) else 0, device=device)
    if group is not None:
        dist.all_reduce(b2b, op=dist.ReduceOp.MIN, group=group)
    back_to_back = bool(b2b.item())
    combiner = None
    if group is not None:
        import expert_parallel
        combiner = expert_parallel.NvlinkCombiner(HEADLINE_T, device, group)
    with ClockSampler(device) as clocks:
        r = time_step([inp], args.steps, warmup, flush, group, do_flush=not back_to_back, combiner=combiner,
                      clocks=clocks)
    check = ep_check(combiner, [inp], r["out"], group) if combiner is not None else None
    call_ms = torch.tensor(r["call_ms"], dtype=torch.float64, device=device)
    mean_ms = call_ms.mean()
    if group is not None:
        dist.all_reduce(mean_ms, op=dist.ReduceOp.MAX, group=group)
    per_rank = None
    if group is not None:
        mine = torch.tensor([float(statistics.mean(r["call_ms"])) * 1e3, float(st["E_act"]), float(st["sum_Tk"]),
                             r["stage_ms"]["shard0"] * 1e3, r["stage_ms"]["combine"] * 1e3],
                            dtype=torch.float64, device=device)
        allr = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine, group=group)
        per_rank = [{"rank": q, "us_per_call": round(float(v[0]), 2), "E_act": int(v[1]), "sum_Tk": int(v[2]),
                     "layer_us": round(float(v[3]), 2), "combine_us": round(float(v[4]), 2)}
                    for q, v in enumerate(allr)]
    mean_ms = float(mean_ms)
    flushed_ms = torch.tensor(r["call_ms_flushed"], dtype=torch.float64, device=device).mean()
    if group is not None:
        dist.all_reduce(flushed_ms, op=dist.ReduceOp.MAX, group=group)

    e2e = time_e2e([inp], args.steps, warmup, group, combiner)
    e2e_ms = torch.tensor(e2e["ms"], dtype=torch.float64, device=device)
    if group is not None:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX, group=group)
    if combiner is not None:
        combiner.close()
        combiner = None

    # the kernel breakdown of the headline: the library's stage events at
    # N=1; at N>1 the same call on one GPU without the combine
    if group is None:
        stage = r["stage_ms"]
    else:
        stage = time_step([inp], max(5, args.steps // 2), warmup, flush, None, do_flush=not back_to_back,
                          flushed_too=False)["stage_ms"]
    kb, kf = kernel_bytes(st), kernel_flops(st)
    dominant = "gemm1" if stage["gemm1"] >= stage["gemm2"] else "gemm2"
    # a kernel is tensor-bound when its FLOPs at the dense e4m3 peak take
    # longer than its bytes at the HBM peak
    bound = ("tensor" if kf[dominant] / (2.0 * peaks["bf16_tflops"] * 1e12) > kb[dominant] / (peaks["hbm_gbs"] * 1e9)
             else "hbm")
    rl = roofline_entry(stage[dominant], kb[dominant], kf[dominant], peaks, bound)
    rl.update({"bound": bound, "kernel": dominant,
               "traffic": NCU_TRAFFIC_BYTES.get((dominant, HEADLINE_T)),
               "algorithmic_bytes": kb[dominant], "kernel_us": round(stage[dominant] * 1e3, 2),
               "algorithmic_flops": kf[dominant],
               "peak_source": (("measured HBM copy, MEASURED_PEAKS.json hbm_gbs" if bound == "hbm" else
                                "2 x measured cuBLAS bf16 burst (MEASURED_PEAKS.json bf16_tflops): dense e4m3")
                               if peaks["source"] == "measured" else "fallback 6.65 TB/s / 1.59 PFLOP/s")})

    # decode (T <= 64): front end, GEMM1, GEMM2, finalize; larger T: route,
    # permute (two kernels above 1024 tokens), gather, GEMM1, GEMM2, finalize,
    # and with bf16 hidden states the per-token quantiser first. At N>1 the
    # layer writes no output (no finalize) and the combine kernel follows,
    # so the count per call is the same.
    if HEADLINE_T <= 64:
        launches_per_call = 4
    else:
        launches_per_call = (6 if HEADLINE_T <= 1024 else 7) + (1 if BF16_HIDDEN else 0)
    line = {
        "metric": METRIC,
        "value": round(mean_ms * 1e3, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": round(mean_ms, 5),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8_e4m3 (fp32 accumulate)",
        "data": DATA,
        "config": headline_config(desc, HEADLINE_T, offset, st, world, back_to_back),
        "value_l2_write_flushed": round(float(flushed_ms) * 1e3, 2),
        "roofline": rl,
        "stages_us": {k: round(v * 1e3, 2) for k, v in stage.items()},
        "e2e": {"value": round(float(e2e_ms) * 1e3, 2), "unit": UNIT, "h2d_bytes_per_step": e2e["h2d"],
                "d2h_bytes_per_step": e2e["d2h"]},
        "gpu_launches": launches_per_call * args.steps,
        **({"per_rank": per_rank} if per_rank is not None else {}),
        **({"ep_check": check} if check is not None else {}),
        "clocks": clocks.summary(),
    }

    extras = not args.no_extras and args.workload == "decode" and not BF16_HIDDEN
    n_extra = max(5, args.steps // 2)
    if extras and world == 1:
        sweep = []
        for T in (1, 4, 16, 64):
            seed = first_seed_with_local_pick(T, device) if T == 1 else SEED
            p = point(T, "uniform", n_extra, warmup, flush, peaks, device, seed=seed)
            if T == 1:
                p["seed_rule"] = f"first seed >= {SEED} whose token picks a local expert"
            if T <= 16:
                p["fixed_latency_split"] = fixed_latency_split(p, n_extra, warmup, flush, peaks, device)
            sweep.append(p)
        line["sweep"] = sweep
        line["prefill"] = point(4096, "hot", n_extra, warmup, flush, peaks, device)
        # the reference's own Blackwell kernel on the same box and inputs
        line["reference_kernel"] = [
            reference_kernel_point(p["T"], p["variant"], p["seed"], n_extra, warmup, flush, device,
                                   p["us_per_call"]) for p in sweep + [line["prefill"]]]
    if extras:
        line["ep_t8192"] = all_shard_point(
            8192, "uniform", "config3: T=8192, all 256 experts in 8 shards, NVLink combine", n_extra, warmup,
            flush, peaks, device, group, world, rank)
        line["stress"] = all_shard_point(
            16384, "zipf", "config4 stress: T=16384, Zipf(1.2) expert popularity, all 256 experts in 8 shards",
            max(3, n_extra // 2), warmup, flush, peaks, device, group, world, rank)
        line["token_parallel_t8192"] = token_parallel_point(8192, max(3, n_extra // 2), warmup, peaks, device,
                                                            group, world, rank)
    if extras and world == 1:
        line["cpu_baseline"] = cpu_oracle_time(inp)
        c0 = workloads.make_inputs(16, 0, device)
        line["cpu_baseline_config0"] = cpu_oracle_time(c0)
        del c0
        # the other two sizes of the CPU baseline, on the sweep's T=1 inputs
        # and the prefill point's
        pts = []
        for T, variant, seed in ((1, "uniform", line["sweep"][0]["seed"]), (4096, "hot", SEED)):
            ci = workloads.make_inputs(T, seed, device, variant)
            pts.append({"T": T, "variant": variant, "seed": seed, **cpu_oracle_time(ci)})
            del ci
        line["cpu_baseline_points"] = pts

    if group is not None:
        dist.barrier(group=group)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if group is not None:
        torch.cuda.synchronize()
        dist.barrier(group=group)
        dist.destroy_process_group()


def run_reference(args, world: int, rank: int, warmup: int) -> None:
    """The reference algorithm on the host cores (rank 0 only): every step
    is one whole call of the CPU restatement (all active experts)."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import moe_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    HEADLINE_T, variant, desc = WORKLOADS[args.workload]
    # the inputs come from the same seeded generators on the same device as
    # our arm's (CPU and CUDA generators differ), so the tokens, routing and
    # weights are the same; only the active experts' weights are drawn, then
    # everything is copied to host memory outside the timing
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    r = workloads.make_routing_inputs(HEADLINE_T, SEED, dev, variant, 0)
    active = moe_oracle.active_local_experts(r["routing_logits"].cpu(), r["routing_bias"].cpu(), 2.5, 0)
    # the routing statistics of our arm's rank 0 (offset 0), from the
    # restatement's routing: the line's config is our arm's
    idx, _ = moe_oracle.route(r["routing_logits"].cpu(), r["routing_bias"].cpu(), 2.5)
    le = idx.long()
    local = (le >= 0) & (le < 32)
    counts = torch.bincount(le[local], minlength=32)
    st = {"T": HEADLINE_T, "E_act": int((counts > 0).sum()), "sum_Tk": int(counts.sum())}
    inp = workloads.make_inputs(HEADLINE_T, SEED, dev, variant, 0, 2.5, experts=active, weight_seed=SEED + 1)
    inp = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    if dev == "cuda":
        torch.cuda.empty_cache()
    cargs = workloads.as_args(inp)
    times = []
    for i in range(warmup + args.steps):
        t0 = time.perf_counter()
        moe_oracle.moe_forward(*cargs)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt * 1e6)
    v = statistics.mean(times)
    base = {"value": round(v, 1), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"T={HEADLINE_T}: every step one whole call (routing + all {len(active)} active experts)",
            "median_us": round(statistics.median(times), 1)}
    line = {
        "metric": METRIC, "value": round(v, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": warmup, "ms_per_step": round(v / 1e3, 3), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (dequantised e4m3)", "data": DATA,
        "config": headline_config(desc, HEADLINE_T, 0, st, world, weights_exceed_l2(st)),
        "impl": "reference",
        "cpu_baseline": base,
        "e2e": {"value": round(v, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
