#!/usr/bin/env python3
"""Decode benchmark: BF16 split-K attention decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl b200|reference]

One "step" is one decode call over the whole workload (every sequence of the
batch, one query token each).  Default workload: BASELINE cfg2 (Llama-3-8B
GQA: B=32, Hq=32, Hkv=8, D=128, S=4096), whose 512 MiB KV cache is larger
than the 126 MB L2, so consecutive steps stream from HBM without a flush.

Metric: achieved HBM GB/s = algorithmic bytes per step (valid K+V, Q read,
O write) / step time, summed over ranks; us/step is reported beside it.
Multi-GPU (torchrun, one process per GPU, NCCL): cfg1/2/3/5 are batch-sharded
with no collective; by default one global batch is split over the ranks
(strong scaling: B/N sequences per rank, token-balanced for cfg3), and
`--scaling weak` gives every rank a whole replica instead; cfg4 is sequence-sharded (each rank holds S/N tokens; the decode
kernel stores its partial states into every rank's exchange buffer over
NVLink and a merge kernel combines them on each rank, or with
`--transport nccl` the states are all-gathered over NCCL: strong scaling).

Timing: W warm-up steps and ~30 ms of further steps, a barrier and a
synchronize, a ~0.5 ms device-side hold (so that the first timed steps are
queued before they start), then K steps between CUDA events on the launching
stream, a synchronize and a barrier; the max over ranks.

`--impl reference` times the reference's CPU path on the host cores: the
torch FP32 decode of attention_decode/reference.py:47-60 (restated with the
same torch calls in oracle/reference_torch.py, all host threads) on the whole
workload (cfg5: its first 16 sequences), on rank 0 only.
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
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "hpc-ops-sm120_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

HBM_FALLBACK_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0
L2_BYTES = 126 * 1000 * 1000
METRIC = "decode achieved HBM GB/s (algorithmic valid K+V + Q + O bytes / step time)"


def parse_args():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--config", default="cfg2", choices=("cfg1", "cfg2", "cfg3", "cfg4", "cfg5"))
    p.add_argument("--impl", default="b200", choices=("b200", "reference", "ref-kernel", "sdpa", "fa2"),
                   help="b200: this library; reference: the reference's FP32 algorithm on host cores; "
                        "ref-kernel: the reference's CUDA kernel rebuilt for sm_100a (baseline/build_ref_kernel.py); "
                        "sdpa: torch scaled_dot_product_attention; fa2: flash_attn_with_kvcache "
                        "(comparison arms, 1 GPU)")
    p.add_argument("--kv", default="bf16", choices=("bf16", "fp8"),
                   help="K/V cache element type: bf16 (the reference's) or fp8 e4m3 with per-tensor scales "
                        "(attention_decode_fp8; head_dim 128)")
    p.add_argument("--scaling", default="strong", choices=("weak", "strong"),
                   help="N>1 batch-sharded configs: each rank decodes its share of one global batch "
                        "(strong, the default: B/N sequences, token-balanced for cfg3) or a whole replica "
                        "of the config (weak)")
    p.add_argument("--transport", default="p2p", choices=("p2p", "nccl"),
                   help="cfg4 at N>1: state exchange through NVLink peer memory (p2p) or an NCCL all_gather")
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--graph", type=int, default=0,
                   help="also time replays of a CUDA graph holding this many steps (0: off)")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle timing")
    p.add_argument("--e2e-steps", type=int, default=None, help="steps of the end-to-end pass (default: --steps, at most 500)")
    args = p.parse_args()
    if args.warmup < 3:
        p.error("--warmup must be at least 3")
    if args.steps < 1:
        p.error("--steps must be positive")
    return args


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            data = json.load(fh)
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy read+write)"
    except (OSError, KeyError, ValueError):
        return HBM_FALLBACK_GBS, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def profile_traffic(kernel_key: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as fh:
            return json.load(fh).get(kernel_key)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Clock/throttle samples around the timed region: nvidia-smi every 100 ms
    (the recipe's query) and, where the NVML bindings load, a thread reading
    the SM clock, the clock-event reasons and the power every ~2 ms (read-only
    queries), so that even a timed region of a few ms has samples inside it.
    ``mark_start``/``mark_stop`` bracket the timed region on the host."""

    NVML_REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
                    ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    FIELDS = (
        "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, device: torch.device):
        self.proc = None
        self.lines: list[str] = []
        self.target = None
        self.fast: list[tuple] = []  # (host time, sm MHz, reasons bitmask, power W)
        self.window = [None, None]
        self._stop_fast = threading.Event()
        self._fast_thread = None
        try:
            props = torch.cuda.get_device_properties(device)
            self.target = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        except Exception:
            self.target = None

    def _fast_loop(self, handle, nvml):
        while not self._stop_fast.is_set():
            try:
                self.fast.append((time.perf_counter(), nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM),
                                  nvml.nvmlDeviceGetCurrentClocksEventReasons(handle),
                                  nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0))
            except Exception:
                return
            time.sleep(0.002)

    def mark_start(self):
        self.window[0] = time.perf_counter()

    def mark_stop(self):
        self.window[1] = time.perf_counter()

    def start(self):
        try:
            import pynvml as nvml

            nvml.nvmlInit()
            handle = nvml.nvmlDeviceGetHandleByPciBusId(self.target) if self.target else nvml.nvmlDeviceGetHandleByIndex(0)
            self._fast_thread = threading.Thread(target=self._fast_loop, args=(handle, nvml), daemon=True)
            self._fast_thread.start()
        except Exception:
            self._fast_thread = None
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
        if self.target:
            cmd += ["-i", self.target]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def _fast_summary(self):
        self._stop_fast.set()
        if self._fast_thread is not None:
            self._fast_thread.join(timeout=2)
        t0, t1 = self.window
        inside = [x for x in self.fast if t0 is not None and t1 is not None and t0 <= x[0] <= t1]
        if not inside:
            return None
        reasons = sorted(name for name, bit in self.NVML_REASONS if any(x[2] & bit for x in inside))
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_mhz_min": min(x[1] for x in inside),
                "power_w_max": max(x[3] for x in inside), "reasons": reasons, "samples": len(inside)}

    def stop(self) -> dict:
        fast = self._fast_summary()
        if self.proc is None:
            out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
            if fast is not None:
                out.update(sm_mhz=fast["sm_mhz"], reasons=fast["reasons"], timed_region_nvml=fast)
            return out
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
                power.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        out = {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "power_w_max": max(power) if power else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }
        if fast is not None:
            # the timed region's own samples decide the median clock and the
            # reasons; the nvidia-smi samples (warm-up included) stay beside them
            out["nvidia_smi"] = {k: out[k] for k in ("sm_mhz", "power_w_max", "reasons", "samples")}
            out.update(sm_mhz=fast["sm_mhz"], power_w_max=fast["power_w_max"],
                       reasons=sorted(set(fast["reasons"]) | reasons), samples=fast["samples"],
                       sm_mhz_min=fast["sm_mhz_min"], source="NVML every 2 ms inside the timed region")
        return out


# ---------------------------------------------------------------- timed region
# The timed steps start behind a short device-side hold: torch's bounded
# cycle-count sleep kernel (~0.5 ms at the B200's 1.965 GHz) on the timing
# stream, launched after the barrier and synchronize and before the start
# event.  By the time it ends the host has queued the first timed steps, so a
# host-side pause while they are being launched (a thread switch, a driver
# query) does not enter the device time; the timed region itself is K whole
# steps on the device, unchanged.  The end-to-end pass has no hold.
HOLD_CYCLES = 1_000_000


def hold_queue():
    sleep = getattr(torch.cuda, "_sleep", None)  # a private torch helper: skip the hold if it is gone
    if sleep is not None:
        sleep(HOLD_CYCLES)


def timed_start_note():
    if getattr(torch.cuda, "_sleep", None) is None:
        return "right after the barrier and synchronize (no device-side hold available)"
    return f"behind a {HOLD_CYCLES}-cycle device-side hold (host launch jitter kept out)"


def settle(step, device, warmup, world=1):
    """Runs the W warm-up steps, then further steps for ~30 ms (SM clocks at
    their loaded operating point right before the timing); returns how many
    further steps ran.  Every rank runs the same count (sequence-sharded steps
    exchange states with all ranks)."""
    stream = torch.cuda.current_stream(device)
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0.record(stream)
    for _ in range(warmup):
        step()
    w1.record(stream)
    torch.cuda.synchronize(device)
    est_s = max_over_ranks(max(w0.elapsed_time(w1) * 1e-3 / warmup, 1e-6), world, device)
    extra = int(min(5000, max(0, 0.03 / est_s - warmup)))
    for _ in range(extra):
        step()
    torch.cuda.synchronize(device)
    return extra


# ---------------------------------------------------------------- CPU baseline
CPU_SAMPLE_BYTES = 1_100_000_000  # a step of the CPU arm streams at most ~1.1 GB


def cpu_sample_sequences(cfg, seqlens=None) -> int:
    """Sequences of the workload one CPU step covers: the whole batch when its
    bytes fit CPU_SAMPLE_BYTES (cfg1-cfg4), else the leading sequences that do
    (cfg5: 16 of 128)."""
    per_seq = [cfg.algorithmic_bytes(None) // cfg.batch] * cfg.batch if seqlens is None else [
        2 * 2 * cfg.head_dim * cfg.kv_heads * int(n) + 4 * cfg.query_heads * cfg.head_dim
        for n in seqlens.clamp(0, cfg.kv_len).tolist()]
    total, n = 0, 0
    for b in per_seq:
        if n and total + b > CPU_SAMPLE_BYTES:
            break
        total += b
        n += 1
    return n


def cpu_reference_step(q, k, v, seqlens):
    """One decode step of the reference's CPU path (reference.py:47-60,
    restated with the same torch calls in oracle/reference_torch.py)."""
    from oracle import reference_torch

    if seqlens is None:
        return reference_torch.reference_fp32(q, k, v)
    return reference_torch.reference_varlen_fp32(q, k, v, seqlens.tolist())


def cpu_step_bytes(cfg, q, seqlens) -> int:
    tokens = q.shape[0] * cfg.kv_len if seqlens is None else int(seqlens.clamp(0, cfg.kv_len).sum())
    return 2 * 2 * cfg.head_dim * cfg.kv_heads * tokens + 4 * q.shape[0] * cfg.query_heads * cfg.head_dim


def cpu_baseline_throughput(q, k, v, seqlens, cfg, budget_s: float):
    """The reference's CPU path on the host cores (all threads) over the
    same inputs as the GPU arm, copied to the host (untimed); whole steps are
    repeated until `budget_s` is spent.  Returns (GB/s, cores, sample)."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    n = cpu_sample_sequences(cfg, seqlens.cpu() if seqlens is not None else None)
    qc, kc, vc = (x[:n].cpu() for x in (q, k, v))
    lc = seqlens[:n].cpu() if seqlens is not None else None
    step_bytes = cpu_step_bytes(cfg, qc, lc)
    cpu_reference_step(qc, kc, vc, lc)  # warm-up
    elapsed, steps = 0.0, 0
    while elapsed < budget_s and steps < 200:
        t0 = time.perf_counter()
        cpu_reference_step(qc, kc, vc, lc)
        elapsed += time.perf_counter() - t0
        steps += 1
    what = "the whole step" if n == cfg.batch else f"{n} of {cfg.batch} sequences per step"
    sample = (f"{what} of {cfg.name} ({step_bytes / 1e9:.3f} GB), {steps} steps in {elapsed:.1f} s; "
              f"torch FP32 on CPU with {cores} threads (the reference's reference_fp32 calls, "
              f"oracle/reference_torch.py)")
    return step_bytes * steps / elapsed / 1e9, cores, sample


def run_reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from attention_decode.workloads import BASELINE_CONFIGS

    cfg = BASELINE_CONFIGS[args.config]
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    # The same seeded workload as the GPU arm, generated on the host; a step
    # is the whole workload (or, for cfg5, its leading 16 sequences).
    seqlens = cfg.make_seqlens(args.seed)
    n = cpu_sample_sequences(cfg, seqlens)
    q, k, v, lens = cfg.make_inputs("cpu", seed=args.seed, batch_slice=slice(0, n))
    step_bytes = cpu_step_bytes(cfg, q, lens)
    for _ in range(args.warmup):
        cpu_reference_step(q, k, v, lens)
    t_all = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(q, k, v, lens)
    sec_per_step = (time.perf_counter() - t_all) / args.steps
    value = step_bytes / sec_per_step / 1e9
    what = "the whole step" if n == cfg.batch else f"{n} of {cfg.batch} sequences per step"
    desc = (f"{what} of {cfg.name} ({step_bytes / 1e9:.3f} GB); torch FP32 on CPU with {cores} threads "
            f"(the reference's reference_fp32 calls, oracle/reference_torch.py)")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": sec_per_step * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) bf16 Q/K/V" + (", K ~ N(0,8^2) with x50 spikes" if cfg.extreme else "") + ")",
        "config": cfg.as_dict(),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm
def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def run_gpu_arm(args):
    rank, world, local_rank = dist_env()
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    import attention_decode as ad
    from attention_decode import _lib
    from attention_decode.workloads import BASELINE_CONFIGS

    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    cfg = BASELINE_CONFIGS[args.config]
    sequence_sharded = cfg.name == "cfg4" and world > 1
    if args.kv == "fp8" and (sequence_sharded or cfg.head_dim != 128):
        raise SystemExit("bench: --kv fp8 runs single-GPU / batch-sharded configs with head_dim 128")
    strong = args.scaling == "strong" and world > 1 and not sequence_sharded
    shard_index = None
    if strong and cfg.batch < world:
        # fewer sequences than ranks: there is no batch split to measure
        if rank == 0:
            print(json.dumps({"impl": "b200", "metric": METRIC, "config": cfg.as_dict(), "n_gpus": world,
                              "unavailable": f"{cfg.name} has {cfg.batch} sequence(s): a batch split over "
                                             f"{world} ranks leaves ranks empty (use --scaling weak)"}), flush=True)
        dist.destroy_process_group()
        return 0
    if strong:
        from attention_decode import sharded

        lengths = cfg.make_seqlens(args.seed)
        if lengths is not None:  # balance the streamed tokens across ranks
            shard_index = sharded.balance_by_tokens(lengths.tolist(), world)[rank]
        else:
            shard_index = list(range(cfg.batch))[sharded.batch_shard(cfg.batch, rank, world)]
        q, k, v, seqlens = cfg.make_inputs(device, seed=args.seed, batch_slice=shard_index)
    else:
        q, k, v, seqlens = cfg.make_inputs(device, seed=args.seed + (0 if sequence_sharded else 1009 * rank))
    if sequence_sharded:
        from attention_decode import sharded

        lo, hi = sharded.token_shard(cfg.kv_len, rank, world)
        k = k[:, :, lo:hi].contiguous()
        v = v[:, :, lo:hi].contiguous()
        torch.cuda.empty_cache()
        step_fn = sharded.SequenceShardedDecode(q, k, v, group=None, transport=args.transport)
        bytes_per_rank = 2 * 2 * cfg.head_dim * cfg.kv_heads * cfg.batch * (hi - lo) + (2 * 2 * cfg.batch * cfg.query_heads * cfg.head_dim if rank == 0 else 0)
        step = step_fn
        scaling = "strong"
        parallelism = (
            f"sequence-shard sp{world} (partial states stored to every rank over NVLink by the decode kernel, merged on each rank)"
            if args.transport == "p2p"
            else f"sequence-shard sp{world} (all_gather of partial states over NCCL)"
        )
    else:
        if strong:
            tokens = int(seqlens.clamp(0, cfg.kv_len).sum()) if seqlens is not None else len(shard_index) * cfg.kv_len
            bytes_per_rank = 2 * 2 * cfg.head_dim * cfg.kv_heads * tokens + 4 * len(shard_index) * cfg.query_heads * cfg.head_dim
        else:
            bytes_per_rank = cfg.algorithmic_bytes(seqlens)
        fp8_scales = None
        if args.kv == "fp8":
            # per-tensor e4m3 quantisation of the same K/V (amax -> 448); the
            # step then reads one byte per element
            ks = float(k.float().abs().max()) / 448.0
            vs = float(v.float().abs().max()) / 448.0
            k = (k.float() / ks).to(torch.float8_e4m3fn)
            v = (v.float() / vs).to(torch.float8_e4m3fn)
            torch.cuda.empty_cache()
            fp8_scales = (ks, vs)
            bytes_per_rank = (bytes_per_rank - 4 * cfg.batch * cfg.query_heads * cfg.head_dim) // 2 + \
                4 * cfg.batch * cfg.query_heads * cfg.head_dim
        sets, kv_total = rotation_sets(cfg, device, args.seed + 1009 * rank, (q, k, v), shard_index)
        if fp8_scales is not None:
            sets = [sets[0]] + [(qi, (ki.float() / fp8_scales[0]).to(torch.float8_e4m3fn),
                                 (vi.float() / fp8_scales[1]).to(torch.float8_e4m3fn)) for qi, ki, vi in sets[1:]]
        n_sets = len(sets)
        rotation = [0]

        def decode(qq, kk, vv, lens):
            if fp8_scales is not None:
                return ad.attention_decode_fp8(qq, kk, vv, lens, k_scale=fp8_scales[0], v_scale=fp8_scales[1])
            return ad.attention_decode(qq, kk, vv, lens)

        def step():
            i = rotation[0]
            rotation[0] = (i + 1) % n_sets
            qq, kk, vv = sets[i]
            return decode(qq, kk, vv, seqlens)

        scaling = "strong" if strong else "weak"
        if strong:
            parallelism = (f"batch-shard dp{world}, one global batch split over ranks "
                           f"({'token-balanced' if seqlens is not None else 'B/N sequences'} per rank, no collective)")
        else:
            parallelism = f"batch-shard dp{world} (no collective)" if world > 1 else "single GPU"

    # Correctness gate on a subset of sequences (full rows, CPU oracle).
    out = step()
    if not sequence_sharded:
        rotation[0] = 0
    torch.cuda.synchronize(device)
    check = {"rows_checked": 0, "max_abs_err": None}
    if not sequence_sharded or rank == 0:
        from oracle import attention_decode_oracle as oracle

        full_k, full_v = (k, v) if not sequence_sharded else (None, None)
        if full_k is not None:
            nb = min(2, q.shape[0])
            if args.kv == "fp8":
                bits = [q[:nb].contiguous().cpu().view(torch.int16).numpy().view(np.uint16)] + [
                    oracle.e4m3_to_f32(x[:nb].contiguous().cpu().view(torch.uint8).numpy()) * np.float32(sc)
                    for x, sc in ((full_k, fp8_scales[0]), (full_v, fp8_scales[1]))]
            else:
                bits = [x[:nb].contiguous().cpu().view(torch.int16).numpy().view(np.uint16) for x in (q, full_k, full_v)]
            if seqlens is None:
                want = oracle.reference_fp32(*bits)
            else:
                want = oracle.reference_varlen_fp32(*bits, seqlens[:nb].cpu().numpy())
            want = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(want))
            got = out[:nb].float().cpu().numpy()
            err = np.abs(got - want)
            if not (np.isfinite(got).all() and np.all(err <= 2e-2 + 1e-2 * np.abs(want))):
                raise SystemExit(f"bench: correctness gate failed (max abs err {err.max()})")
            check = {"rows_checked": int(nb * cfg.query_heads), "max_abs_err": float(err.max())}

    lib = _lib.load_library()
    launches0 = ctypes_count(lib)
    stream = torch.cuda.current_stream(device)
    # Clock samples cover the warm-up and the timed region; the sampler starts
    # first so that the GPU never idles between the warm-up and the timing (an
    # idle B200 lowers its SM clock within a fraction of a second and the first
    # steps after that run slower).
    sampler = ClockSampler(device)
    sampler.start()
    time.sleep(0.3)
    # Warm-up: the W steps asked for, then enough further steps to run the GPU
    # for ~30 ms, right before the timed steps.
    settle_steps = settle(step, device, args.warmup, world)

    # ---- device-timed region
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(device)
    launches_before = ctypes_count(lib)
    sampler.mark_start()
    hold_queue()
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize(device)
    sampler.mark_stop()
    launches_timed = ctypes_count(lib) - launches_before
    barrier(world)
    clocks = sampler.stop()
    error_word = ad.read_error_flag(local_rank)
    if error_word:
        raise SystemExit(f"bench: a kernel reported device error word {error_word} (bounded wait expired)")
    ms_step = start.elapsed_time(stop) / args.steps
    ms_step = max_over_ranks(ms_step, world, device)
    total_bytes = bytes_per_rank * (world if not sequence_sharded else 1)
    if sequence_sharded:
        total_bytes = cfg.algorithmic_bytes()
    if strong:
        total_bytes = cfg.algorithmic_bytes(cfg.make_seqlens(args.seed))
    value = total_bytes / (ms_step * 1e-3) / 1e9

    # ---- dominant kernel: event pairs around each streaming-kernel launch
    kernel_steps = min(args.steps, 500)
    _lib.check(lib, lib.adb_timing_enable(1))
    for _ in range(kernel_steps):
        step()
    _lib.check(lib, lib.adb_timing_enable(0))
    import ctypes

    tot_ms, n_launch = ctypes.c_double(0), ctypes.c_int64(0)
    _lib.check(lib, lib.adb_timing_read(ctypes.byref(tot_ms), ctypes.byref(n_launch)))
    isolated_ms = tot_ms.value / max(n_launch.value, 1)
    isolated_ms = max_over_ranks(isolated_ms, world, device)
    # Every step is exactly one decode_stream_kernel launch (plus, when
    # sequence-sharded, the state exchange and the small merge), so the kernel's
    # average duration in the timed region is the timed region over its
    # launches.  Event pairs around single launches (isolated_ms) also time
    # the launch latency that back-to-back launches hide.
    kernels_per_step = max(1, launches_timed // args.steps) if not sequence_sharded else 1
    kernel_ms = ms_step / kernels_per_step
    kernel_bytes = bytes_per_rank
    peak, peak_src = measured_peaks()
    achieved = kernel_bytes / (kernel_ms * 1e-3) / 1e9
    traffic = profile_traffic(f"{cfg.name}_decode_stream_kernel" + ("_fp8" if args.kv == "fp8" else ""))

    # ---- per-step distribution: events around each step of a separate pass
    # (the events between steps cut the programmatic-launch overlap, so the
    # median here sits above us_per_step)
    pct_n = min(args.steps, 300)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(pct_n)]
    torch.cuda.synchronize(device)
    for a, b in ev:
        a.record(stream)
        step()
        b.record(stream)
    torch.cuda.synchronize(device)
    per_step = sorted(a.elapsed_time(b) * 1e3 for a, b in ev)
    pct = {"p10": per_step[len(per_step) // 10], "p50": per_step[len(per_step) // 2],
           "p90": per_step[(9 * len(per_step)) // 10], "steps": pct_n}

    # ---- optional: the same steps replayed from a CUDA graph
    graph_line = None
    if args.graph > 0 and not sequence_sharded:
        gstream = torch.cuda.Stream(device=device)
        gstream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(gstream):
            for _ in range(3):
                step()
        torch.cuda.current_stream(device).wait_stream(gstream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gstream):
            for _ in range(args.graph):
                step()
        for _ in range(3):
            graph.replay()
        replays = max(1, args.steps // args.graph)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        g0.record(stream)
        for _ in range(replays):
            graph.replay()
        g1.record(stream)
        torch.cuda.synchronize(device)
        g_ms = g0.elapsed_time(g1) / (replays * args.graph)
        g_ms = max_over_ranks(g_ms, world, device)
        graph_line = {"steps_per_graph": args.graph, "replays": replays, "us_per_step": g_ms * 1e3,
                      "value": total_bytes / (g_ms * 1e-3) / 1e9}
        del graph

    # ---- end to end through the public API: pinned H2D of Q, decode, D2H of O
    e2e_steps = args.e2e_steps or min(args.steps, 500)
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()
    q_dev = torch.empty_like(q)
    lens_host = seqlens.cpu().pin_memory() if seqlens is not None else None
    lens_dev = torch.empty_like(seqlens) if seqlens is not None else None
    if sequence_sharded:
        e2e_call = step_fn.with_query(q_dev)
    else:
        e2e_rotation = [0]

        def e2e_call():  # the K/V caches rotate as in the timed region
            i = e2e_rotation[0]
            e2e_rotation[0] = (i + 1) % n_sets
            return decode(q_dev, sets[i][1], sets[i][2], lens_dev)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        if lens_host is not None:
            lens_dev.copy_(lens_host, non_blocking=True)
        o = e2e_call()
        out_host.copy_(o.view(out_host.shape), non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    barrier(world)
    e2e_s = max_over_ranks(e2e_s, world, device)
    h2d = q.numel() * 2 + (seqlens.numel() * 4 if seqlens is not None else 0)
    d2h = q.numel() * 2

    # ---- CPU baseline (rank 0, N=1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.kv == "bf16":
        gbs, cores, desc = cpu_baseline_throughput(q, k, v, seqlens, cfg, budget_s=10.0)
        cpu = {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": desc}

    if sequence_sharded or n_sets == 1:
        l2_note = "KV cache larger than the 126 MB L2: every step streams from HBM, no flush needed"
    else:
        l2_note = (f"KV cache smaller than L2: steps rotate among {n_sets} independent input sets "
                   f"({n_sets * kv_total / 1e6:.0f} MB > 2 x L2), so every step streams from HBM")
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "warmup_settle_steps": settle_steps,
            "timed_start": timed_start_note(),
            "ms_per_step": ms_step,
            "us_per_step": ms_step * 1e3,
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": "bf16" if args.kv == "bf16" else "e4m3 K/V (per-tensor scales), bf16 Q/O, f16 products, f32 softmax",
            "data": "synthetic (seeded N(0,1) bf16 Q/K/V" + (", K ~ N(0,8^2) with x50 spikes" if cfg.extreme else "") + ")",
            "config": dict(cfg.as_dict(), parallelism=parallelism, l2=l2_note, kv=args.kv),
            "pct_of_8tbs": 100.0 * (total_bytes / (ms_step * 1e-3) / 1e9) / (NOMINAL_HBM_GBS * (world if not sequence_sharded else world)),
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "kernel": "decode_stream_kernel (whole decode step, one launch)",
                "kernel_us": kernel_ms * 1e3,
                "kernel_us_isolated_launch": isolated_ms * 1e3,
                "peak_source": peak_src,
                "frac_of_8tbs": achieved / NOMINAL_HBM_GBS,
            },
            "cpu_baseline": cpu,
            "e2e": {
                "value": total_bytes / e2e_s / 1e9,
                "unit": "GB/s",
                "us_per_step": e2e_s * 1e6,
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "note": "per step: pinned H2D of Q, attention_decode() through the C ABI, D2H of O, host sync; the KV cache is resident decode state"
                        + ("" if sequence_sharded or n_sets == 1 else f" (rotating among the timed region's {n_sets} input sets)"),
            },
            "gpu_launches": launches_timed,
            "graph": graph_line,
            "per_step_us": pct,
            "clocks": clocks,
            "correctness": check,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        if sequence_sharded:
            step_fn.release()
        dist.destroy_process_group()
    del launches0
    return 0


def rotation_sets(cfg, device, seed, first, batch_slice=None):
    """Input sets that steps rotate among.  A KV cache smaller than twice the
    L2 would be served from L2 on the next step, so enough independent seeded
    sets are made that every step streams from HBM (the KV rotation of the
    reference's bench_extreme.py:103-107).  Every set has the shapes of
    `first`: the same sequences of the batch (`batch_slice`, a rank's share
    under strong scaling).  Returns (sets, KV bytes per set)."""
    q, k, v = first
    kv_total = 2 * k.numel() * k.element_size()
    n_sets = 1 if kv_total >= 2 * L2_BYTES else min(64, -(-2 * L2_BYTES // kv_total))
    sets = [(q, k, v)]
    for i in range(1, n_sets):
        qi, ki, vi, _ = cfg.make_inputs(device, seed=seed + 7919 * i, batch_slice=batch_slice)
        assert ki.shape == k.shape and qi.shape == q.shape
        sets.append((qi, ki, vi))
    return sets, kv_total


def run_comparison_arm(args):
    """Another GPU implementation of the same step on the same inputs, timed
    like this library's arm (events around --steps back-to-back calls): the
    reference's own kernel rebuilt for sm_100a, or torch SDPA.  One GPU; other
    ranks exit."""
    rank, world, local_rank = dist_env()
    if rank != 0:
        return 0
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    import attention_decode as ad
    from attention_decode.workloads import BASELINE_CONFIGS

    cfg = BASELINE_CONFIGS[args.config]

    def unavailable(why):
        print(json.dumps({"impl": args.impl, "config": cfg.as_dict(), "unavailable": why}), flush=True)
        return 0

    if world > 1:
        return unavailable("comparison arms run on one GPU")
    q, k, v, seqlens = cfg.make_inputs(device, seed=args.seed + 1009 * rank)
    if args.impl == "ref-kernel":
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        import importlib.util

        from build_ref_kernel import MODULE, module_path

        path = module_path()
        if not path.is_file():
            return unavailable(f"{path} not built (python baseline/build_ref_kernel.py --reference-root <checkout>)")
        group = cfg.query_heads // cfg.kv_heads
        if seqlens is not None:
            return unavailable("reference kernel has no sequence lengths (csrc/decode.cu:223-258)")
        if group not in (1, 4):
            return unavailable(f"reference kernel supports GQA groups 1 and 4, not {group} (csrc/decode.cu:239)")
        if k.numel() > 2**31 - 1:
            return unavailable("reference kernel limits tensors to INT_MAX elements (csrc/decode.cu:231)")
        spec = importlib.util.spec_from_file_location(MODULE, str(path))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)

        def call(qq, kk, vv):
            return mod.forward(qq, kk, vv)

        label = "reference csrc/decode.cu rebuilt for sm_100a (capability gate relaxed, otherwise unchanged)"
    elif args.impl == "fa2":
        try:
            from flash_attn import flash_attn_with_kvcache
        except Exception as exc:  # not installed or no kernels for this build
            return unavailable(f"flash_attn import failed: {type(exc).__name__}: {exc}"[:300])
        cache_lens = seqlens.to(torch.int32) if seqlens is not None else None

        def call(qq, kk, vv):
            # flash_attn reads [B, S, H, D] caches and [B, 1, Hq, D] queries;
            # the layout change of the cache is made once per input set, below
            out = flash_attn_with_kvcache(qq.transpose(1, 2), kk, vv, cache_seqlens=cache_lens)
            return out.transpose(1, 2)

        label = "flash_attn.flash_attn_with_kvcache (cache transposed to [B, S, Hkv, D] once, outside the timing)"
    else:
        import torch.nn.functional as F

        mask = None
        if seqlens is not None:
            mask = (torch.arange(cfg.kv_len, device=device)[None, :] < seqlens[:, None].long())[:, None, None, :]

        def call(qq, kk, vv):
            return F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, enable_gqa=True)

        label = "torch.nn.functional.scaled_dot_product_attention(enable_gqa=True" + (", boolean padding mask)" if mask is not None else ")")
    want = ad.attention_decode(q, k, v, seqlens)
    sets, _ = rotation_sets(cfg, device, args.seed + 1009 * rank, (q, k, v))
    if args.impl == "fa2":
        sets = [(qi, ki.transpose(1, 2).contiguous(), vi.transpose(1, 2).contiguous()) for qi, ki, vi in sets]
        q, k, v = sets[0]
        torch.cuda.empty_cache()
    try:
        out = call(q, k, v)
        torch.cuda.synchronize(device)
    except Exception as exc:
        return unavailable(f"{args.impl} call failed: {type(exc).__name__}: {exc}"[:300])
    max_err = float((out.float() - want.float()).abs().max())
    rotation = [0]

    def step():
        i = rotation[0]
        rotation[0] = (i + 1) % len(sets)
        return call(*sets[i])

    # the same warm-up, settle and hold as this library's arm
    sampler = ClockSampler(device)
    sampler.start()
    time.sleep(0.3)
    settle_steps = settle(step, device, args.warmup)
    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    sampler.mark_start()
    hold_queue()
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize(device)
    sampler.mark_stop()
    clocks = sampler.stop()
    ms_step = start.elapsed_time(stop) / args.steps
    total_bytes = cfg.algorithmic_bytes(seqlens)
    line = {
        "impl": args.impl,
        "metric": METRIC,
        "value": total_bytes / (ms_step * 1e-3) / 1e9,
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "warmup_settle_steps": settle_steps,
        "timed_start": timed_start_note(),
        "ms_per_step": ms_step,
        "us_per_step": ms_step * 1e3,
        "higher_is_better": True,
        "dtype": "bf16",
        "config": cfg.as_dict(),
        "implementation": label,
        "input_sets": len(sets),
        "max_abs_diff_vs_b200": max_err,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


def ctypes_count(lib) -> int:
    import ctypes

    n = ctypes.c_int64(0)
    lib.adb_launch_count(ctypes.byref(n))
    return n.value


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.impl in ("ref-kernel", "sdpa", "fa2"):
        return run_comparison_arm(args)
    return run_gpu_arm(args)


if __name__ == "__main__":
    raise SystemExit(main())
