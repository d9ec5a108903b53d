"""Benchmark: Boltz-2 Pairformer ms/block at N = 512 (bf16 trunk contract).

One step = one full Pairformer block (TriMulOut, TriMulIn, TriAttStart,
TriAttEnd, Transition(z), then the fp32 single track) applied to z in place on
synthetic seeded inputs: z ~ N(0,1) [1, 512, 512, 128] fp32, s ~ N(0,1)
[1, 512, 384], masks all ones, weights ~ N(0, 1/128) with unit-mean norm
weights.  Consecutive steps chain like the trunk's consecutive blocks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

With N > 1 the driver starts one rank per GPU (torch.distributed.run); every
rank runs its own independent block (separate inputs, no collective in the
data path: weak scaling) and the step time is the max over ranks.  Rank 0
prints one JSON line.  ``--impl reference`` times the CPU restatement of the
reference path (the oracle) on this host's cores instead; under torchrun only
rank 0 runs it.
"""

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Pairformer ms/block at N=512 bf16"
UNIT = "ms/block"
N_TOKENS = 512
C_S, C_Z = 384, 128
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--n", type=int, default=N_TOKENS, help="tokens (default 512, the metric's config)")
    # The end-to-end pipeline's fill (first input copy) and drain (last
    # output copy) are inside the timed region; 24 steps amortise them the
    # way a longer job would (at ~3 ms per step the region stays < 0.1 s).
    p.add_argument("--e2e-steps", type=int, default=64)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-sub-records", action="store_true",
                   help="skip the row-sharded N=2048 block and the diffusion sampler sub-records")
    p.add_argument("--sharded", action="store_true",
                   help="one block at --n (default 2048) row-sharded over the ranks (strong scaling)")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            data = json.loads(path.read_text())
            return {k: float(data[k]) for k in FALLBACK_PEAKS}, "measured"
        except (KeyError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def seeded_block(cls, seed=1234):
    """Weights ~ N(0, 1/128), norm weights N(1, 1/128), from a fixed CPU generator."""
    module = cls()
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            mean = 1.0 if "norm" in name and name.endswith("weight") else 0.0
            p.copy_(torch.randn(p.shape, generator=g) * (1.0 / 128) ** 0.5 + mean)
    return module.eval()


def synthetic_inputs(n, seed):
    g = torch.Generator().manual_seed(seed)
    s = torch.randn(1, n, C_S, generator=g)
    z = torch.randn(1, n, n, C_Z, generator=g)
    mask = torch.ones(1, n)
    pair_mask = torch.ones(1, n, n)
    return s, z, mask, pair_mask


def bench_config(n, world):
    """The workload description shared by both arms."""
    return {"workload": f"Pairformer block N={n} (TriMulOut+In, TriAttStart+End, Transition(z), single track)",
            "tokens": n, "c_s": C_S, "c_z": C_Z, "heads": "4x32", "parallelism": f"dp{world} (one block per GPU)",
            "l2": "inputs larger than L2: z 128 MiB fp32 plus per-op intermediates up to 256 MiB"}


def max_over_ranks(value, dist, device):
    """Max of a per-rank float over the process group (identity without one)."""
    if dist is None:
        return value
    t = torch.tensor([float(value)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_info():
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return model


# ---------------------------------------------------------------------------
# CPU restatement of the reference path (oracle), bounded sample
# ---------------------------------------------------------------------------
def cpu_block_sample(n):
    """Time one full Pairformer block of the CPU oracle at n tokens on all host
    threads: every op runs over the whole pair tensor (no row sampling, no
    extrapolation).  Returns (ms, sample description, threads)."""
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref = seeded_block(oracle.PairformerLayer)
    s, z, mask, pair_mask = synthetic_inputs(n, seed=99)
    timings = {}
    with torch.inference_mode():
        t_start = time.perf_counter()
        for name in ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end"):
            t = time.perf_counter()
            z = z + getattr(ref, name)(z, pair_mask)
            timings[name] = time.perf_counter() - t
        t = time.perf_counter()
        z = z + ref.transition_z(z)
        timings["transition_z"] = time.perf_counter() - t
        t = time.perf_counter()
        sn = torch.nn.functional.layer_norm(s, (C_S,), ref.pre_norm_s.weight, ref.pre_norm_s.bias, 1e-5)
        s = s + ref.attention(sn, z, mask, sn)
        s = s + ref.transition_s(s, bf16=False)
        timings["single_track"] = time.perf_counter() - t
        total_ms = 1000.0 * (time.perf_counter() - t_start)
    assert torch.isfinite(z).all() and torch.isfinite(s).all()
    sample = (f"one full Pairformer block at N={n} (every op over the whole pair tensor) on {threads} threads "
              f"({cpu_info()}); parts_s=" + json.dumps({k: round(v, 3) for k, v in timings.items()}))
    return total_ms, sample, threads


def run_reference(args):
    """Reference arm: the CPU restatement of the reference path (the oracle),
    one full block per step, on this host's cores; rank 0 only."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    n = args.n
    t_run = time.perf_counter()
    for _ in range(args.warmup):
        cpu_block_sample(n)
    values = []
    sample = ""
    threads = os.cpu_count() or 1
    t_timed = time.perf_counter()
    for _ in range(args.steps):
        ms, sample, threads = cpu_block_sample(n)
        values.append(ms)
    timed_s = time.perf_counter() - t_timed
    value = statistics.mean(values)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16-rounding oracle)", "data": "synthetic",
        "config": bench_config(n, world),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                         "min_ms": round(min(values), 3), "max_ms": round(max(values), 3)},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": {"timed_steps": round(timed_s, 2), "whole_run": round(time.perf_counter() - t_run, 2)},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def algorithmic_work(name, a):
    """(kind, amount per launch, label) of one C-ABI call, from its arguments."""
    if name == "bl_batched_gemm":
        batch, m, n, k = a[11], a[12], a[13], a[14]
        return "flops", 2.0 * batch * m * n * k, f"bl_batched_gemm[b={batch},m={m},n={n},k={k}]"
    if name in ("bl_triangle_attention", "bl_triangle_attention_residual"):
        # q k^T and p v: 4 N^2 n_outer H d; the residual form adds linear_o (2 N n_outer 128^2)
        heads, d, n, n_outer = a[14], a[15], a[16], a[17]
        label = f"{name}[n={n},heads={heads},d={d}]" if n_outer == n else \
            f"{name}[n={n},n_outer={n_outer},heads={heads},d={d}]"
        flops = 4.0 * n * n * n_outer * heads * d
        if name == "bl_triangle_attention_residual":
            flops += 2.0 * n * n_outer * 128 * 128
        return "flops", flops, label
    if name == "bl_layernorm":
        size = {0: 4, 1: 2}
        rows, cols = a[2], a[3]
        return "bytes", rows * cols * (size[a[1]] + size[a[9]]), f"bl_layernorm[rows={rows},cols={cols}]"
    if name == "bl_swiglu_rows":
        rows, width = a[2], a[3]
        return "bytes", rows * width * 6, f"bl_swiglu_rows[rows={rows},width={width}]"
    if name == "bl_gate":
        return "bytes", a[3] * 6, f"bl_gate[n={a[3]}]"
    # Fused pair kernels: bytes each must move per pair row (128 channels).
    if name == "bl_attention_projection":  # fp32 row in, q|k|v|g bf16 out, 4 bf16 bias values
        n, rows = a[1], a[1] * a[2]
        return "bytes", rows * (512 + 1024 + 8), f"bl_attention_projection[n={n}]"
    if name == "bl_trimul_projection":  # fp32 row in, 256 gated channels + x_hat (bf16) out
        n, rows = a[1], a[1] * a[2]
        return "bytes", rows * (512 + 512 + 256), f"bl_trimul_projection[n={n}]"
    if name == "bl_trimul_output":  # 128 plane values + x_hat in, z read-modify-write (or bf16 out)
        n, rows = a[1], a[1] * a[2]
        out = 1024 if a[9] else 256
        return "bytes", rows * (256 + 256 + out), f"bl_trimul_output[n={n}]"
    if name == "bl_pair_transition":  # LN read + z read-modify-write (or bf16 out)
        rows = a[1]
        return "bytes", rows * (512 + (1024 if a[7] else 256)), f"bl_pair_transition[rows={rows}]"
    if name == "bl_pair_bias":
        rows, heads = a[1], a[6]
        return "bytes", rows * (512 + 4 * heads), f"bl_pair_bias[rows={rows},heads={heads}]"
    return "bytes", 0.0, name


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 20 ms from before
    the warm-up; ``stop(window)`` keeps the samples taken inside the timed
    region (host monotonic times)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device, interval_ms=20):
        self.samples = []  # (host monotonic seconds, fields)
        self.proc = None
        self.first = threading.Event()
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(interval_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, RuntimeError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append((time.monotonic(), parts))
                self.first.set()

    def wait_ready(self, timeout=10.0):
        """Block until nvidia-smi has produced its first sample (it takes a moment to start)."""
        if self.proc is not None:
            self.first.wait(timeout)

    def stop(self, window):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.05)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        t0, t1 = window
        inside = [parts for t, parts in self.samples if t0 <= t <= t1]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, sm_max, reasons = [], [], set()
        for parts in inside:
            try:
                sm.append(float(parts[0]))
                sm_max.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(sm_max) if sm_max else None,
                "reasons": sorted(reasons), "samples": len(sm), "interval_ms": 20,
                "timed_region_s": round(t1 - t0, 4)}


def run_b200(args):
    world, rank, local = dist_env()
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist_mod

        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        dist = dist_mod

    from boltz_lumi_b200 import _lib, layers

    n = args.n
    block = seeded_block(layers.PairformerLayer).to(device)
    s_h, z_h, mask_h, pmask_h = synthetic_inputs(n, seed=1000 + rank)
    s, z, mask, pmask = (t.to(device) for t in (s_h, z_h, mask_h, pmask_h))

    def step():
        nonlocal s, z
        s, z = block(s, z, mask, pmask)

    def barrier():
        if dist is not None:
            dist.barrier()

    clocks = ClockSampler(device)
    clocks.wait_ready()
    with torch.inference_mode():
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()

        # Untimed profiling step: per-call device time of every C-ABI entry point.
        observer = _lib.CallObserver(timed=("*",))
        _lib.set_observer(observer)
        step()
        _lib.set_observer(None)
        torch.cuda.synchronize()
        launches_per_step = observer.calls
        per_label = {}
        for name, a, e0, e1 in observer.records:
            kind, amount, label = algorithmic_work(name, a)
            entry = per_label.setdefault(label, {"name": name, "kind": kind, "amount": amount, "ms": 0.0, "n": 0})
            entry["ms"] += e0.elapsed_time(e1)
            entry["n"] += 1
        top_label = max(per_label, key=lambda k: per_label[k]["ms"])
        top = per_label[top_label]

        # Timed region: K chained blocks; the dominant kernel is event-timed in place.
        observer = _lib.CallObserver(timed=(top["name"],))
        barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _lib.set_observer(observer)
        t0 = time.monotonic()
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
        t1 = time.monotonic()
        _lib.set_observer(None)
        barrier()
        clock_info = clocks.stop((t0, t1))
        elapsed_ms = start.elapsed_time(end)
        launches_timed = observer.calls
        top_times = [e0.elapsed_time(e1) for name, a, e0, e1 in observer.records
                     if algorithmic_work(name, a)[2] == top_label]
        elapsed_ms = max_over_ranks(elapsed_ms, dist, device)
        ms_per_step = elapsed_ms / args.steps
        value = ms_per_step / world  # aggregate: `world` blocks complete per step

        # End to end through the public module API with pinned host buffers.
        z_host = z_h.pin_memory()
        s_host = s_h.pin_memory()
        z_back = torch.empty_like(z_host).pin_memory()
        s_back = torch.empty_like(s_host).pin_memory()
        h2d = z_host.numel() * 4 + s_host.numel() * 4 + mask_h.numel() * 4 + pmask_h.numel() * 4
        d2h = z_back.numel() * 4 + s_back.numel() * 4
        # Three streams, four device buffer sets: the host->device copy of
        # step k + 1 and the device->host copy of step k - 1 run while step k
        # computes (PCIe is full duplex).  A buffer set is held from its input
        # copy to the end of its output copy; with four sets the two copy
        # directions run back to back even when one of them jitters (measured:
        # 3.2 ms per step with four sets, 3.4-4.5 ms with three).  Every step
        # still moves all of its inputs in and all of z and s out.
        nbuf = 4
        mask_host, pmask_host = mask_h.pin_memory(), pmask_h.pin_memory()
        bufs = [{"z": torch.empty_like(z_h, device=device), "s": torch.empty_like(s_h, device=device),
                 "m": torch.empty_like(mask_h, device=device), "p": torch.empty_like(pmask_h, device=device)}
                for _ in range(nbuf)]
        s_in, s_comp, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_in = [torch.cuda.Event() for _ in range(nbuf)]
        ev_comp = [torch.cuda.Event() for _ in range(nbuf)]
        ev_out = [torch.cuda.Event() for _ in range(nbuf)]
        outputs = [None] * nbuf
        barrier()
        torch.cuda.synchronize()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(s_in)
        s_comp.wait_event(e_start)
        s_out.wait_event(e_start)
        steps_e2e = args.e2e_steps
        for k in range(steps_e2e + 2):
            if k < steps_e2e:  # inputs of step k
                b = bufs[k % nbuf]
                if k >= nbuf:
                    s_in.wait_event(ev_out[k % nbuf])  # step k - nbuf has left this buffer set
                with torch.cuda.stream(s_in):
                    b["z"].copy_(z_host, non_blocking=True)
                    b["s"].copy_(s_host, non_blocking=True)
                    b["m"].copy_(mask_host, non_blocking=True)
                    b["p"].copy_(pmask_host, non_blocking=True)
                ev_in[k % nbuf].record(s_in)
            j = k - 1
            if 0 <= j < steps_e2e:  # compute step j
                b = bufs[j % nbuf]
                s_comp.wait_event(ev_in[j % nbuf])
                with torch.cuda.stream(s_comp):
                    outputs[j % nbuf] = block(b["s"], b["z"], b["m"], b["p"])
                ev_comp[j % nbuf].record(s_comp)
            j = k - 2
            if 0 <= j < steps_e2e:  # results of step j
                so, zo = outputs[j % nbuf]
                s_out.wait_event(ev_comp[j % nbuf])
                with torch.cuda.stream(s_out):
                    z_back.copy_(zo, non_blocking=True)
                    s_back.copy_(so, non_blocking=True)
                ev_out[j % nbuf].record(s_out)
        e_end.record(s_out)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e_start.elapsed_time(e_end)
        e2e_ms = max_over_ranks(e2e_ms, dist, device)
        e2e_value = e2e_ms / args.e2e_steps / world
        assert torch.isfinite(z_back).all() and torch.isfinite(s_back).all(), "non-finite block output"
        status = _lib.device_status(reset=True)
        if status:
            raise RuntimeError(f"device-side bounded wait timed out (status {status:#x})")

    peaks, peak_source = load_peaks()
    avg_ms = statistics.mean(top_times) if top_times else top["ms"] / max(top["n"], 1)
    # The burst GEMM figure for a timed region shorter than a second (the clocks
    # stay at their maximum there), the sustained one for a longer region.
    region_s = (clock_info or {}).get("timed_region_s") or elapsed_ms / 1e3
    peak_key = "bf16_tflops" if region_s < 1.0 else "bf16_tflops_sustained"
    if top["kind"] == "flops":
        achieved = top["amount"] / (avg_ms * 1e-3) / 1e12
        peak = peaks[peak_key]
        roofline = {"bound": "tensor", "unit": "TFLOP/s"}
    else:
        achieved = top["amount"] / (avg_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        roofline = {"bound": "hbm", "unit": "GB/s"}
    roofline.update({
        "achieved": round(achieved, 2), "peak": peak, "frac": round(achieved / peak, 4),
        "traffic": traffic_for(top_label), "kernel": top_label, "avg_launch_ms": round(avg_ms, 4),
        "launches_timed": len(top_times), "algorithmic_per_launch": top["amount"],
        "peak_source": f"{peak_source} ({peak_key if top['kind'] == 'flops' else 'hbm_gbs'}; "
                       f"timed region {region_s:.3f} s)",
    })

    roofline_sfu = None
    if top_label.startswith("bl_triangle_attention"):
        # The attention core's other bound (the exponentials): one ex2
        # per score on the MUFU pipe, 16 per clock per SM.  The peak is derived
        # from that rate, the SM count and the sampled SM clock (there is no
        # measured SFU figure).
        dims = {key: int(val) for key, val in re.findall(r"(\w+)=(\d+)", top_label)}
        exps = float(dims["n"] ** 2 * dims.get("n_outer", dims["n"]) * dims["heads"])  # one per score
        clock_mhz = (clock_info or {}).get("sm_mhz") or 1965.0
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        sfu_peak = 16 * sms * clock_mhz * 1e6
        sfu_achieved = exps / (avg_ms * 1e-3)
        roofline_sfu = {"bound": "sfu", "unit": "ex2/s", "achieved": float(f"{sfu_achieved:.4g}"),
                        "peak": float(f"{sfu_peak:.4g}"), "frac": round(sfu_achieved / sfu_peak, 4),
                        "kernel": top_label, "exps_per_launch": exps,
                        "peak_source": f"derived: 16 ex2/clk/SM x {sms} SMs x {clock_mhz:.0f} MHz (sampled)"}

    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 4), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) inputs, N(0,1/128) weights)",
        "config": bench_config(n, world),
        "e2e": {"value": round(e2e_value, 4), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": args.e2e_steps,
                "pipeline": "pinned host buffers; H2D of step k+1 and D2H of step k-1 overlap step k (3 streams, 4 device buffer sets)"},
        "gpu_launches": launches_timed,
        "launches_per_step": launches_per_step,
        "roofline": roofline,
        **({"roofline_sfu": roofline_sfu} if roofline_sfu else {}),
        "clocks": clock_info,
        "kernels_ms_per_step": {k: round(v["ms"], 4) for k, v in sorted(per_label.items(), key=lambda kv: -kv[1]["ms"])},
    }
    if not args.no_sub_records:
        # Multi-GPU partitions beyond the replica headline: the row-sharded N = 2048 block
        # (strong scaling, NCCL collectives) and the sample-parallel diffusion sampler
        # (one input per GPU).  Every rank takes part; rank 0 reports.
        line["sharded"] = measure_sharded(2048, min(args.steps, 10), 2, 2, dist, device)
        line["diffusion"] = measure_diffusion(dist, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # Same procedure as the reference arm: one untimed warm-up block, then one timed block.
        cpu_block_sample(n)
        cpu_ms, sample, threads = cpu_block_sample(n)
        line["cpu_baseline"] = {"value": round(cpu_ms, 2), "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def traffic_for(label):
    """DRAM bytes per launch of `label` from the committed ncu summary, if one exists."""
    for path in sorted((ROOT / "profiles").glob("*.md")):
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:") and label in line:
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


def measure_sharded(n, steps, warmup, e2e_steps, dist, device):
    """One Pairformer block at n tokens row-sharded over the ranks (each rank holds
    n / world rows of z; the channel regrouping of the triangle-multiplication planes,
    the row <-> column transposes and the bias gathers run on NCCL over NVLink).  Total work per step is fixed (strong scaling).  Returns the
    record (device time per block, max over ranks) on every rank."""
    from boltz_lumi_b200 import _lib, layers
    from boltz_lumi_b200.sharded import ShardedPairformer, SingleComm, TorchComm

    comm = TorchComm() if dist is not None else SingleComm()
    world, rank = comm.world, comm.rank
    n_loc = n // world
    block = seeded_block(layers.PairformerLayer).to(device)
    s_h, z_h, mask_h, pmask_h = synthetic_inputs(n, seed=1000)  # one block, split by rows
    zr_h = z_h[0, rank * n_loc:(rank + 1) * n_loc].contiguous()
    del z_h
    s, mask, pmask = s_h.to(device), mask_h.to(device), pmask_h.to(device)
    z_rows = zr_h.to(device)
    sharded = ShardedPairformer(block, comm)

    def barrier():
        if dist is not None:
            dist.barrier()

    with torch.inference_mode():
        for _ in range(max(warmup, 1)):
            s, z_rows = sharded(s, z_rows, mask, pmask)
        torch.cuda.synchronize()
        observer = _lib.CallObserver(timed=())
        _lib.set_observer(observer)
        barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            s, z_rows = sharded(s, z_rows, mask, pmask)
        end.record()
        torch.cuda.synchronize()
        _lib.set_observer(None)
        barrier()
        ms = max_over_ranks(start.elapsed_time(end), dist, device) / steps
        launches = observer.calls
        # End to end: this rank's rows and s in from pinned memory, back out, every step.
        zr_pin, s_pin = zr_h.pin_memory(), s_h.pin_memory()
        z_back, s_back = torch.empty_like(zr_pin).pin_memory(), torch.empty_like(s_pin).pin_memory()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            zd, sd = zr_pin.to(device, non_blocking=True), s_pin.to(device, non_blocking=True)
            so, zo = sharded(sd, zd, mask, pmask)
            z_back.copy_(zo, non_blocking=True)
            s_back.copy_(so, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e = max_over_ranks(e0.elapsed_time(e1), dist, device) / e2e_steps
        assert torch.isfinite(z_back).all() and torch.isfinite(s_back).all(), "non-finite block output"
    flops = 4.0 * n ** 3 * 4 * 32 * 2 + 2 * 2.0 * 128 * n ** 3 + 2.0 * n * n * (128 * 1024 + 512 * 128)
    return {
        "metric": f"Pairformer ms/block at N={n} row-sharded bf16", "value": round(ms, 4), "unit": UNIT,
        "n_gpus": world, "steps": steps, "warmup": max(warmup, 1), "ms_per_step": round(ms, 4),
        "higher_is_better": False, "scaling": "strong",
        "workload": f"one Pairformer block N={n}, z rows split over {world} GPU(s) "
                    "(triangle-multiplication products channel-sharded through all_to_all, row/column "
                    "transposes around the ending-node attention, all_gather of the bias rows and s; NCCL)",
        "tokens": n, "rows_per_gpu": n_loc, "parallelism": f"row-sharded x{world}",
        "e2e": {"value": round(e2e, 4), "unit": UNIT, "h2d_bytes_per_step": zr_pin.numel() * 4 + s_pin.numel() * 4,
                "d2h_bytes_per_step": zr_pin.numel() * 4 + s_pin.numel() * 4, "steps": e2e_steps},
        "gpu_launches": launches,
        "tensor_tflops_pair_ops": round(flops / (ms * 1e-3) / 1e12, 1),
    }


DIFFUSION = {"tokens": 384, "steps": 200, "multiplicity": 5, "depth": 24, "c_token": 768, "heads": 16}


def measure_diffusion(dist, device, steps=DIFFUSION["steps"]):
    """Predictions per hour of the sample-parallel diffusion sampler (one input per GPU,
    its multiplicity samples on that GPU, weak scaling; boltz_lumi_b200.sampling): the
    200-step EDM sampler of AF3 Algorithm 18 over a 24-layer token transformer of this
    package's diffusion kernels, coordinates gathered with one all_gather at the end.
    Time = device time of the whole sampling call (max over ranks)."""
    from boltz_lumi_b200 import sampling
    from boltz_lumi_b200.sharded import SingleComm, TorchComm

    comm = TorchComm() if dist is not None else SingleComm()
    cfg = DIFFUSION
    n, mult = cfg["tokens"], cfg["multiplicity"]
    model = sampling.seeded_model(depth=cfg["depth"], c_token=cfg["c_token"], heads=cfg["heads"], seed=5,
                                  device=device)
    inputs = [sampling.synthetic_conditioning(n, cfg["depth"], cfg["heads"], seed=100 + i, device=device)
              for i in range(comm.world)]

    denoisers = {}

    def runner(sampler):
        def run(i, samples, gens):
            if i not in denoisers:  # one CUDA-graphed score model per input, kept across calls
                denoisers[i] = sampling.make_denoiser(model, *inputs[i], cuda_graphs=True)
            return sampler.sample(denoisers[i], n, gens, device)
        return run

    with torch.inference_mode():
        sampling.distributed_sample(runner(sampling.EDMSampler(steps=3)), comm.world, mult, n, 1, comm, device)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        coords = sampling.distributed_sample(runner(sampling.EDMSampler(steps=steps)), comm.world, mult, n, 2,
                                             comm, device)
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1), dist, device)
        assert torch.isfinite(coords).all(), "non-finite coordinates"
    return {
        "metric": "predictions/hour (sample-parallel diffusion sampler, one input per GPU)",
        "value": round(comm.world * 3600e3 / ms, 2), "unit": "predictions/hour", "higher_is_better": True,
        "n_gpus": comm.world, "scaling": "weak", "seconds_per_prediction": round(ms / 1e3, 3),
        "workload": (f"{cfg['tokens']} tokens, {steps} EDM steps, multiplicity {mult}, {cfg['depth']}-layer token "
                     f"transformer (c={cfg['c_token']}, {cfg['heads']} heads) on this package's diffusion kernels, "
                     "score model replayed from a CUDA graph; coordinates of all inputs x samples gathered on "
                     "every rank"),
        "data": "synthetic (seeded trunk conditioning and weights)",
    }


def run_sharded(args):
    """``--sharded``: the row-sharded block alone, as its own JSON line."""
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist_mod

        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        dist = dist_mod
    n = args.n if args.n != N_TOKENS else 2048
    clocks = ClockSampler(device)
    clocks.wait_ready()
    t0 = time.monotonic()
    record = measure_sharded(n, args.steps, args.warmup, args.e2e_steps, dist, device)
    clock_info = clocks.stop((t0, time.monotonic()))
    if rank == 0:
        line = dict(record)
        line.update({"vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) inputs, N(0,1/128) weights)",
                     "config": {"workload": record.pop("workload"), "tokens": n, "parallelism": record["parallelism"],
                                "l2": "inputs larger than L2 (z slab >= 256 MiB fp32)"},
                     "clocks": clock_info, "cpu_baseline": None})
        line.pop("workload", None)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.sharded:
        return run_sharded(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
