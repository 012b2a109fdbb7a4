"""Benchmark: BF16 GB/s encoded per quant type.

Default workload (--workload kquant): the single-tensor encoder sweep, 4096
rows x 14336 columns of BF16 (N(0, 0.02) with 0.1% outliers at +-8 sigma,
per-column log-normal imatrix with sigma 1.5) to Q4_K, Q5_K, Q6_K and Q8_0.
--workload iq: the IQ codebook configuration, [4096 x 4096] and
[14336 x 4096] Student-t tensors to every IQ type.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step encodes every tensor once to every type.  `value` is device-resident
(inputs in HBM); `e2e` goes through the host-buffer C-ABI entry point with
pinned host input and output.  L2 (126 MB) is flushed before every timed
encode.  Under torchrun every rank encodes its own copy (weak scaling, no
collective on the data path); the time is the max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_ROWS, NE0 = 4096, 14336
SEED = 20261201
SWEEP = ["Q4_K", "Q5_K", "Q6_K", "Q8_0"]
METRIC = "BF16 GB/s encoded per quant type"
TYPE_IDS = {"Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ2_XS": 17, "IQ3_XXS": 18,
            "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23}
OUT_BYTES_PER_ELT = {"Q8_0": 34 / 32, "Q2_K": 84 / 256, "Q3_K": 110 / 256, "Q4_K": 144 / 256, "Q5_K": 176 / 256, "Q6_K": 210 / 256,
                     "IQ2_XXS": 66 / 256, "IQ2_XS": 74 / 256, "IQ2_S": 82 / 256, "IQ3_XXS": 98 / 256,
                     "IQ3_S": 110 / 256, "IQ4_NL": 18 / 32, "IQ4_XS": 136 / 256}
# Algorithmic f32 operations per input element of the reference encoders,
# counted by executing the oracle's op-counting build (oracle/opcount) on 32
# evenly spaced rows of each benchmark tensor: every f32 add, sub, mul, div,
# sqrt, compare, min/max and round-to-integer executed by the algorithm as
# written (no CSE or hoisting credited), data-dependent neighbour searches
# included.  The kernels execute fewer operations than this (loop invariants
# hoisted, products shared), so the figure is the work done, not the
# instructions issued.
FLOPS_PER_ELT = {"Q4_K": 745.4, "Q5_K": 745.4, "Q6_K": 151.0, "Q8_0": 5.1, "Q2_K": 768.8, "Q3_K": 152.1,
                 "IQ2_XXS": 1839.0, "IQ2_XS": 3738.2, "IQ2_S": 713.8, "IQ3_XXS": 1498.4, "IQ3_S": 963.8,
                 "IQ4_NL": 274.7, "IQ4_XS": 274.7}
# FP32 ceiling for separately rounded adds and multiplies on sm_100: 128 per
# clock per SM, scalar or packed f32x2 alike (shoehorn_b200/fp32-rate measures
# 121-126 for add-only/mul-only chains); fused multiply-adds would reach 250
# flops/clk/SM but are excluded by the parity contract.
FP32_OPS_PER_CLK_PER_SM = 128


IQ_TYPES = ["IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ4_NL", "IQ4_XS"]


def _to_bf16(w):
    u = w.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # RNE to BF16


def make_workload(seed=SEED):
    """Encoder sweep: 4096 rows x 14336, N(0, 0.02) + 0.1% outliers at +-8 sigma,
    imatrix log-normal (sigma 1.5)."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((N_ROWS, NE0), dtype=np.float32)
    w *= np.float32(0.02)
    k = int(round(w.size * 0.001))
    idx = rng.choice(w.size, size=k, replace=False)
    w.reshape(-1)[idx] = rng.choice(np.array([-0.16, 0.16], dtype=np.float32), size=k)
    im = np.exp(rng.normal(0.0, 1.5, size=NE0)).astype(np.float32)
    return _to_bf16(w), im


def make_iq_workload(seed=SEED):
    """IQ codebook config: [4096 rows x 4096] and [14336 rows x 4096] Student-t
    (nu=5) scaled to std 0.02, imatrix log-normal (sigma 1)."""
    out = []
    for i, rows in enumerate((4096, 14336)):
        rng = np.random.default_rng(seed + 1 + i)
        w = (rng.standard_t(5.0, size=(rows, 4096)) * (0.02 / np.sqrt(5.0 / 3.0))).astype(np.float32)
        im = np.exp(rng.normal(0.0, 1.0, size=4096)).astype(np.float32)
        out.append((f"{rows}x4096", _to_bf16(w), im))
    return out


def workload_tensors(name):
    if name == "iq":
        return make_iq_workload()
    bits, im = make_workload()
    return [(f"{N_ROWS}x{NE0}", bits, im)]


def captured_traffic(type_name, in_bytes):
    """DRAM bytes per launch of a type's encoder from the committed ncu capture
    (profiles/traffic_encoder_sweep.txt), for the 4096 x 14336 tensor only."""
    path = os.path.join(ROOT, "profiles", "traffic_encoder_sweep.txt")
    if in_bytes != N_ROWS * NE0 * 2 or not os.path.exists(path):
        return None
    for line in open(path):
        f = line.split()
        if len(f) >= 4 and not line.startswith("#") and f[1] == type_name:
            return int(f[2]) + int(f[3])
    return None


def max_over_ranks(x, dev):
    """The maximum of a per-rank float over all ranks (one all-reduce outside
    any timed region); x itself when no process group is running."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    tt = torch.tensor([float(x)], device=dev, dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    return float(tt.item())


def aggregate_gbs(world, n_types, in_bytes, seconds):
    """Whole-job BF16 GB/s for weak scaling: every rank encodes its own copy of
    the workload to every type, and the job takes the slowest rank's time."""
    return world * n_types * in_bytes / seconds / 1e9


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), ws


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax.append(float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(tensors, types, budget_s=12.0):
    """The reference algorithm (the C restatement in oracle/) on host cores:
    a bounded sample of rows of the same tensors per type."""
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    per_type = {}
    tot_bytes, tot_t = 0, 0.0
    samples = []
    for name in types:
        ty = TYPE_IDS[name]
        b_bytes, b_t = 0, 0.0
        for tname, bits, im in tensors:
            ne0 = bits.shape[1]
            rows = 16
            t0 = time.perf_counter()
            O.encode_tensor_bf16(ty, bits[:rows], im, n_threads=cores)
            dt = time.perf_counter() - t0
            target = budget_s / len(types) / len(tensors)
            rows = int(min(bits.shape[0], max(rows, rows * target / max(dt, 1e-3) * 0.8)))
            rows = max(min(cores, bits.shape[0]), rows - rows % cores)
            t0 = time.perf_counter()
            O.encode_tensor_bf16(ty, bits[:rows], im, n_threads=cores)
            dt = time.perf_counter() - t0
            b_bytes += rows * ne0 * 2
            b_t += dt
            samples.append(f"{name} {tname}: first {rows} rows")
        per_type[name] = b_bytes / b_t / 1e9
        tot_bytes += b_bytes
        tot_t += b_t
    return {"value": tot_bytes / tot_t / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "per_type": {k: round(v, 5) for k, v in per_type.items()}, "sample": "; ".join(samples)}


def workload_label(args, tensors, types):
    shapes = " + ".join(t[0] for t in tensors)
    return f"{'IQ codebook' if args.workload == 'iq' else 'encoder sweep'} {shapes} BF16 ({','.join(types)}), imatrix-weighted"


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    tensors = workload_tensors(args.workload)
    types = args.types.split(",")
    for _ in range(args.warmup):
        cpu_baseline(tensors, types, budget_s=2.0)
    vals = []
    cb = None
    t_start = time.perf_counter()
    for _ in range(args.steps):
        cb = cpu_baseline(tensors, types, budget_s=args.ref_budget)
        vals.append(cb["value"])
    wall = time.perf_counter() - t_start
    value = statistics.median(vals)
    line = {"metric": METRIC, "value": round(value, 5), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": workload_label(args, tensors, types), "types": types, "l2": "n/a (host CPU)"},
            "cpu_baseline": {"value": round(value, 5), "unit": "GB/s", "cores": cb["cores"], "kind": "port",
                             "sample": cb["sample"]},
            "e2e": {"value": round(value, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "per_type_gbs": cb["per_type"]}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    import shoehorn_b200 as sh

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local_rank)
    ctx = sh.Context(local_rank)
    types = [t for t in args.types.split(",") if sh.type_supported(TYPE_IDS[t])]
    tensors = workload_tensors(args.workload)
    dtens = []
    for tname, bits, im in tensors:
        src = torch.from_numpy(bits.view(np.int16)).to(dev)
        imt = torch.from_numpy(im).to(dev)
        outs = {t: torch.empty((bits.shape[0], sh.row_bytes(TYPE_IDS[t], bits.shape[1])), dtype=torch.uint8,
                               device=dev) for t in types}
        dtens.append((tname, src, imt, outs))
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def encode(t, d):
        ctx.encode_rows(TYPE_IDS[t], d[1], d[2], out=d[3][t], stream=stream)

    for _ in range(args.warmup):
        for t in types:
            for d in dtens:
                flush.zero_()
                encode(t, d)
    ctx.sync(stream)
    torch.cuda.synchronize()

    ev = {(t, i): [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)] for t in types for i in range(len(dtens))}
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    smi_index = int(vis[local_rank]) if len(vis) > local_rank and vis[local_rank].isdigit() else local_rank
    sampler = ClockSampler(smi_index)
    sampler.start()
    launches0 = ctx.launch_count()
    for k in range(args.steps):
        for t in types:
            for i, d in enumerate(dtens):
                flush.zero_()  # evict the input from L2 before every timed encode
                s, e = ev[(t, i)][k]
                s.record(stream)
                encode(t, d)
                e.record(stream)
    torch.cuda.synchronize()
    launches = ctx.launch_count() - launches0
    ctx.sync(stream)
    # per type: median over steps of the summed tensor times
    per_type_ms, per_type_min = {}, {}
    for t in types:
        steps_ms = [sum(ev[(t, i)][k][0].elapsed_time(ev[(t, i)][k][1]) for i in range(len(dtens)))
                    for k in range(args.steps)]
        per_type_ms[t] = statistics.median(steps_ms)
        per_type_min[t] = min(steps_ms)
    step_ms = max_over_ranks(sum(per_type_ms.values()), dev)

    # end to end: host (pinned) buffers through the C-ABI host entry point
    htens = []
    for (tname, bits, im), d in zip(tensors, dtens):
        src_h = torch.from_numpy(bits.view(np.int16)).pin_memory()
        outs_h = {t: torch.empty(tuple(d[3][t].shape), dtype=torch.uint8).pin_memory() for t in types}
        htens.append((src_h, im, outs_h))
    for t in types:
        for src_h, im, outs_h in htens:
            ctx.encode_tensor_host(TYPE_IDS[t], src_h, im, out=outs_h[t])
    if world > 1:
        dist.barrier()
    e2e_t = {t: [] for t in types}
    for _ in range(max(1, min(args.steps, 3))):
        for t in types:
            t0 = time.perf_counter()
            for src_h, im, outs_h in htens:
                ctx.encode_tensor_host(TYPE_IDS[t], src_h, im, out=outs_h[t])
            e2e_t[t].append(time.perf_counter() - t0)
    e2e_step = max_over_ranks(sum(statistics.median(v) for v in e2e_t.values()), dev)
    clocks = sampler.stop()

    in_bytes = sum(int(d[1].numel()) * 2 for d in dtens)
    elts = in_bytes // 2
    value = aggregate_gbs(world, len(types), in_bytes, step_ms * 1e-3)
    e2e_value = aggregate_gbs(world, len(types), in_bytes, e2e_step)
    per_type = {t: round(in_bytes / (per_type_ms[t] * 1e-3) / 1e9, 3) for t in types}

    # roofline of the dominant kernel (largest share of the step)
    dom = max(types, key=lambda t: per_type_ms[t])
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}
    props = torch.cuda.get_device_properties(dev)
    sm_mhz = clocks.get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)
    if dom == "Q8_0":
        alg = elts * (2 + OUT_BYTES_PER_ELT[dom])
        hbm = peaks.get("hbm_gbs", 6650.0)
        roof = {"bound": "hbm", "achieved": round(alg / (per_type_ms[dom] * 1e-3) / 1e9, 2), "peak": hbm,
                "unit": "GB/s",
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if "hbm_gbs" in peaks else "fallback"}
    else:
        alg = elts * FLOPS_PER_ELT[dom]
        # no multiply-add contraction is allowed (parity), so the ceiling is
        # separate f32 adds/multiplies
        peak = props.multi_processor_count * FP32_OPS_PER_CLK_PER_SM * sm_mhz * 1e6 / 1e12
        roof = {"bound": "fp32", "achieved": round(alg / (per_type_ms[dom] * 1e-3) / 1e12, 3),
                "peak": round(peak, 3), "unit": "TFLOP/s",
                "peak_source": f"{props.multi_processor_count} SMs x {FP32_OPS_PER_CLK_PER_SM} separate f32 add/mul "
                               f"per clock (no FMA by the parity contract; 121-126 measured by fp32-rate) x median "
                               f"SM clock {sm_mhz:.0f} MHz (MEASURED_PEAKS.json has no FP32 figure)",
                "flops_per_elt": FLOPS_PER_ELT[dom], "flops_source": "oracle op-count build, as-written algorithm"}
    roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
    roof["kernel"] = f"{dom} encoder"
    roof["traffic"] = captured_traffic(dom, in_bytes)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(tensors, types, budget_s=args.ref_budget)

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": workload_label(args, tensors, types), "types": types,
                           "tensors": [t[0] for t in tensors],
                           "l2": "flushed (512 MB write) before every timed encode",
                           "parallelism": f"weak: each of {world} ranks encodes its own copy"},
                "per_type_gbs": per_type,
                "per_type_ms": {t: round(v, 4) for t, v in per_type_ms.items()},
                "per_type_ms_min": {t: round(v, 4) for t, v in per_type_min.items()},
                "e2e": {"value": round(e2e_value, 3), "unit": "GB/s",
                        "h2d_bytes_per_step": len(types) * in_bytes,
                        "d2h_bytes_per_step": sum(int(d[3][t].numel()) for d in dtens for t in types)},
                "roofline": roof, "clocks": clocks, "gpu_launches": launches,
                "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="kquant", choices=["kquant", "iq"])
    ap.add_argument("--types", default=None, help="comma-separated types (default: the workload's)")
    ap.add_argument("--ref-budget", type=float, default=12.0, help="seconds of CPU work per reference sample")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    if args.types is None:
        args.types = ",".join(IQ_TYPES if args.workload == "iq" else SWEEP)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
