"""Benchmark: BF16 GB/s encoded per quant type, and the Llama-3-8B-shape
error-table + solve + encode wall time, on 1..N GPUs of one box.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--sections sweep,iq,model] [--no-cpu]

Sections of one run (all by default; the JSON line's headline `value` is the
sweep's):
  sweep  the single-tensor encoder sweep: 4096 rows x 14336 BF16 (N(0, 0.02)
         with 0.1% outliers at +-8 sigma, per-column log-normal imatrix,
         sigma 1.5) to Q4_K, Q5_K, Q6_K and Q8_0.  A step encodes the tensor
         once to every type.
  iq     the IQ codebook configuration: [4096 x 4096] and [14336 x 4096]
         Student-t (nu 5) tensors with a log-normal (sigma 1) imatrix, to every
         IQ type.  Reported per type beside the sweep.
  model  the Llama-3-8B shape (synthetic BF16 weights N(0, 0.02), log-normal
         imatrix): the full error table (the reference's 128-row sampling, and
         every row), the solve for a 5.5 GiB weight budget and the encode of
         the chosen mix, through the host pipeline library.

Under torchrun (one process per GPU, NCCL) every section shards rows: rank r
of N owns rows [n*r/N, n*(r+1)/N) of every tensor (the row-range sharding of
the pipeline), so the total work is fixed and N GPUs share it (strong
scaling).  Nothing crosses ranks on the data path; the model section
all-gathers the per-row f64 errors once, before the solve.  Times are taken
per rank and the job's time is the slowest rank's.

`value` is device-resident (inputs in HBM; the L2 is flushed by a read of a
512 MB buffer before every timed encode); `e2e` goes through the host-buffer
C-ABI entry point (pinned host input and output, copies inside the timing).
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

from shoehorn_b200 import workloads  # noqa: E402

SWEEP = ["Q4_K", "Q5_K", "Q6_K", "Q8_0"]
IQ_TYPES = ["IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ4_NL", "IQ4_XS"]
METRIC = "BF16 GB/s encoded per quant type"
TYPE_IDS = {"Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ2_XS": 17,
            "IQ3_XXS": 18, "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "F16": 1}
OUT_BYTES_PER_ELT = {"Q8_0": 34 / 32, "Q2_K": 84 / 256, "Q3_K": 110 / 256, "Q4_K": 144 / 256, "Q5_K": 176 / 256,
                     "Q6_K": 210 / 256, "IQ2_XXS": 66 / 256, "IQ2_XS": 74 / 256, "IQ2_S": 82 / 256,
                     "IQ3_XXS": 98 / 256, "IQ3_S": 110 / 256, "IQ4_NL": 18 / 32, "IQ4_XS": 136 / 256}
# Algorithmic f32 operations per input element of the reference encoders,
# counted by executing the oracle's op-counting build (oracle/opcount) on 32
# evenly spaced rows of each benchmark tensor: every f32 add, sub, mul, div,
# sqrt, compare, min/max and round-to-integer executed by the algorithm as
# written (no CSE or hoisting credited), data-dependent neighbour searches
# included.  The kernels execute fewer operations than this (loop invariants
# hoisted, products shared, repeated grids skipped), so the figure is the
# work done, not the instructions issued.
FLOPS_PER_ELT = {"Q4_K": 745.4, "Q5_K": 745.4, "Q6_K": 151.0, "Q8_0": 5.1, "Q2_K": 768.8, "Q3_K": 152.1,
                 "IQ2_XXS": 1839.0, "IQ2_XS": 3738.2, "IQ2_S": 713.8, "IQ3_XXS": 1498.4, "IQ3_S": 963.8,
                 "IQ4_NL": 274.7, "IQ4_XS": 274.7}
# FP32 ceiling for separately rounded adds and multiplies on sm_100: 128 per
# clock per SM (an issue-rate probe measured 121 scalar and 126 packed f32x2
# add-only or mul-only operations per clock per SM); fused multiply-adds would
# reach 256 flops/clk/SM but are excluded by the parity contract.
FP32_OPS_PER_CLK_PER_SM = 128
# Model-level configurations: shape (layers, hidden, KV width, FFN, vocab),
# weight budget, and whether the weights are held in host memory or
# generated as the pipeline streams them (the 70B shape's 141 GB of BF16 is
# never held).  --budget = weight budget + f16 KV at ctx 8192 + the
# compute estimate, with --reserve 0 (main.rs:294-337).
MODEL_CTX = 8192
MODELS = {
    "llama3-8b": {"layers": 32, "hidden": 4096, "kv": 1024, "ffn": 14336, "vocab": 128256, "budget_gib": 5.5,
                  "streaming": False,
                  "workload": "Llama-3-8B shape (32 layers, hidden 4096, GQA 32/8, FFN 14336, vocab 128256 untied), "
                              "synthetic BF16 N(0, 0.02), log-normal imatrix; weight budget 5.5 GiB"},
    "llama3-70b": {"layers": 80, "hidden": 8192, "kv": 1024, "ffn": 28672, "vocab": 128256, "budget_gib": 40.0,
                   "streaming": True,
                   "workload": "Llama-3-70B shape (80 layers, hidden 8192, GQA 64/8, FFN 28672, vocab 128256 untied), "
                               "synthetic BF16 N(0, 0.015) generated as it streams, log-normal imatrix with 1% of "
                               "columns x100; weight budget 40 GiB; encoded bytes copied to the host and discarded"},
}


def model_budget_arg(name):
    """The --budget that leaves exactly the configuration's weight budget."""
    m = MODELS[name]
    kv = m["layers"] * MODEL_CTX * 8 * (128 + 128) * 2
    compute = 512 * m["vocab"] * 4 + 512 * m["hidden"] * 4 * 8
    return str(int(m["budget_gib"] * (1 << 30)) + kv + compute)


def shard_rows(n, rank, world):
    return n * rank // world, n * (rank + 1) // world


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


def aggregate_gbs(total_in_bytes, n_types, seconds):
    """Whole-job BF16 GB/s: the full tensors' bytes, encoded once to each type,
    over the slowest rank's time (the ranks share the rows)."""
    return n_types * total_in_bytes / seconds / 1e9


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


# ---------------------------------------------------------------------------
# CPU baselines: the reference algorithm (the C restatement in oracle/) on the
# host cores, on bounded samples of the same workloads.
# ---------------------------------------------------------------------------
def cpu_baseline(tensors, types, budget_s=12.0):
    """Per type: the first rows of each tensor, sized to ~budget_s of CPU work
    in total.  GB/s of BF16 input."""
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    per_type, samples = {}, []
    tot_bytes, tot_t = 0, 0.0
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


def model_shapes(name="llama3-8b"):
    """(name, ne0, n_rows, candidates, count) of a model configuration's
    solvable tensors, one entry per distinct shape (main.rs:347-380 ladder:
    11 candidates, 6 for token_embd/output)."""
    m = MODELS[name]
    L, E, KV, FF, V = m["layers"], m["hidden"], m["kv"], m["ffn"], m["vocab"]
    big = ["IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ4_XS", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "F16"]
    small = ["IQ4_XS", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "F16"]
    return [("attn_q", E, E, big, L), ("attn_k", E, KV, big, L), ("attn_v", E, KV, big, L),
            ("attn_output", E, E, big, L), ("ffn_gate", E, FF, big, L), ("ffn_up", E, FF, big, L),
            ("ffn_down", FF, E, big, L), ("token_embd", E, V, small, 1), ("output", E, V, small, 1)]


def cpu_model_baseline(mix_elements, name="llama3-8b"):
    """The reference's error table and encode for a model configuration on
    the host cores, extrapolated from a sample: per tensor shape, the error
    of `rows` rows (of the 128 the reference samples) for every candidate;
    per type of the chosen mix, the encode of a 4096-wide slab.  Synthetic
    rows with the configuration's distribution (N(0, 0.02) BF16, log-normal
    imatrix)."""
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(7)
    rows = max(cores, 16)
    sample = []
    measure_s = 0.0
    exact_s = 0.0
    for tname, ne0, n_rows, cands, count in model_shapes(name):
        bits = workloads.to_bf16((rng.standard_normal((rows, ne0), dtype=np.float32) * np.float32(0.02)))
        im = np.exp(rng.normal(0.0, 1.0, size=ne0)).astype(np.float32)
        t0 = time.perf_counter()
        for c in cands:
            O.row_errors_bf16(TYPE_IDS[c], bits, None if tname == "token_embd" else im, n_threads=cores)
        dt = time.perf_counter() - t0
        sampled = min(128, n_rows)
        measure_s += dt * sampled / rows * count
        exact_s += dt * n_rows / rows * count
        sample.append(f"{tname}: {rows} rows x {len(cands)} candidates")
    encode_s = 0.0
    bits = workloads.to_bf16(rng.standard_normal((rows * 4, 4096), dtype=np.float32) * np.float32(0.02))
    im = np.exp(rng.normal(0.0, 1.0, size=4096)).astype(np.float32)
    for ty, elems in mix_elements.items():
        if ty not in TYPE_IDS or ty == "F16":
            continue
        t0 = time.perf_counter()
        O.encode_tensor_bf16(TYPE_IDS[ty], bits, im, n_threads=cores)
        dt = time.perf_counter() - t0
        encode_s += dt * elems / bits.size
        sample.append(f"encode {ty}: {bits.shape[0]} rows x 4096")
    return {"measure_s": round(measure_s, 3), "measure_exact_s": round(exact_s, 2), "encode_s": round(encode_s, 2),
            "wall_s": round(measure_s + encode_s, 2), "wall_exact_s": round(exact_s + encode_s, 2), "cores": cores,
            "kind": "port", "sample": "; ".join(sample) + " (extrapolated by rows and elements per type)"}


# ---------------------------------------------------------------------------
# GPU sections
# ---------------------------------------------------------------------------
class Timer:
    def __init__(self, torch, stream):
        self.torch, self.stream = torch, stream

    def __call__(self, fn):
        s = self.torch.cuda.Event(enable_timing=True)
        e = self.torch.cuda.Event(enable_timing=True)
        s.record(self.stream)
        fn()
        e.record(self.stream)
        return s, e


def run_encode_section(sh, torch, ctx, dev, stream, tensors, types, steps, warmup, rank, world, flush):
    """Device-resident encode of this rank's rows of every tensor to every type,
    then the same through the host-buffer entry point.  Returns per-rank
    timings (ms per step, per type)."""
    dtens = []
    for tname, bits, im in tensors:
        lo, hi = shard_rows(bits.shape[0], rank, world)
        src = torch.from_numpy(bits[lo:hi].view(np.int16)).to(dev)
        imt = torch.from_numpy(im).to(dev)
        outs = {t: torch.empty((hi - lo, sh.row_bytes(TYPE_IDS[t], bits.shape[1])), dtype=torch.uint8, device=dev)
                for t in types}
        dtens.append((tname, src, imt, outs, lo))

    def encode(t, d):
        ctx.encode_rows(TYPE_IDS[t], d[1], d[2], row0=d[4], out=d[3][t], stream=stream)

    def evict():
        # evict the inputs from L2 by reading 512 MB (a write would leave dirty
        # lines whose write-back lands inside the next timed encode)
        flush.max()

    timer = Timer(torch, stream)
    for _ in range(warmup):
        for t in types:
            for d in dtens:
                evict()
                encode(t, d)
    ctx.sync(stream)
    torch.cuda.synchronize()
    ev = {(t, i): [] for t in types for i in range(len(dtens))}
    launches0 = ctx.launch_count()
    for _ in range(steps):
        for t in types:
            for i, d in enumerate(dtens):
                evict()
                ev[(t, i)].append(timer(lambda: encode(t, d)))
    torch.cuda.synchronize()
    launches = ctx.launch_count() - launches0
    ctx.sync(stream)
    per_type_ms, per_type_min = {}, {}
    for t in types:
        steps_ms = [sum(ev[(t, i)][k][0].elapsed_time(ev[(t, i)][k][1]) for i in range(len(dtens)))
                    for k in range(steps)]
        per_type_ms[t] = statistics.median(steps_ms)
        per_type_min[t] = min(steps_ms)
    # end to end: this rank's rows from pinned host memory through the C ABI
    htens = []
    for (tname, bits, im), d in zip(tensors, dtens):
        lo, hi = shard_rows(bits.shape[0], rank, world)
        src_h = torch.from_numpy(bits[lo:hi].view(np.int16)).pin_memory()
        outs_h = {t: torch.empty(tuple(d[3][t].shape), dtype=torch.uint8).pin_memory() for t in types}
        htens.append((src_h, im, outs_h, lo))
    for t in types:
        for src_h, im, outs_h, lo in htens:
            ctx.encode_tensor_host(TYPE_IDS[t], src_h, im, row0=lo, out=outs_h[t])
    e2e_t = {t: [] for t in types}
    for _ in range(max(1, min(steps, 3))):
        for t in types:
            t0 = time.perf_counter()
            for src_h, im, outs_h, lo in htens:
                ctx.encode_tensor_host(TYPE_IDS[t], src_h, im, row0=lo, out=outs_h[t])
            e2e_t[t].append(time.perf_counter() - t0)
    e2e_per_type = {t: statistics.median(v) for t, v in e2e_t.items()}
    rank_elts = sum(int(d[1].numel()) for d in dtens)
    out_bytes = sum(int(d[3][t].numel()) for d in dtens for t in types)
    return {"per_type_ms": per_type_ms, "per_type_min": per_type_min, "e2e_per_type_s": e2e_per_type,
            "launches": launches, "rank_elts": rank_elts, "rank_out_bytes": out_bytes}


def roofline_for(t, elts, ms, sm_mhz, n_sms, peaks):
    """Roofline of one type's encode call (one launch over `elts` elements in
    `ms`): HBM for Q8_0, separate f32 add/mul issue for the rest."""
    if t == "Q8_0":
        alg = elts * (2 + OUT_BYTES_PER_ELT[t])
        hbm = peaks.get("hbm_gbs", 6650.0)
        r = {"bound": "hbm", "achieved": round(alg / (ms * 1e-3) / 1e9, 2), "peak": hbm, "unit": "GB/s",
             "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks else "fallback 6650"}
    else:
        alg = elts * FLOPS_PER_ELT[t]
        peak = n_sms * FP32_OPS_PER_CLK_PER_SM * sm_mhz * 1e6 / 1e12
        r = {"bound": "fp32", "achieved": round(alg / (ms * 1e-3) / 1e12, 3), "peak": round(peak, 3),
             "unit": "TFLOP/s",
             "peak_source": f"{n_sms} SMs x {FP32_OPS_PER_CLK_PER_SM} separate f32 add/mul per clock x median SM "
                            f"clock {sm_mhz:.0f} MHz (MEASURED_PEAKS.json has no FP32 figure)",
             "flops_per_elt": FLOPS_PER_ELT[t], "flops_source": "oracle op-count build, as-written algorithm"}
    r["frac"] = round(r["achieved"] / r["peak"], 4)
    return r


def captured_traffic(type_name, elts):
    """DRAM bytes per launch of a type's encoder from the committed ncu capture
    (profiles/traffic_encoder_sweep.txt, one launch over the whole 4096 x
    14336 tensor), scaled to `elts` elements."""
    path = os.path.join(ROOT, "profiles", "traffic_encoder_sweep.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        f = line.split()
        if len(f) >= 4 and not line.startswith("#") and f[1] == type_name:
            return int((int(f[2]) + int(f[3])) * elts / (4096 * 14336))
    return None


def run_ours(args):
    import torch
    import torch.distributed as dist
    import shoehorn_b200 as sh

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    dev = torch.device("cuda", local_rank)
    ctx = sh.Context(local_rank)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    flush.zero_()
    sections = args.sections.split(",")
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}
    props = torch.cuda.get_device_properties(dev)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    smi_index = int(vis[local_rank]) if len(vis) > local_rank and vis[local_rank].isdigit() else local_rank

    line = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic"}
    sampler = ClockSampler(smi_index)
    sampler.start()

    # ---- sweep (headline) ----
    types = [t for t in args.types.split(",") if sh.type_supported(TYPE_IDS[t])]
    sweep_tensors = [(f"{workloads.SWEEP_SHAPE[0]}x{workloads.SWEEP_SHAPE[1]}", *workloads.sweep_tensor())]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    r = run_encode_section(sh, torch, ctx, dev, stream, sweep_tensors, types, args.steps, args.warmup, rank, world,
                           flush)
    in_bytes = sum(b.size * 2 for _, b, _ in sweep_tensors)
    step_ms = max_over_ranks(sum(r["per_type_ms"].values()), dev)
    e2e_s = max_over_ranks(sum(r["e2e_per_type_s"].values()), dev)
    per_type_ms_max = {t: max_over_ranks(r["per_type_ms"][t], dev) for t in types}
    value = aggregate_gbs(in_bytes, len(types), step_ms * 1e-3)
    line.update({"value": round(value, 3), "unit": "GB/s", "ms_per_step": round(step_ms, 4)})
    line["config"] = {"workload": f"encoder sweep {sweep_tensors[0][0]} BF16 ({','.join(types)}), imatrix-weighted",
                      "types": types, "tensors": [t[0] for t in sweep_tensors],
                      "l2": "evicted (512 MB read) before every timed encode",
                      "parallelism": f"rows sharded over {world} rank(s), no collective on the data path"}
    line["per_type_gbs"] = {t: round(in_bytes / (per_type_ms_max[t] * 1e-3) / 1e9, 3) for t in types}
    line["per_type_ms"] = {t: round(v, 4) for t, v in per_type_ms_max.items()}
    line["e2e"] = {"value": round(aggregate_gbs(in_bytes, len(types), e2e_s), 3), "unit": "GB/s",
                   "h2d_bytes_per_step": len(types) * in_bytes,
                   "d2h_bytes_per_step": int(sum(OUT_BYTES_PER_ELT[t] for t in types) * in_bytes / 2)}
    line["gpu_launches"] = r["launches"]
    sweep_rank = r

    # ---- IQ configuration ----
    iq = None
    if "iq" in sections:
        iq_types = [t for t in IQ_TYPES if sh.type_supported(TYPE_IDS[t])]
        iq_tensors = workloads.iq_tensors()
        ri = run_encode_section(sh, torch, ctx, dev, stream, iq_tensors, iq_types, max(1, args.steps // 4),
                                min(args.warmup, 3), rank, world, flush)
        iq_bytes = sum(b.size * 2 for _, b, _ in iq_tensors)
        iq_ms = {t: max_over_ranks(ri["per_type_ms"][t], dev) for t in iq_types}
        iq_step = sum(iq_ms.values())
        iq_e2e = max_over_ranks(sum(ri["e2e_per_type_s"].values()), dev)
        iq = {"workload": "IQ codebook " + " + ".join(t[0] for t in iq_tensors) + " BF16 Student-t, imatrix-weighted",
              "value": round(aggregate_gbs(iq_bytes, len(iq_types), iq_step * 1e-3), 3), "unit": "GB/s",
              "per_type_gbs": {t: round(iq_bytes / (iq_ms[t] * 1e-3) / 1e9, 3) for t in iq_types},
              "per_type_ms": {t: round(v, 4) for t, v in iq_ms.items()},
              "e2e": {"value": round(aggregate_gbs(iq_bytes, len(iq_types), iq_e2e), 3), "unit": "GB/s"},
              "gpu_launches": ri["launches"], "_rank": ri, "_tensors": iq_tensors, "_types": iq_types}

    # ---- model configuration: error table + solve + encode ----
    model = None
    if "model" in sections:
        from shoehorn_b200 import host
        comm = host.Comm(rank, world)
        mc = MODELS[args.model]
        modes = tuple(args.model_modes.split(","))
        recs = host.bench_model(args.model, device=local_rank, modes=modes, budget=model_budget_arg(args.model),
                                reserve="0", ctx=MODEL_CTX, streaming=mc["streaming"],
                                out_path="-" if mc["streaming"] else "", comm=comm)
        model = {"model": args.model, "workload": mc["workload"], "elements": recs[0]["elements"],
                 "weights_in_host_memory": not mc["streaming"]}
        for rec in recs:
            key = "exact" if rec["exact_errors"] else "sampled"
            m = {k: round(max_over_ranks(rec[k], dev), 4)
                 for k in ("measure_s", "gather_s", "solve_s", "setup_s", "encode_s", "wall_s")}
            m["plan_bytes"] = rec["plan_bytes"]
            m["budget_bytes"] = rec["budget_bytes"]
            m["mix_elements"] = rec["mix_elements"]
            m["peak_rss_gb_max_rank"] = round(max_over_ranks(rec["peak_rss_bytes"], dev) / 1e9, 2)
            model[key] = m
        model["generate_s"] = round(max_over_ranks(recs[0]["generate_s"], dev), 2)

    clocks = sampler.stop()
    line["clocks"] = clocks

    # roofline of the dominant kernel of the sweep, on rank 0's launch
    sm_mhz = clocks.get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)
    dom = max(types, key=lambda t: sweep_rank["per_type_ms"][t])
    roof = roofline_for(dom, sweep_rank["rank_elts"], sweep_rank["per_type_ms"][dom], sm_mhz,
                        props.multi_processor_count, peaks)
    roof["kernel"] = f"{dom} encode call (row sigma^2 pre-pass + encoder)" if dom != "Q8_0" else "Q8_0 encoder"
    roof["traffic"] = captured_traffic(dom, sweep_rank["rank_elts"])
    roof["per_type_frac"] = {t: roofline_for(t, sweep_rank["rank_elts"], sweep_rank["per_type_ms"][t], sm_mhz,
                                             props.multi_processor_count, peaks)["frac"] for t in types}
    if dom in ("Q4_K", "Q5_K"):
        # frac counts the as-written operations while the kernel skips grids
        # whose levels repeat; the pipe's measured occupancy sits beside it
        roof["fma_pipe_active"] = 0.489
        roof["fma_pipe_source"] = "ncu sm__pipe_fma_cycles_active of enc_qk45_kernel<15>, profiles/enc_qk45_q4k_4096x14336.md"
    line["roofline"] = roof
    if iq:
        ri = iq.pop("_rank")
        iq_tensors = iq.pop("_tensors")
        iq_types = iq.pop("_types")
        iq["roofline_frac"] = {t: roofline_for(t, ri["rank_elts"], ri["per_type_ms"][t], sm_mhz,
                                               props.multi_processor_count, peaks)["frac"] for t in iq_types}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(sweep_tensors, types, budget_s=args.ref_budget)
        if iq:
            iq["cpu_baseline"] = cpu_baseline(iq_tensors, iq_types, budget_s=args.ref_budget)
        if model:
            first = model.get("sampled") or model.get("exact")
            model["cpu_baseline"] = cpu_model_baseline(first["mix_elements"], args.model)
    line["cpu_baseline"] = cpu
    if iq:
        line["iq"] = iq
    if model:
        line["model"] = model
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_reference(args):
    """The reference algorithm on the host cores (the C restatement in
    oracle/; the reference itself is a Rust crate, not buildable here), on
    the sweep's config and metric; rank 0 only."""
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    tensors = [(f"{workloads.SWEEP_SHAPE[0]}x{workloads.SWEEP_SHAPE[1]}", *workloads.sweep_tensor())]
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
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"encoder sweep {tensors[0][0]} BF16 ({','.join(types)}), imatrix-weighted",
                       "types": types, "tensors": [t[0] for t in tensors], "l2": "n/a (host CPU)",
                       "parallelism": f"host threads of one process ({os.cpu_count()} cores)"},
            "cpu_baseline": {"value": round(value, 5), "unit": "GB/s", "cores": cb["cores"], "kind": "port",
                             "sample": cb["sample"]},
            "e2e": {"value": round(value, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "per_type_gbs": cb["per_type"]}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sections", default="sweep,iq,model", help="comma-separated: sweep (always), iq, model")
    ap.add_argument("--types", default=",".join(SWEEP), help="comma-separated types of the sweep")
    ap.add_argument("--model", default="llama3-8b", choices=sorted(MODELS), help="configuration of the model section")
    ap.add_argument("--model-modes", default="sampled,exact",
                    help="error tables of the model section: sampled (the reference's 128 rows), exact (every row)")
    ap.add_argument("--ref-budget", type=float, default=12.0, help="seconds of CPU work per reference sample")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
