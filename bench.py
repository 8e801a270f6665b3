"""Benchmark of train.cpp's quantized-weight hot path on B200 (one JSON line on rank 0).

Headline (the metric's configuration): GGUF legacy-block dequantization bandwidth, one
4096 x 11008 tensor in each of Q4_0, Q4_1, Q5_0, Q5_1 and Q8_0 per step (1.07 GB of algorithmic
traffic: packed bytes read + F32 bytes written). value = algorithmic GB/s of the whole job.
With N GPUs (torchrun, one process per GPU) every rank dequantizes its own five-tensor set: the
path shards by tensor with no collective, so per-GPU work is fixed ("scaling": "weak").

Secondary (same line, key "mul_mat"): the F32 mul_mat of the fused Linear step (Q5_0 weight
4096 x 14336, 2048 tokens: fused dequant forward, dX through transpose(W), dW) and of the GQA
batched broadcast (A [128,2048,8,8] . B [128,2048,32,8], forward + composed backward, planes of
ne[3] sharded across ranks), as TFLOP/s counting 2*K*M*N once per product.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-secondary]

--impl reference times train.cpp's own CPU dequantizer (gguf_tensor_to_f32 of the reference,
compiled from its sources into oracle/_ref) on the host cores, on the same workload and metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "train.cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import synth  # noqa: E402

FORMATS = [synth.TYPE_Q4_0, synth.TYPE_Q4_1, synth.TYPE_Q5_0, synth.TYPE_Q5_1, synth.TYPE_Q8_0]
NE0, NE1 = 4096, 11008
N_BLOCKS = NE0 * NE1 // 32
METRIC = "dequant HBM GB/s; F32 mul_mat TFLOP/s (roofline %) at 1/2/4/8 B200 vs CPU"


def algorithmic_bytes(qtype: int, n_blocks: int) -> int:
    return n_blocks * (synth.BLOCK_BYTES[qtype] + 128)


STEP_BYTES = sum(algorithmic_bytes(t, N_BLOCKS) for t in FORMATS)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_value(name: str, key: str):
    """A figure recorded from an ncu capture in profiles/<name> ("key: value" lines), or None."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ clocks sampler
class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, sampled every millisecond by NVML in a
    background thread while the timed region runs (`mark_start` / `mark_stop` bracket it; only
    samples taken between them are reported). Reads only; no GPU setting is touched. Falls back
    to nvidia-smi at 200 ms when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples: list[tuple[float, float, int]] = []  # (time, sm MHz, reason mask)
        self.sm_max = None
        self.window = [None, None]
        self.stop_evt = threading.Event()
        self.thread = None
        self.nvml = None
        self.handle = None
        self.smi = None
        self.smi_out = None

    def _open_nvml(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = getattr(torch.cuda.get_device_properties(self.cuda_index), "uuid", None)
        try:
            handle = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}") if uuid is not None else None
        except pynvml.NVMLError:
            handle = None
        if handle is None:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)
        self.nvml, self.handle = pynvml, handle
        self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))

    def _poll(self):
        nv, h = self.nvml, self.handle
        while not self.stop_evt.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((time.perf_counter(), sm, mask))
            except Exception:  # noqa: BLE001 -- a failed read only loses a sample
                pass
            time.sleep(0.001)

    def __enter__(self):
        try:
            self._open_nvml()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001
            self.nvml = None
            self.smi_out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            try:
                self.smi = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.cuda_index), f"--query-gpu={self.SMI_FIELDS}",
                     "--format=csv,noheader,nounits", "-lms", "200"],
                    stdout=self.smi_out, stderr=subprocess.DEVNULL)
            except OSError:
                self.smi = None
        time.sleep(0.05)  # the sampler is running before the timed region starts
        return self

    def mark_start(self):
        self.window[0] = time.perf_counter()

    def mark_stop(self):
        self.window[1] = time.perf_counter()

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop_evt.set()
            self.thread.join(timeout=5)
        if self.smi is not None:
            time.sleep(0.25)
            self.smi.terminate()
            try:
                self.smi.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.smi.kill()

    def summary(self) -> dict:
        if self.nvml is not None:
            t0, t1 = self.window
            rows = [s for s in self.samples if t0 is not None and t1 is not None and t0 <= s[0] <= t1]
            if not rows:  # region shorter than one poll: the nearest samples either side
                rows = self.samples[-2:]
            if not rows:
                return {"sm_mhz": None, "sm_max_mhz": self.sm_max, "reasons": ["unsampled"], "samples": 0,
                        "source": "nvml"}
            reasons = sorted({name for name, const in self.REASONS for _, _, m in rows
                              if m & int(getattr(self.nvml, const))})
            return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": self.sm_max,
                    "reasons": reasons, "samples": len(rows), "source": "nvml, 1 ms poll"}
        rows = []
        if self.smi_out is not None:
            self.smi_out.flush()
            for line in Path(self.smi_out.name).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.smi_out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = [n for n, _ in self.REASONS]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi, 200 ms"}


# ------------------------------------------------------------------ CPU baseline (reference code)
def write_cfg2_gguf(path: Path, blocks: dict, chunks: int = 1) -> list[tuple[str, int, int]]:
    """The five cfg2 tensors as a GGUF file, each split into `chunks` row ranges (separate GGUF
    tensors, identical bytes) so several host threads can run the reference's per-tensor
    dequantizer at once. Returns (name, type, n_elements) per GGUF tensor."""
    tensors, names = [], []
    rows_per = NE1 // chunks
    for t in FORMATS:
        bb = synth.BLOCK_BYTES[t]
        raw = blocks[t]
        for c in range(chunks):
            r0 = c * rows_per
            r1 = NE1 if c == chunks - 1 else r0 + rows_per
            part = raw[r0 * (NE0 // 32) * bb: r1 * (NE0 // 32) * bb]
            name = f"w.{t}.{c}"
            tensors.append((name, t, (NE0, r1 - r0), part))
            names.append((name, t, NE0 * (r1 - r0)))
    synth.write_gguf(path, tensors)
    return names


def reference_dequant_rate(blocks: dict, threads: int, reps: int, warmup: int = 1) -> dict:
    """Times train.cpp's gguf_tensor_to_f32 (host dequant) over the cfg2 workload; one thread per
    chunk, `threads` at a time; `warmup` untimed passes first. Falls back to the oracle
    restatement if oracle/_ref is absent."""
    import oracle

    chunks = -(-threads // len(FORMATS)) if threads > len(FORMATS) else 1  # >= one GGUF tensor per thread
    use_ref = oracle.ref_available()
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "cfg2.gguf"
        names = write_cfg2_gguf(path, blocks, chunks)
        outs = {n: np.empty(ne, dtype=np.float32) for n, _, ne in names}
        if use_ref:
            L = oracle.ref_lib()
            handle = L.ref_gguf_open(str(path).encode())

            def work(item):
                n, _, ne = item
                L.ref_gguf_tensor_to_f32(handle, n.encode(), outs[n].ctypes.data, ne)
        else:
            O = oracle.oracle_lib()
            raw = {}
            for t in FORMATS:
                raw[t] = blocks[t]

            def work(item):
                n, t, ne = item
                c = int(n.split(".")[2])
                bb = synth.BLOCK_BYTES[t]
                nb = ne // 32
                start = c * (NE1 // chunks) * (NE0 // 32) * bb
                src = raw[t][start: start + nb * bb]
                O.oracle_dequant(t, src.ctypes.data, nb, outs[n].ctypes.data)

        def run_once():
            items = list(names)
            lock = threading.Lock()

            def worker():
                while True:
                    with lock:
                        if not items:
                            return
                        it = items.pop(0)
                    work(it)

            ths = [threading.Thread(target=worker) for _ in range(min(threads, len(names)))]
            t0 = time.perf_counter()
            for th in ths:
                th.start()
            for th in ths:
                th.join()
            return time.perf_counter() - t0

        for _ in range(max(1, warmup)):  # untimed (the first also pages the file in)
            run_once()
        times = [run_once() for _ in range(reps)]
        if use_ref:
            oracle.ref_lib().ref_gguf_close(handle)
    med = statistics.median(times)
    return {"value": STEP_BYTES / med / 1e9, "unit": "GB/s", "cores": min(threads, len(names)),
            "kind": "reference" if use_ref else "port",
            "sample": f"full dequant workload (5 x 4096x11008 tensors, {STEP_BYTES/1e9:.3f} GB algorithmic), "
                      f"median of {reps} passes, {len(names)} GGUF tensors over {min(threads, len(names))} threads",
            "seconds_per_step": med}


def make_blocks(seed_base: int) -> dict:
    return {t: synth.random_blocks(t, N_BLOCKS, seed=seed_base + t) for t in FORMATS}


def mixed_traffic_ceiling(tc, torch) -> dict:
    """What HBM delivers for the dequant's traffic mix on this GPU, measured live: streaming kernels
    of the library that read 1 byte per R written (R = 5 and 6 bracket the cfg2 ratio of 5.43) and
    do none of its arithmetic. `bulk_*`: writes staged in shared memory and stored by bulk copies,
    the dequant kernel's store path (the ceiling its fraction is taken against); `st_global_*`:
    16-byte streaming stores from registers (512 contiguous bytes per warp), the path it replaced."""
    stream = torch.cuda.current_stream()
    out = torch.empty(1 << 28, dtype=torch.float32, device="cuda")  # 1 GiB written per launch
    res = {}
    for bulk in (True, False):
        for ratio in (5, 6):
            n16 = (out.numel() * 4 // 16 // ratio) // 256 * 256
            src = torch.ones(n16 * 4, dtype=torch.float32, device="cuda")
            for _ in range(3):
                tc.stream_probe(src, out, ratio, bulk=bulk)
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(20):
                tc.stream_probe(src, out, ratio, bulk=bulk)
            e.record(stream)
            torch.cuda.synchronize()
            ms = a.elapsed_time(e) / 20
            key = f"{'bulk' if bulk else 'st_global'}_read1_write{ratio}_GBps"
            res[key] = round(n16 * 16 * (1 + ratio) / (ms * 1e-3) / 1e9, 1)
            del src
    del out
    return res


# ------------------------------------------------------------------ the reference arm
def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    blocks = make_blocks(1000)
    threads = os.cpu_count() or 1
    # each step is one pass over the workload; warmup passes run untimed
    import oracle  # noqa: F401

    res = reference_dequant_rate(blocks, threads, reps=max(1, args.steps), warmup=args.warmup)
    line = {
        "metric": METRIC, "impl": "reference", "value": round(res["value"], 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(res["seconds_per_step"] * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8->f32", "data": "synthetic (seeded PCG64 blocks per the configs)",
        "config": {"workload": "dequant sweep: Q4_0/Q4_1/Q5_0/Q5_1/Q8_0, one 4096x11008 tensor each",
                   "step_bytes": STEP_BYTES, "device": "host CPU"},
        "cpu_baseline": {"value": round(res["value"], 3), **{k: res[k] for k in ("unit", "cores", "kind", "sample")}},
        "e2e": {"value": round(res["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    import trc_cuda as tc

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    tc.lib()
    stream = torch.cuda.current_stream()
    peaks = measured_peaks()

    # ---- inputs: this rank's five tensors (weak scaling: a different seed per rank)
    blocks = make_blocks(1000 + 97 * rank)
    d_blocks = {t: torch.from_numpy(blocks[t]).cuda() for t in FORMATS}
    d_out = {t: torch.empty(N_BLOCKS * 32, dtype=torch.float32, device="cuda") for t in FORMATS}
    pinned = {t: torch.from_numpy(blocks[t]).pin_memory() for t in FORMATS}
    staging = {t: torch.empty_like(d_blocks[t]) for t in FORMATS}
    readback = torch.empty(len(FORMATS) * 32, dtype=torch.float32).pin_memory()

    # one launch for the whole step: the batched entry point a model loader uses
    step = tc.DequantBatch([(t, d_blocks[t], d_out[t]) for t in FORMATS])

    def per_format_launch_us(reps: int) -> dict:
        """Per-format launch times (one tensor per launch), CUDA events on the launching stream
        around each launch; the median of the reps (one slow launch, such as the first after the
        warm-up, would otherwise carry a mean). A 256 MB read before every launch evicts L2, so the
        25-48 MB of packed input come from HBM, not from the previous launch's L2 lines. (A read,
        not a write: a write would leave L2 full of dirty lines, whose write-back the timed launch
        would pay for.)"""
        scrub = torch.zeros(64 << 20, dtype=torch.float32, device="cuda")
        for t in FORMATS:
            for _ in range(2):
                tc.gguf_tensor_to_f32(t, d_blocks[t], out=d_out[t])
        pairs = {t: [] for t in FORMATS}
        for _ in range(reps):  # formats interleaved, so no format is timed only first or last
            for t in FORMATS:
                scrub.sum()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                tc.gguf_tensor_to_f32(t, d_blocks[t], out=d_out[t])
                b.record(stream)
                pairs[t].append((a, b))
        torch.cuda.synchronize()
        del scrub
        return {t: statistics.median(a.elapsed_time(b) for a, b in pairs[t]) for t in FORMATS}

    # correctness guard for the measured configuration (first tensor of each format, a slice)
    step()
    torch.cuda.synchronize()
    import oracle

    for t in FORMATS:
        nb = 4096
        want = oracle.dequant(t, blocks[t][: nb * synth.BLOCK_BYTES[t]], nb)
        got = d_out[t][: nb * 32].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"dequant mismatch for type {t}"

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timed region (one batched launch per step)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = tc.launch_count()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        clk.mark_start()
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
        clk.mark_stop()
    launches = tc.launch_count() - launches0
    barrier()
    ms = max_over_ranks(start.elapsed_time(stop)) / args.steps
    value = world * STEP_BYTES / (ms * 1e-3) / 1e9

    # roofline of the dominant kernel (dequant_kernel): its launch covers the whole step, so the
    # algorithmic bytes per launch are the step's bytes and its duration is the event-timed step
    achieved = STEP_BYTES / (ms * 1e-3) / 1e9
    per_launch_ms = per_format_launch_us(max(3, args.steps // 2))
    per_format = {synth_name(t): {"us": round(per_launch_ms[t] * 1e3, 2),
                                  "GBps": round(algorithmic_bytes(t, N_BLOCKS) / (per_launch_ms[t] * 1e-3) / 1e9, 1)}
                  for t in FORMATS}
    traffic = profile_value("dequant_cfg2_ncu.txt", "dram_bytes_per_launch_mean")
    ceiling = mixed_traffic_ceiling(tc, torch)
    ceiling_best = max(v for k, v in ceiling.items() if k.startswith("bulk_"))  # the dequant's store path

    # ---- end to end through the public API with host buffers: H2D packed bytes (pinned) +
    # dequant (trc_cuda_load_quant) + D2H readback of the first block of each result
    def e2e_step():
        for i, t in enumerate(FORMATS):
            tc.gguf_load_tensor(t, pinned[t], d_out[t], staging[t])
        for i, t in enumerate(FORMATS):
            readback[i * 32:(i + 1) * 32].copy_(d_out[t][:32], non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    h2d = sum(blocks[t].nbytes for t in FORMATS)
    e2e = {"value": round(world * STEP_BYTES / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": readback.numel() * 4,
           "ms_per_step": round(e2e_ms, 4), "api": "trc_cuda_load_quant (host packed -> device F32)"}

    # The bound of e2e: the same packed bytes as plain pinned host -> device copies, nothing else.
    def h2d_only():
        for t in FORMATS:
            staging[t][: pinned[t].numel()].copy_(pinned[t], non_blocking=True)

    h2d_only()
    torch.cuda.synchronize()
    barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for _ in range(args.steps):
        h2d_only()
    c1.record(stream)
    torch.cuda.synchronize()
    barrier()
    h2d_ms = max_over_ranks(c0.elapsed_time(c1)) / args.steps
    e2e["h2d_GBps"] = round(h2d / (e2e_ms * 1e-3) / 1e9, 2)
    e2e["h2d_copy_only_GBps"] = round(h2d / (h2d_ms * 1e-3) / 1e9, 2)
    e2e["frac_of_h2d_copy"] = round(h2d_ms / e2e_ms, 4)

    # ---- secondary: the whole-model dequant (cfg3) and the mul_mat workloads (tensor cores)
    secondary = whole = None
    if not args.no_secondary:
        whole = run_whole_model(tc, torch, rank, world, barrier, max_over_ranks, peaks, args)
        if world > 1:
            whole["all_gather"] = run_gather(tc, torch, rank, world, barrier, max_over_ranks, args)
        # the GEMM workloads' own clock record: dense tensor-core work can run under the power cap
        with ClockSampler(local) as gclk:
            gclk.mark_start()
            secondary = run_gemm_workloads(tc, torch, rank, world, barrier, max_over_ranks, peaks, args)
            gclk.mark_stop()
        secondary["clocks"] = gclk.summary()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = reference_dequant_rate(blocks, threads=1, reps=3)
        cpu.pop("seconds_per_step", None)

    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8->f32", "data": "synthetic (seeded PCG64 blocks per the configs)",
            "config": {"workload": "dequant sweep: Q4_0/Q4_1/Q5_0/Q5_1/Q8_0, one 4096x11008 tensor each per rank",
                       "step_bytes_per_rank": STEP_BYTES, "parallelism": f"shard-by-tensor x{world}",
                       "l2": "no flush needed: 1.07 GB touched per step > 126 MB L2, each tensor revisited "
                             "only after the other four"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                         "peak_source": peaks["source"], "kernel": "dequant_kernel (one launch per step, 5 tensors)",
                         "per_format_single_tensor_launches": per_format,
                         "mixed_traffic_ceiling": ceiling,
                         "frac_of_mixed_traffic_ceiling": round(achieved / ceiling_best, 4)},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks, "gpu_launches": launches,
        }
        if whole is not None:
            line["whole_model"] = whole
            # the configuration the path shards (cfg3: 226 tensors dealt to the ranks by LPT, total
            # work fixed), at top level beside the weak-scaling headline
            line["sharded_workload"] = {
                "workload": "whole-model dequant, Llama-7B-shaped GGUF, sharded by tensor", "metric": "GB/s",
                "value": whole["value"], "ms_per_step": whole["ms_per_step"], "scaling": "strong",
                "n_gpus": world, "total_bytes": whole["total_bytes"],
                "e2e_GBps": whole.get("e2e", {}).get("value")}
        if secondary is not None:
            line["mul_mat"] = secondary
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def synth_name(t: int) -> str:
    return {v: k for k, v in synth.TYPE_BY_NAME.items()}[t]


def run_only(args) -> None:
    """One mul_mat workload on this GPU, printed as JSON (used for bounded profiling runs)."""
    import torch

    import trc_cuda as tc

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    tc.lib()
    res = run_gemm_workloads(tc, torch, 0, 1, lambda: None, lambda x: x, measured_peaks(), args)
    print(json.dumps({"only": args.only, "mul_mat": res}), flush=True)


def ref_dequant_seconds(items, reps: int = 3) -> dict:
    """Median seconds of train.cpp's own gguf_tensor_to_f32 (oracle/_ref, one host thread) per
    tensor: items are (name, type, ne0, ne1, packed numpy blocks). None if oracle/_ref is absent."""
    import oracle

    if not oracle.ref_available():
        return None
    L = oracle.ref_lib()
    out = {}
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "sample.gguf"
        synth.write_gguf(path, [(n, t, (ne0, ne1), b) for n, t, ne0, ne1, b in items])
        handle = L.ref_gguf_open(str(path).encode())
        try:
            for n, t, ne0, ne1, _ in items:
                dst = np.empty(ne0 * ne1, dtype=np.float32)
                L.ref_gguf_tensor_to_f32(handle, n.encode(), dst.ctypes.data, ne0 * ne1)  # page in
                times = []
                for _ in range(reps):
                    t0 = time.perf_counter()
                    L.ref_gguf_tensor_to_f32(handle, n.encode(), dst.ctypes.data, ne0 * ne1)
                    times.append(time.perf_counter() - t0)
                out[n] = statistics.median(times)
        finally:
            L.ref_gguf_close(handle)
    return out


def run_whole_model(tc, torch, rank, world, barrier, max_over_ranks, peaks, args) -> dict:
    """Whole-model dequant (the Llama-7B-shaped GGUF: 226 tensors, 6.74 G weights, 31.87 GB of
    algorithmic traffic), sharded by tensor across ranks with the byte-balanced LPT partition and
    no collective. Total work is fixed, so this is strong scaling. Packed blocks are drawn on the
    device (seeded), then checked against the oracle on a slice of every tensor class."""
    import sharding
    import oracle

    stream = torch.cuda.current_stream()
    tensors = synth.llama7b_tensors()
    sizes = [algorithmic_bytes(t, ne[0] * ne[1] // 32) for _, t, ne in tensors]
    shards = sharding.lpt_shards(sizes, world)
    mine = shards[rank]
    gen = torch.Generator(device="cuda").manual_seed(7000 + rank)
    packed, outs, jobs = [], [], []
    for i in mine:
        _, t, ne = tensors[i]
        nb = ne[0] * ne[1] // 32
        b = synth.random_blocks_torch(t, nb, gen, "cuda")
        o = torch.empty(nb * 32, dtype=torch.float32, device="cuda")
        packed.append(b)
        outs.append(o)
        jobs.append((t, b, o))
    batch = tc.DequantBatch(jobs)
    batch()
    torch.cuda.synchronize()
    # correctness guard: the first 2048 blocks of the first tensor of each type, bit-exact
    seen = set()
    for (t, b, o) in jobs:
        if t in seen:
            continue
        seen.add(t)
        nb = min(2048, o.numel() // 32)
        want = oracle.dequant(t, b[: nb * synth.BLOCK_BYTES[t]].cpu().numpy(), nb)
        got = o[: nb * 32].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"whole-model dequant mismatch, type {t}"

    for _ in range(max(3, args.warmup)):
        batch()
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 20))
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = tc.launch_count()
    barrier()
    torch.cuda.synchronize()
    a.record(stream)
    for _ in range(reps):
        batch()
    e.record(stream)
    torch.cuda.synchronize()
    launches = (tc.launch_count() - launches0) // reps
    barrier()
    my_ms = a.elapsed_time(e) / reps
    ms = max_over_ranks(my_ms)
    total = sum(sizes)
    res = {
        "value": round(total / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "scaling": "strong", "total_bytes": total, "tensors": len(tensors),
        "rank0_tensors": len(shards[0]), "rank0_bytes": sum(sizes[i] for i in shards[0]),
        "lpt_imbalance": round(sharding.imbalance(sizes, shards), 4),
        "per_gpu_frac_of_hbm": round(sum(sizes[i] for i in mine) / (my_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
        "launches_per_step": launches, "steps": reps,
        "workload": "Llama-7B-shaped GGUF: Q8_0 attention, Q4_0 MLP, Q5_1 embedding/output; "
                    "device-resident packed blocks, LPT shard by tensor",
    }

    # end to end: packed bytes from pinned host memory through trc_cuda_load_quant, one staging
    # buffer per stream-ordered tensor, plus a readback of one block per tensor
    pinned = [b.cpu().pin_memory() for b in packed]
    staging = torch.empty(max(b.numel() for b in packed), dtype=torch.uint8, device="cuda")
    readback = torch.empty(len(jobs) * 32, dtype=torch.float32).pin_memory()

    def e2e_step():
        for i, (t, _, o) in enumerate(jobs):
            tc.gguf_load_tensor(t, pinned[i], o, staging)
        for i, (_, _, o) in enumerate(jobs):
            readback[i * 32:(i + 1) * 32].copy_(o[:32], non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e2e_reps = max(2, min(args.steps, 5))
    barrier()
    a.record(stream)
    for _ in range(e2e_reps):
        e2e_step()
    e.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(a.elapsed_time(e) / e2e_reps)
    res["e2e"] = {"value": round(total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 3),
                  "h2d_bytes_per_step": sum(b.numel() for b in packed), "d2h_bytes_per_step": readback.numel() * 4,
                  "steps": e2e_reps, "api": "trc_cuda_load_quant per tensor (host packed -> device F32)"}
    del pinned, staging, packed, outs, jobs, batch

    if rank == 0 and world == 1 and not args.no_cpu:
        # bounded CPU sample: one tensor of each class through the reference, scaled by the counts
        items = [("q8", synth.TYPE_Q8_0, 4096, 4096), ("q4", synth.TYPE_Q4_0, 4096, 11008),
                 ("q51", synth.TYPE_Q5_1, 4096, 32000)]
        counts = {"q8": 128, "q4": 96, "q51": 2}
        secs = ref_dequant_seconds([(n, t, a0, a1, synth.random_blocks(t, a0 * a1 // 32, seed=99))
                                    for n, t, a0, a1 in items])
        if secs is not None:
            cpu_s = sum(counts[n] * secs[n] for n in counts)
            res["cpu_baseline"] = {"value": round(total / cpu_s / 1e9, 3), "unit": "GB/s", "cores": 1,
                                   "kind": "reference",
                                   "sample": "one tensor of each class (Q8_0 4096x4096, Q4_0 4096x11008, Q5_1 "
                                             "4096x32000), median of 3, scaled by the class counts 128/96/2",
                                   "extrapolated_seconds": round(cpu_s, 2)}
    return res


NVLINK_PEER_GBS = 770.0  # peer copy per direction per GPU measured on this pool's B200s (900 nominal)


def run_gather(tc, torch, rank, world, barrier, max_over_ranks, args) -> dict:
    """The path's one collective: a dequantized tensor sharded by rows that every GPU then needs
    whole (the Q5_1 token embedding, 4096 x 32000, 524 MB of F32). Fused: each rank dequantizes
    its rows and stores them into every rank's buffer over NVLink in the same launch
    (trc_cuda_dequant_many_to_peers). Baseline: the same dequant into a local shard followed by
    NCCL all_gather_into_tensor. Both are checked bit-exact against the oracle on slices."""
    import torch.distributed as dist
    import sharding
    import oracle

    t, ne0, rows = synth.TYPE_Q5_1, 4096, 32000
    row_bytes = ne0 // 32 * synth.BLOCK_BYTES[t]
    gen = torch.Generator(device="cuda").manual_seed(5151)  # the same packed tensor on every rank
    packed = synth.random_blocks_torch(t, rows * ne0 // 32, gen, "cuda")
    rr = sharding.plane_range(rows, rank, world)
    mine = packed[rr.start * row_bytes: rr.stop * row_bytes]
    f32_bytes = rows * ne0 * 4
    buf = tc.PeerBuffer(f32_bytes)
    full = buf.tensor()
    jobs = [(t, mine, full[rr.start * ne0: rr.stop * ne0])]
    shard = torch.empty((rr.stop - rr.start) * ne0, dtype=torch.float32, device="cuda")
    full_nccl = torch.empty(rows * ne0, dtype=torch.float32, device="cuda")

    def fused():
        tc.dequantize_to_peers(jobs, buf)

    def nccl():
        tc.gguf_tensor_to_f32(t, mine, out=shard)
        dist.all_gather_into_tensor(full_nccl, shard)

    stream = torch.cuda.current_stream()
    reps = max(3, min(args.steps, 20))

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        barrier()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        e.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(a.elapsed_time(e) / reps)

    t_fused = timed(fused)
    t_nccl = timed(nccl)
    # parity: the first 1024 blocks of every rank's shard, in both assembled copies
    ok = True
    for r in range(world):
        lo = sharding.plane_range(rows, r, world).start
        nb = 1024
        want = oracle.dequant(t, packed[lo * row_bytes: lo * row_bytes + nb * synth.BLOCK_BYTES[t]].cpu().numpy(), nb)
        for got in (full, full_nccl):
            g = got[lo * ne0: lo * ne0 + nb * 32].cpu().numpy()
            ok = ok and bool(np.array_equal(g.view(np.uint32), want.view(np.uint32)))
    assert ok, "all-gathered dequant differs from the oracle"
    barrier()
    buf.close()
    egress = (world - 1) / world * f32_bytes  # bytes each rank sends over NVLink

    def line(ms):
        return {"ms": round(ms, 4), "assembled_GBps_per_rank": round(f32_bytes / (ms * 1e-3) / 1e9, 1),
                "nvlink_egress_GBps_per_rank": round(egress / (ms * 1e-3) / 1e9, 1),
                "frac_of_nvlink_peer": round(egress / (ms * 1e-3) / 1e9 / NVLINK_PEER_GBS, 4)}

    return {"tensor": "token_embd Q5_1 4096 x 32000 (524 MB F32), rows sharded over ranks",
            "fused_dequant_to_peers": line(t_fused), "dequant_then_nccl_all_gather": line(t_nccl),
            "nvlink_peak_GBps": NVLINK_PEER_GBS, "nvlink_peak_source": "measured peer copy per direction (pool)",
            "steps": reps}


def tf32_ceiling(tc, torch, barrier, max_over_ranks) -> dict:
    """The tcgen05 kind::tf32 ceiling measured here (trc_cuda_tf32_mma_probe): the GEMM's MMA stream
    alone -- three MMAs per K=8 from shared memory into TMEM, no loads, no split, no epilogue -- on
    CTA pairs (the GEMM's default) and on single CTAs. Best of 5 timed launches of ~5 ms after 2
    warm-ups, CUDA events on the launching stream, max over ranks."""
    stream = torch.cuda.current_stream()
    out = {}
    for cg, key in ((2, "pair"), (1, "single_cta")):
        iters = 8000
        for _ in range(2):
            tc.tf32_mma_probe(cg, iters)
        torch.cuda.synchronize()
        barrier()
        best = None
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            flops = tc.tf32_mma_probe(cg, iters)
            b.record(stream)
            torch.cuda.synchronize()
            ms = a.elapsed_time(b)
            best = ms if best is None else min(best, ms)
        ms = max_over_ranks(best)
        out[key + "_tf32_tflops"] = round(flops / (ms * 1e-3) / 1e12, 1)
    assert tc.device_error() == 0
    out["tf32x3_tflops"] = round(out["pair_tf32_tflops"] / 3, 1)
    out["note"] = ("tcgen05 kind::tf32 MMA stream of the GEMM's main loop alone (CTA pairs, 256x256x8, "
                   "3 MMAs per K=8); tf32x3 = pair rate / 3, F32 FLOPs counted once")
    return out


def run_gemm_workloads(tc, torch, rank, world, barrier, max_over_ranks, peaks, args) -> dict:
    """Fused Linear step (Q5_0 4096x14336, 2048 tokens) per rank, and the GQA batched broadcast
    forward + backward with ne[3] planes sharded across ranks. TFLOP/s count 2*K*M*N once. Each
    fraction is given against two ceilings: half the measured bf16 rate / 3 (derived), and the
    tcgen05 TF32 MMA rate measured by the probe in the same run / 3."""
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device="cuda").manual_seed(11 + rank)
    reps, warm = max(3, min(args.steps, 10)), max(3, args.warmup)
    tf32x3_peak = None  # derived: TF32 = half the bf16 rate, 3 passes
    if peaks.get("bf16_tflops"):
        tf32x3_peak = peaks["bf16_tflops"] / 2 / 3
    ceiling = tf32_ceiling(tc, torch, barrier, max_over_ranks)
    measured_x3 = ceiling["tf32x3_tflops"]

    def timed(fn):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(a.elapsed_time(b)) / reps

    out = {}
    only = getattr(args, "only", None)
    # --- fused Linear step
    K, M, N = 4096, 14336, 2048
    if only == "gqa":
        K = 0
    out["tf32_mma_ceiling"] = ceiling
    if K == 0:
        return gqa_workload(tc, torch, rank, world, timed, gen, tf32x3_peak, args, out)
    wq = torch.from_numpy(synth.random_blocks(synth.TYPE_Q5_0, K * M // 32, seed=21 + rank)).cuda()
    X = torch.randn((N, K), generator=gen, device="cuda")
    dY = torch.randn((N, M), generator=gen, device="cuda") * 1e-2
    Y = torch.empty((N, M), device="cuda")
    dX = torch.empty((N, K), device="cuda")
    dW = torch.zeros((M, K), device="cuda")
    flops = 2.0 * K * M * N
    # Bring the GPU to the power state of sustained tensor-core work first (about 0.3 s of GEMMs,
    # untimed): dense GEMMs meet the 1 kW cap, and whichever product ran first would otherwise be
    # timed at a cooler, faster state than the ones after it.
    for _ in range(250):
        tc.mul_mat(dY.t(), X.t(), out=dW.t(), accumulate=True)
    torch.cuda.synchronize()
    dW.zero_()
    # mul_mat_q's default for this weight: the fused dequant-in-prologue kernel (packed bytes staged
    # by TMA; no F32 copy of W anywhere). Its two-step path (W dequantized into scratch inside the
    # timed call, then the F32 kernel) is timed beside it.
    t_fwd = timed(lambda: tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, X, out=Y))
    t_dx = timed(lambda: tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, dY, transposed=True, out=dX))
    t_fwd_two = timed(lambda: tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, X, out=Y, two_step=True))
    t_dx_two = timed(lambda: tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, dY, transposed=True, out=dX, two_step=True))
    # dW for an F32 LoRA-style copy: dW^T = mul_mat(T(dY), T(X)) accumulated into the grad buffer
    t_dw = timed(lambda: tc.mul_mat(dY.t(), X.t(), out=dW.t(), accumulate=True))
    step_ms = t_fwd + t_dx + t_dw
    check_linear_slices(tc, torch, wq, K, M, X, dY, world)
    out["linear_q5_0"] = {
        "fwd_tflops": round(flops / t_fwd / 1e9, 2), "dx_tflops": round(flops / t_dx / 1e9, 2),
        "dw_tflops": round(flops / t_dw / 1e9, 2), "step_ms": round(step_ms, 4),
        "step_tflops": round(world * 3 * flops / step_ms / 1e9, 2),
        "frac_of_3xtf32_peak": round(3 * flops / step_ms / 1e9 / tf32x3_peak, 4) if tf32x3_peak else None,
        "frac_of_measured_tf32x3": round(3 * flops / step_ms / 1e9 / measured_x3, 4),
        "shape": "W q5_0 [4096,14336], X [4096,2048], dY [14336,2048]; replicas per rank",
        "path": "mul_mat_q from packed W (default): fused dequant-in-prologue tcgen05 kernel, packed bytes staged by TMA",
        "two_step": {"fwd_tflops": round(flops / t_fwd_two / 1e9, 2), "dx_tflops": round(flops / t_dx_two / 1e9, 2),
                     "path": "W dequantized into pooled scratch + F32 tcgen05 kernel, timed together"},
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        out["linear_q5_0"]["cpu_reference"] = linear_cpu_rates(tc, torch, wq, K, M, X, dY)
    del wq, X, dY, Y, dX, dW
    if only == "linear":
        return out
    return gqa_workload(tc, torch, rank, world, timed, gen, tf32x3_peak, args, out)


def gqa_workload(tc, torch, rank, world, timed, gen, tf32x3_peak, args, out) -> dict:
    measured_x3 = out["tf32_mma_ceiling"]["tf32x3_tflops"]
    """GQA batched broadcast, planes of ne[3] sharded across ranks."""
    p3 = args.gqa_p3 if getattr(args, "gqa_p3", 0) else max(1, 8 // world)
    A = torch.randn((p3, 8, 2048, 128), generator=gen, device="cuda")
    B = torch.randn((p3, 32, 2048, 128), generator=gen, device="cuda")
    G = torch.randn((p3, 32, 2048, 2048), generator=gen, device="cuda")
    D = torch.empty((p3, 32, 2048, 2048), device="cuda")
    dA = torch.empty((p3, 8, 2048, 128), device="cuda")
    dB = torch.empty((p3, 32, 2048, 128), device="cuda")
    gflop = 2.0 * 128 * 2048 * 2048 * 32 * p3
    t_f = timed(lambda: tc.mul_mat(A, B, out=D))
    # dA = repeat_back(T(mul_mat(T(G), T(B)))): one plane-reducing GEMM writing T(dA)
    t_a = timed(lambda: tc.mul_mat_repeat_back(G.transpose(-1, -2), B.transpose(-1, -2), dA.transpose(-1, -2)))
    t_b = timed(lambda: tc.mul_mat(A.transpose(-1, -2), G, out=dB))
    check_gqa_planes(tc, torch, A, B, G, D, dA, dB, world)
    out["gqa_bcast"] = {
        "fwd_tflops": round(world * gflop / t_f / 1e9, 2), "da_tflops": round(world * gflop / t_a / 1e9, 2),
        "db_tflops": round(world * gflop / t_b / 1e9, 2), "step_ms": round(t_f + t_a + t_b, 4),
        "step_tflops": round(world * 3 * gflop / (t_f + t_a + t_b) / 1e9, 2),
        "frac_of_3xtf32_peak": round(3 * gflop / (t_f + t_a + t_b) / 1e9 / tf32x3_peak, 4) if tf32x3_peak else None,
        "frac_of_measured_tf32x3": round(3 * gflop / (t_f + t_a + t_b) / 1e9 / measured_x3, 4),
        "shape": f"A [128,2048,8,{p3}] . B [128,2048,32,{p3}] per rank (ne[3] sharded over {world})",
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        out["gqa_bcast"]["cpu_reference"] = gqa_cpu_rates(A, B, G)
    out["peak_3xtf32_tflops"] = round(tf32x3_peak, 1) if tf32x3_peak else None
    out["peak_note"] = "TF32 dense taken as half the measured bf16 burst rate; 3 passes"
    return out


def _normwise(got: np.ndarray, want: np.ndarray) -> float:
    return float(np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want)))


def check_linear_slices(tc, torch, wq, K, M, X, dY, world: int) -> None:
    """Correctness guard for the timed Linear step, outside the timed region: every product the
    step times, run once more into fresh outputs, on 16 token (or output) columns against the oracle
    (the reference's summation order), normwise <= 1e-5."""
    import oracle

    threads = max(1, (os.cpu_count() or 1) // world)
    N = X.shape[0]
    Wn = oracle.dequant(synth.TYPE_Q5_0, wq.cpu().numpy()).reshape(M, K)
    j = np.arange(7, N, N // 16)[:16]
    Xj, dYj = X[j].cpu().numpy(), dY[j].cpu().numpy()
    want_y = oracle.mul_mat(Wn, Xj, n_threads=threads)[0, 0]
    want_dx = oracle.mul_mat(np.ascontiguousarray(Wn.T), dYj, n_threads=threads)[0, 0]
    Y = torch.empty((N, M), device="cuda")
    dX = torch.empty((N, K), device="cuda")
    for two_step in (False, True):
        tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, X, out=Y, two_step=two_step)
        tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, dY, transposed=True, out=dX, two_step=two_step)
        e_y, e_dx = _normwise(Y.cpu().numpy()[j], want_y), _normwise(dX.cpu().numpy()[j], want_dx)
        assert e_y <= 1e-5 and e_dx <= 1e-5, f"Linear step parity (two_step={two_step}): fwd {e_y:.2e}, dX {e_dx:.2e}"
    dW = torch.zeros((M, K), device="cuda")
    tc.mul_mat(dY.t(), X.t(), out=dW.t(), accumulate=True)
    k = np.arange(3, K, K // 16)[:16]
    want_dw = oracle.mul_mat(np.ascontiguousarray(dY.cpu().numpy().T), np.ascontiguousarray(X.cpu().numpy().T[k]),
                             n_threads=threads)[0, 0]
    e_dw = _normwise(dW.cpu().numpy()[:, k].T, want_dw)
    assert e_dw <= 1e-5, f"Linear step parity: dW {e_dw:.2e}"
    assert tc.device_error() == 0


def check_gqa_planes(tc, torch, A, B, G, D, dA, dB, world: int) -> None:
    """Correctness guard for the timed GQA step (outputs of its last timed launches): one (i2, i3)
    plane of the forward and of dB, and one reduced plane of dA, against the oracle."""
    import oracle

    threads = max(1, (os.cpu_count() or 1) // world)
    torch.cuda.synchronize()
    i3, i2, ga = A.shape[0] - 1, 13, 5
    a, b, g = A[i3, i2 % 8].cpu().numpy(), B[i3, i2].cpu().numpy(), G[i3, i2].cpu().numpy()
    e_f = _normwise(D[i3, i2].cpu().numpy(), oracle.mul_mat(a, b, n_threads=threads)[0, 0])
    e_b = _normwise(dB[i3, i2].cpu().numpy(), oracle.mul_mat(np.ascontiguousarray(a.T), g, n_threads=threads)[0, 0])
    want_da = sum(oracle.mul_mat(np.ascontiguousarray(G[i3, p].cpu().numpy().T),
                                 np.ascontiguousarray(B[i3, p].cpu().numpy().T), n_threads=threads)[0, 0]
                  for p in range(ga, 32, 8))
    e_a = _normwise(np.ascontiguousarray(dA[i3, ga].t().cpu().numpy()), want_da)
    assert max(e_f, e_a, e_b) <= 1e-5, f"GQA step parity: fwd {e_f:.2e}, dA {e_a:.2e}, dB {e_b:.2e}"
    assert tc.device_error() == 0


def _ref_gflops(a_base, a_trans, b_base, b_trans, flops: float) -> float | None:
    """GFLOP/s of train.cpp's CPU mul_mat (oracle/_ref, one thread) on one slice, best of 2."""
    import oracle

    if not oracle.ref_available():
        return None
    best = None
    for _ in range(2):
        t0 = time.perf_counter()
        oracle.ref_mul_mat(a_base, a_trans, b_base, b_trans)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return round(flops / best / 1e9, 3)


def _extrapolated_s(rates: dict, flops_per_product: float) -> float | None:
    """Seconds the reference CPU backend would take for the whole step (each product's FLOPs at
    its measured slice rate)."""
    vals = [rates[k] for k in rates if k.endswith("_gflops")]
    if any(v is None or v <= 0 for v in vals):
        return None
    return round(sum(flops_per_product / (v * 1e9) for v in vals), 1)


def linear_cpu_rates(tc, torch, wq, K, M, X, dY) -> dict:
    """The reference CPU backend on deterministic slices of the Linear step (it would take hours
    in full): forward on 16 token columns, dX on 4, dW on 4 of its K columns."""
    W = tc.gguf_tensor_to_f32(synth.TYPE_Q5_0, wq).view(M, K).cpu().numpy()
    Xn, dYn = X.cpu().numpy(), dY.cpu().numpy()
    rates = {
        "fwd_gflops": _ref_gflops(W, False, Xn[:16], False, 2.0 * K * M * 16),
        "dx_gflops": _ref_gflops(W, True, dYn[:4], False, 2.0 * K * M * 4),
        "dw_gflops": _ref_gflops(dYn, True, np.ascontiguousarray(Xn[:, :4]), True, 2.0 * X.shape[0] * M * 4),
    }
    return {**rates, "extrapolated_step_s": _extrapolated_s(rates, 2.0 * K * M * X.shape[0]),
            "cores": 1, "kind": "reference",
            "sample": "forward: 16 of 2048 token columns; dX: 4 columns; dW: 4 of 4096 output columns"}


def gqa_cpu_rates(A, B, G) -> dict:
    """The reference CPU backend on one (i2, i3) plane of the GQA workload, sliced for the
    transposed-view backward products."""
    a = A[0, 0].cpu().numpy()          # [2048, 128]: ne [128, 2048]
    b = B[0, 0].cpu().numpy()
    g = G[0, 0].cpu().numpy()          # [2048, 2048]
    rates = {
        "fwd_gflops": _ref_gflops(a, False, b, False, 2.0 * 128 * 2048 * 2048),
        "da_gflops": _ref_gflops(g, True, np.ascontiguousarray(b[:, :16]), True, 2.0 * 2048 * 2048 * 16),
        "db_gflops": _ref_gflops(a, True, np.ascontiguousarray(g[:64]), False, 2.0 * 2048 * 128 * 64),
    }
    planes = G.shape[0] * G.shape[1]  # the rank's (i2, i3) planes
    return {**rates, "extrapolated_step_s": _extrapolated_s(rates, 2.0 * 128 * 2048 * 2048 * planes),
            "cores": 1, "kind": "reference",
            "sample": "one plane; forward in full, dA on 16 of 128 columns, dB on 64 of 2048 columns"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (bounded profiling runs)")
    ap.add_argument("--only", choices=["linear", "gqa"], default=None,
                    help="run only one mul_mat workload (bounded cases for profiling)")
    ap.add_argument("--gqa-p3", type=int, default=0, help="ne[3] planes per rank for the GQA workload (0 = 8/N)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.only is not None:
        run_only(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
