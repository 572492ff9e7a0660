"""Benchmark of the five-value int8 GEMM on B200 (BASELINE.json metric "five-value int8 GEMM TMAC/s").

Workload: every five-value GEMM of one FastConformer block at T = 375 encoder frames
(a 30 s window): ff1 1024->4096, ff1 4096->1024 (alpha 1/2, beta 1), qkv 1024->3072 (stored fused), pos 1024->1024
at 2T - 1 = 749 rows, out 1024->1024 (beta 1), pw1 1024->2048, pw2 1024->1024 (beta 1), ff2 as ff1. Weights are
seeded synthetic five-value planes (P(0) = 1/3, P(+-lo) = P(+-hi) = 1/6, lo ~ U(0.005, 0.02), hi = lo * U(2, 4),
fp16-rounded); activations fp32 N(0, 1). One step = the nine GEMMs from fp32 activations, each quantised per row
and multiplied on the tensor cores, as p2_sgemm_fvb does (csrc/blas.c:1481-1499).

Timing: W warm-up steps, then exactly K steps between a barrier + synchronize, CUDA events on the launching stream,
max over ranks. Steps rotate over enough independent copies of the inputs that they exceed twice the 126 MB L2.
Each GPU runs its own copy of the workload (windows are independent: weak scaling, no collective on the data path).

--impl reference times phonon-2-c itself (its library compiled from source, exact mode: its int8 path needs AArch64
dot products) on the host cores, on the same workload and metric.
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
import __graft_entry__ as ge  # noqa: E402

T_FRAMES = 375
METRIC = "five-value int8 GEMM TMAC/s"
L2_BYTES = 126 * 1024 * 1024


def block_gemms(T=T_FRAMES):
    from phonon2_b200 import synth
    return [(name, synth.block_rows(rows, T), K, N, alpha, beta)
            for name, K, N, alpha, beta, rows in synth.BLOCK_SHAPES]


def block_macs(T=T_FRAMES) -> int:
    return sum(M * K * N for _, M, K, N, _, _ in block_gemms(T))


def gemm_bytes(M, K, N, beta, codes=False) -> int:
    """Algorithmic HBM bytes of one GEMM launch on quantised A: int8 A, the weight (the planes at 3 bits per weight,
    or the cached int8w codes at 8), lo/hi, the fp32 C store and, when accumulating, the C read."""
    w = K * N if codes else 3 * K * N // 8
    return M * K + w + 8 * N + 4 * M * N + (4 * M * N if beta != 0.0 else 0)


TRAFFIC_FILES = {"vindex": "fv_gemm_t_block_T375_traffic.md", "planes": "fv_gemm_block_T375_traffic.md"}


def block_traffic(weights):
    """DRAM bytes per step of the block GEMMs (int8w) from a committed ncu capture of the same kernels (a static
    figure: ncu cannot run inside the bench), or None."""
    import re
    if weights not in TRAFFIC_FILES:
        return None
    f = ROOT / "profiles" / TRAFFIC_FILES[weights]
    if not f.exists():
        return None
    m = re.search(r"^traffic_bytes_per_step: (\d+)$", f.read_text(), re.M)
    return int(m.group(1)) if m else None


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML by a background thread about every half millisecond; the
    summary keeps the samples taken between mark_start() and mark_end() (the timed region), and says so."""
    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("sw_power_cap", 0x4))

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples = []
        self.thread = None
        self.stop = False
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def loop():
                while not self.stop:
                    t = time.perf_counter()
                    self.samples.append((t, pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), reasons(h)))
                    time.sleep(0.0005)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
        except Exception:   # no NVML: the summary says there were no samples
            self.thread = None
        return self

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __exit__(self, *exc):
        self.stop = True
        if self.thread:
            self.thread.join(timeout=2)

    def summary(self):
        inside = [x for x in self.samples if self.t0 is not None and self.t1 is not None and self.t0 <= x[0] <= self.t1]
        rows, where = (inside, "timed region") if inside else (self.samples, "around the timed region")
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        active = sorted({name for _, _, r in rows for name, bit in self.REASONS if r & bit})
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": self.max_mhz, "reasons": active,
                "samples": len(rows), "sampled": f"NVML every 0.5 ms, {where}"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- the reference on the host cores -------------------------------------------------------------------------------

def cpu_reference_step(orc, sets):
    for (A, w, C, alpha, beta) in sets:
        orc.ref_sgemm_fvb(A, w, C, alpha=alpha, beta=beta)


def build_cpu_sets(T=T_FRAMES):
    from phonon2_b200 import synth
    sets = []
    for i, (name, M, K, N, alpha, beta) in enumerate(block_gemms(T)):
        w = synth.five_value(K, N, seed=100 + i)
        A = synth.activations(M, K, seed=200 + i)
        sets.append((A, w, np.zeros((M, N), np.float32), alpha, beta))
    return sets


def cpu_baseline(seconds=12.0):
    """phonon-2-c's exact path (its only x86 path) on all host cores, one block's GEMMs at T = 375, repeated for
    about `seconds`."""
    orc = ge.load_oracle()
    if not orc.ref_available():
        return None
    sets = build_cpu_sets()
    cpu_reference_step(orc, sets)   # warm-up (thread pool start, page faults)
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_reference_step(orc, sets)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= seconds or reps >= 1000:
            break
    value = block_macs() * reps / dt / 1e12
    return {"value": value, "unit": "TMAC/s", "cores": orc.ref_threads(), "kind": "reference",
            "sample": f"phonon-2-c p2_sgemm_fvb (exact mode, AVX2) over one block's 9 GEMMs at T={T_FRAMES}, "
                      f"{reps} repetitions in {dt:.1f} s, P2_THREADS = all host cores"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    ge.load_package()   # for the synthetic model and inputs (phonon2_b200.model); the library itself is not loaded
    orc = ge.load_oracle()
    if not orc.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "phonon-2-c library not built (oracle/_ref missing)"}))
        return
    sets = build_cpu_sets()
    for _ in range(args.warmup):
        cpu_reference_step(orc, sets)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(orc, sets)
    dt = time.perf_counter() - t0
    value = block_macs() * args.steps / dt / 1e12
    cores = orc.ref_threads()
    line = {"metric": METRIC, "value": value, "unit": "TMAC/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"one FastConformer block's nine five-value GEMMs at T={T_FRAMES} "
                                   "(BASELINE configs[1]), exact mode (the reference's only x86 path)",
                       "mode": "exact", "T": T_FRAMES},
            "cpu_baseline": {"value": value, "unit": "TMAC/s", "cores": cores, "kind": "reference",
                             "sample": f"{args.steps} steps of the full workload"},
            "e2e": {"value": value, "unit": "TMAC/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    # the encoder object last, as on our arm's line: the end of the line is what a record of the output's tail keeps
    if not args.no_decoder:
        la = long_audio_reference()
        if la is not None:
            line["long_audio"] = {"metric": "long-form transcription audio-sec/sec", "value": la["value"],
                                  "unit": "audio-s/s", "mode": "exact", "cpu_baseline": la,
                                  "e2e": {"value": la["value"], "unit": "audio-s/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}
    if not args.no_encoder:
        enc = encoder_reference()
        if enc is not None:
            line["encoder"] = {"metric": "encoder audio-sec/sec", "value": enc["value"], "unit": "audio-s/s",
                               "workload": encoder_workload("long-audio")[1], "mode": "exact",
                               "cpu_baseline": enc,
                               "e2e": {"value": enc["value"], "unit": "audio-s/s", "h2d_bytes_per_step": 0,
                                       "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ---- ours on the GPU ----------------------------------------------------------------------------------------------

class GpuSet:
    """One independent copy of the workload on the device: weights, fp32 activations, outputs, workspace."""

    def __init__(self, pkg, torch, dev, seed, mode, gemms, codes=False, vindex=False):
        from phonon2_b200 import synth
        from phonon2_b200.device import DeviceFiveValue
        self.items = []
        for i, (name, M, K, N, alpha, beta) in enumerate(gemms):
            w = synth.five_value(K, N, seed=1000 * seed + i)
            B = DeviceFiveValue(w, dev, codes=codes, vindex=vindex)
            A = torch.from_numpy(synth.activations(M, K, seed=2000 * seed + i)).to(dev)
            C = torch.zeros((M, N), dtype=torch.float32, device=dev)
            ws = torch.empty(max(pkg.workspace_bytes(M, N, K, mode), 256), dtype=torch.uint8, device=dev)
            self.items.append((M, K, N, alpha, beta, B, A, C, ws))

    def bytes(self):
        return sum(B.plane_bytes + (B.codes.numel() if B.codes is not None else 0)
                   + (4 * B.vindex.numel() if B.vindex is not None else 0) + A.numel() * 4 + C.numel() * 4
                   + ws.numel() for (_, _, _, _, _, B, A, C, ws) in self.items)

    def run(self, pkg, mode, stream):
        for (M, K, N, alpha, beta, B, A, C, ws) in self.items:
            pkg.sgemm_fvb(M, N, K, alpha, A.data_ptr(), K, B.struct, mode, beta, C.data_ptr(), N, ws.data_ptr(),
                          ws.numel(), stream)

    def quantise(self, pkg, stream):
        for (M, K, N, alpha, beta, B, A, C, ws) in self.items:
            pkg.quant_rows(A.data_ptr(), M, K, K, ws.data_ptr(), ws.data_ptr() + ((M * K + 255) // 256) * 256,
                           stream)

    def run_gemm_only(self, pkg, mode, stream):
        for (M, K, N, alpha, beta, B, A, C, ws) in self.items:
            q = ws.data_ptr()
            sc = q + ((M * K + 255) // 256) * 256
            rest = sc + ((M * 4 + 255) // 256) * 256
            pkg.sgemm_fvb_q8a(M, N, K, alpha, q, sc, B.struct, mode, beta, C.data_ptr(), N, rest,
                              ws.numel() - (rest - q), stream)


def run_ours(args, world, rank, local):
    import torch
    pkg = ge.load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    mode = pkg.MODES[args.mode]
    os.environ["P2_GEMM"] = args.mode   # the host ABI's mode (read once, on its first call)
    gemms = block_gemms()
    stream = torch.cuda.Stream(device=dev)

    # Enough independent copies of the inputs that consecutive steps never find their operands in L2.
    codes = args.weights == "codes"
    vix = args.weights == "vindex"
    first = GpuSet(pkg, torch, dev, 1 + rank * 100, mode, gemms, codes, vix)
    nsets = max(2, int(np.ceil(2 * L2_BYTES / first.bytes())))
    sets = [first] + [GpuSet(pkg, torch, dev, 2 + i + rank * 100, mode, gemms, codes, vix)
                      for i in range(nsets - 1)]
    torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for s in sets:                      # first calls outside capture (kernel attributes, symbol lookups)
            s.run(pkg, mode, stream)
        stream.synchronize()
        pkg.check_device(stream)
        graphs = []
        for s in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                s.run(pkg, mode, stream)
            graphs.append(g)
        gemm_graphs = []                    # the GEMM kernels alone, on quantised A, for the roofline
        for s in sets:
            s.quantise(pkg, stream)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                s.run_gemm_only(pkg, mode, stream)
            gemm_graphs.append(g)
    torch.cuda.synchronize()

    for i in range(args.warmup):
        graphs[i % nsets].replay()
    torch.cuda.synchronize()
    barrier(world)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(0.01)   # the sampler's first samples
        torch.cuda.synchronize()
        clocks.mark_start()
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(args.steps):
                graphs[i % nsets].replay()
            end.record(stream)
        end.synchronize()
        clocks.mark_end()
    torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms, world)
    pkg.check_device(stream)

    macs = block_macs()
    value = macs * args.steps * world / (ms_max / 1e3) / 1e12

    # Roofline of the dominant kernel (the tcgen05 GEMM): algorithmic bytes of the nine launches / their time.
    reps = max(50, min(2000, args.steps))
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        g0.record(stream)
        for i in range(reps):
            gemm_graphs[i % nsets].replay()
        g1.record(stream)
    g1.synchronize()
    gemm_ms = g0.elapsed_time(g1) / reps
    algo_bytes = sum(gemm_bytes(M, K, N, beta, codes) for _, M, K, N, _, beta in gemms)
    peak, peak_kind = load_peaks()
    achieved = algo_bytes / (gemm_ms / 1e3) / 1e9

    # End to end: fp32 activations from pinned host memory, results back to pinned host memory, every step.
    e2e = run_e2e(pkg, torch, dev, stream, sets[0], mode, args, 1 + rank * 100)
    e2e_ms = max_over_ranks(e2e["ms_per_step"], world)   # whole job: every rank's step over the slowest rank's time
    e2e.update({"value": world * block_macs() / (e2e_ms / 1e3) / 1e12, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": world * e2e["h2d_bytes_per_step"],
                "d2h_bytes_per_step": world * e2e["d2h_bytes_per_step"]})

    n_split = sum(1 for (_, _, K, _, _, _) in gemms if K > 1024)
    line = None
    if rank == 0:
        traffic = block_traffic(args.weights) if args.mode == "int8w" else None
        line = {"metric": METRIC, "value": value, "unit": "TMAC/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8" if mode != pkg.EXACT else "f32",
                "data": "synthetic",
                "config": {"workload": f"BASELINE configs[1]: one block's nine five-value GEMMs at T={T_FRAMES}, fp32 "
                                       "A quantised per row then the tcgen05 GEMM",
                           "mode": args.mode, "weights": args.weights, "T": T_FRAMES, "macs_per_step": macs,
                           "l2": f"inputs rotate over {nsets} copies ({nsets * first.bytes() / 2**20:.0f} MiB > 2x L2)",
                           "parallelism": f"replicas x{world}"},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": traffic,
                             "traffic_kind": "static ncu capture (profiles/" + TRAFFIC_FILES[args.weights] + ")"
                             if traffic else None,
                             "peak_kind": peak_kind, "algo_bytes_per_step": algo_bytes,
                             "gemm_us_per_step": gemm_ms * 1e3,
                             "kernel": "fv_gemm_t_kernel" if args.weights == "vindex" and args.mode == "int8w"
                             else "fv_gemm_kernel"},
                "gpu_launches": args.steps * (2 * len(gemms) + n_split),
                "clocks": clocks.summary(),
                "e2e": e2e}
    extras = {}
    if not args.no_encoder:
        extras["encoder"] = encoder_ours(args, world, rank, local, torch, pkg)
    if not args.no_decoder:
        extras["decoder"] = decoder_ours(args, world, rank, local, torch, pkg)
        extras["mel"] = mel_ours(args, world, rank, local, torch, pkg)
        extras["long_audio"] = long_audio_ours(pkg, world, rank, local)
    cfg = None
    if not args.no_configs and world == 1:   # the per-config objects are single-GPU measurements
        cfg = configs_ours(args, world, rank, local, torch, pkg, value, gemm_ms, algo_bytes, peak)
    if rank == 0:
        cpu = world == 1 and not args.no_cpu_baseline
        if cpu:
            line["cpu_baseline"] = cpu_baseline()
        if cfg is not None and cpu:
            for key, n_mel in (("c2", 3000), ("c4", 300)):
                cfg[key]["cpu_ms_exact"] = round(transcribe_reference(n_mel)["value"], 1)
        finish_line(line, extras, cfg)
        if cpu:
            if "encoder" in line:
                line["encoder"]["cpu"] = compact_cpu(encoder_reference())
            if "decoder" in line:
                line["decoder"]["cpu"] = compact_cpu(decoder_reference())
                line["mel"]["cpu"] = compact_cpu(mel_reference())
                line["long_audio"]["cpu"] = compact_cpu(long_audio_reference())
        print(json.dumps(line))


def finish_line(line, extras, cfg):
    """The sub-objects after the headline keys: the per-config object first, then the decoder, log-mel and long-audio
    objects, and the encoder (the metric's second half) last, at the end of the line, which is the part a record that
    keeps only the tail of the output still holds."""
    if cfg is not None:
        line["configs"] = cfg
    for name in ("decoder", "mel", "long_audio", "encoder"):
        if name in extras:
            line[name] = compact(extras[name])
    return line


def compact(obj):
    """The headline-style fields of a sub-object (value, unit, time, e2e), without the long descriptions."""
    keep = {k: obj[k] for k in ("value", "unit", "ms_per_step", "tokens_rank0", "windows", "mode", "weights")
            if k in obj}
    for k in ("e2e", "transcribe_audio"):
        if k in obj:
            keep[k] = {kk: obj[k][kk] for kk in ("value", "unit", "ms_per_step", "h2d_bytes_per_step",
                                                 "d2h_bytes_per_step") if kk in obj[k]}
    return keep


def compact_cpu(c):
    return None if c is None else {"value": c["value"], "unit": c["unit"], "cores": c["cores"], "kind": c["kind"]}


def time_replays(torch, stream, graphs, steps):
    """Milliseconds per replay over `steps` replays rotating over `graphs` (CUDA events on `stream`)."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for i in range(3):
            graphs[i % len(graphs)].replay()
        e0.record(stream)
        for i in range(steps):
            graphs[i % len(graphs)].replay()
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def step_graphs(pkg, torch, dev, stream, mode, gemms, weights, seed, gemm_only=False):
    """CUDA graphs of one step of `gemms` over enough input copies to exceed twice L2, as the headline's."""
    codes, vix = weights == "codes", weights == "vindex"
    first = GpuSet(pkg, torch, dev, seed, mode, gemms, codes, vix)
    nsets = max(2, int(np.ceil(2 * L2_BYTES / first.bytes())))
    sets = [first] + [GpuSet(pkg, torch, dev, seed + 1 + i, mode, gemms, codes, vix) for i in range(nsets - 1)]
    graphs = []
    with torch.cuda.stream(stream):
        for st in sets:
            st.run(pkg, mode, stream)
            if gemm_only:
                st.quantise(pkg, stream)
        stream.synchronize()
        for st in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                (st.run_gemm_only if gemm_only else st.run)(pkg, mode, stream)
            graphs.append(g)
    torch.cuda.synchronize()
    pkg.check_device(stream)
    return graphs


def int8_peak() -> tuple[float, str]:
    """The int8 tcgen05 MMA rate the large-M fractions divide by: measured on this GPU by the probes library when it
    is built, else the rate that probe measured on this pool's B200s (2284 TMAC/s, profiles/probes_tma_mma.md)."""
    import ctypes as C
    if (ROOT / "phonon-2-c_b200" / "libphonon2_probes.so").exists():
        L = probes_lib()
        v = C.c_double()
        if L.p2cu_probe_int8_mma(0, 4000, C.byref(v)) == 0:
            return v.value / 1e12, "measured in this run"
    return 2284.0, "measured on this pool (profiles/probes_tma_mma.md)"


def configs_ours(args, world, rank, local, torch, pkg, headline, gemm_ms, algo_bytes, hbm_peak):
    """Every BASELINE config as a compact object (the headline is configs[1] int8w): c0 the single GEMM, c1 the block
    in every mode and weight form, large_m the north star's M >= 4096 shape, c2 / c4 one window end to end in both
    modes (the speech-like model, so that greedy decoding emits tokens), c3 is the `encoder` object."""
    from phonon2_b200 import model as Mo
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(device=dev)
    gemms = block_gemms()
    seed = 500 + rank * 100
    out = {}
    steps = max(10, min(args.steps, 100))
    # c0: ff1 1024 -> 4096 at M = 375 alone: quantiser + GEMM, and the GEMM alone against its HBM bound
    c0 = [g for g in gemms if g[0] == "ff1.linear1"]
    _, M0, K0, N0, _, _ = c0[0]
    t_step = time_replays(torch, stream, step_graphs(pkg, torch, dev, stream, pkg.INT8W, c0, args.weights, seed),
                          steps)
    t_gemm = time_replays(torch, stream, step_graphs(pkg, torch, dev, stream, pkg.INT8W, c0, args.weights, seed,
                                                     gemm_only=True), steps)
    b0 = gemm_bytes(M0, K0, N0, 0.0)
    out["c0"] = {"tmacs": round(M0 * K0 * N0 / (t_step * 1e9), 1), "us": round(t_step * 1e3, 2),
                 "gemm_us": round(t_gemm * 1e3, 2), "gemm_frac_hbm": round(b0 / (t_gemm * 1e-3) / 1e9 / hbm_peak, 3)}
    # c1: the block in each mode / weight form (TMAC/s per step, the quantiser included)
    c1 = {"int8w_" + args.weights: round(headline, 1)}
    for mode, weights in (("int8", "planes"), ("exact", "planes"), ("int8w", "codes"), ("int8w", "planes")):
        key = f"{mode}_{weights}"
        if key in c1:
            continue
        t = time_replays(torch, stream, step_graphs(pkg, torch, dev, stream, pkg.MODES[mode], gemms, weights, seed),
                         steps if mode != "exact" else 5)
        c1[key] = round(block_macs() / (t * 1e9), 1)
    c1["unit"] = "TMAC/s"
    out["c1"] = c1
    # large M (north star: >= 60 % of the int8 peak at K = 1024, N = 4096, M >= 4096), the GEMM alone
    peak_i8, peak_kind = int8_peak()
    lm = {"int8_peak_tmacs": round(peak_i8), "peak_kind": peak_kind}
    for Mbig in (4096, 8192):
        for weights in ("codes", "planes"):
            t = time_replays(torch, stream, step_graphs(pkg, torch, dev, stream, pkg.INT8W,
                                                        [("ff1.linear1", Mbig, 1024, 4096, 1.0, 0.0)], weights, seed,
                                                        gemm_only=True), 100)
            v = Mbig * 1024 * 4096 / (t * 1e9)
            lm[f"M{Mbig}_{weights}"] = {"tmacs": round(v), "frac_int8": round(v / peak_i8, 3)}
    out["large_m"] = lm
    # c2 / c4: one window end to end, host mel in, host tokens out
    sm = Mo.SyntheticModel(seed=1, attn_out_gain=Mo.SPEECH_ATTN_OUT_GAIN)
    dm = pkg.DeviceModel(sm.struct)
    for key, n_mel in (("c2", 3000), ("c4", 300)):
        mel = Mo.mel(n_mel, seed=n_mel)
        res = {"mel_frames": n_mel}
        for _ in range(2):
            toks = pkg.host_transcribe_windows(sm.struct, [mel], devices=[local])
        t0 = time.perf_counter()
        for _ in range(5):
            toks = pkg.host_transcribe_windows(sm.struct, [mel], devices=[local])
        res["ms_int8w"] = round((time.perf_counter() - t0) / 5 * 1e3, 2)
        res["tokens_int8w"] = int(len(toks[0]))
        res["ms_exact"], res["tokens_exact"] = plan_transcribe_ms(pkg, torch, dm, mel, pkg.EXACT, local)
        res["api"] = "p2_b200_transcribe_windows (int8w); encoder + decoder plans with host copies (exact)"
        out[key] = res
    dm.close()
    # the weight stream of config 4 (BASELINE: HBM GB/s on the planes): the bytes every pass reads at least once (the
    # value-index planes the window-sized GEMMs read, plus lo / hi) over the end-to-end time - a lower bound
    vi_bytes = sum(pkg.fv_vindex_bytes(K, N) + 8 * N for (_, K, N, _, _, _) in synth_block_shapes()) * 24
    out["c4"]["weight_stream_gbs_lower_bound"] = round(vi_bytes / (out["c4"]["ms_int8w"] * 1e-3) / 1e9, 1)
    return out if rank == 0 else None


def synth_block_shapes():
    from phonon2_b200 import synth
    return synth.BLOCK_SHAPES


def plan_transcribe_ms(pkg, torch, dm, mel, mode, local, steps=3):
    """One window through the encoder plan and the decoder in `mode`, timed end to end by the wall clock: the mel
    copied up from page-locked memory, the encoder's graph, the decoder launch, the tokens read back."""
    from phonon2_b200.device import device_view
    enc = pkg.Encoder(dm, [mel.shape[0]], mode)
    dec = pkg.Decoder(dm, 1, enc.total_frames)
    mel_h = torch.empty(mel.shape, dtype=torch.float32, pin_memory=True)
    mel_h.numpy()[...] = mel
    dst = device_view(enc.mel_ptr, mel.shape)
    stream = torch.cuda.Stream(device=torch.device("cuda", local))

    def once():
        with torch.cuda.stream(stream):
            dst.copy_(mel_h, non_blocking=True)
        enc.run(stream)
        dec.decode(enc.out_ptr, enc.frames, stream)
        return dec.read(stream)

    for _ in range(2):
        toks = once()
    t0 = time.perf_counter()
    for _ in range(steps):
        toks = once()
    ms = (time.perf_counter() - t0) / steps * 1e3
    dec.close()
    enc.close()
    return round(ms, 2), int(len(toks[0]))


# ---- the encoder: audio seconds per second --------------------------------------------------

ENC_SECONDS_PER_FRAME = 0.01   # 100 mel frames per second of audio


def shard_windows(frames, world):
    """Windows to ranks as p2_b200_encode_windows assigns them to GPUs: longest first, to the least-loaded rank."""
    order = sorted(range(len(frames)), key=lambda w: -frames[w])
    load, out = [0] * world, [[] for _ in range(world)]
    for w in order:
        r = min(range(world), key=lambda i: load[i])
        out[r].append(w)
        load[r] += frames[w]
    return [sorted(v) for v in out]


def encoder_workload(name, windows=0):
    from phonon2_b200 import model as M
    if name == "long-audio":
        frames = M.long_audio_windows(0)
        if windows:
            frames = frames[:windows]
        return frames, ("BASELINE configs[3]: a 32-minute synthetic log-mel stream as 64 windows of U(25, 35) s "
                        "(seeded), sharded over the GPUs longest-first" + (f"; the first {windows} windows" if windows
                                                                           else ""))
    if name == "window":
        return [3000], "BASELINE configs[2]: one 30 s window (mel [3000 x 128], T' = 375)"
    return [300], "BASELINE configs[4]: one 3 s utterance (mel [300 x 128], T' = 38)"


def encoder_ours(args, world, rank, local, torch, pkg, workload="long-audio", steps=5, windows=0):
    """The encoder on this rank's share of the windows: device-timed graph launches (mel resident), then end to end
    through p2_b200_encode_windows (host mel in, host frames out, this rank's GPU)."""
    from phonon2_b200 import model as M
    from phonon2_b200.device import device_view
    frames, desc = encoder_workload(workload, windows)
    mine = shard_windows(frames, world)[rank]
    sm = M.SyntheticModel(seed=1)
    dm = pkg.DeviceModel(sm.struct, codes=args.weights == "codes")
    mode = pkg.MODES[args.mode]
    mels = [M.mel(frames[w], seed=w) for w in mine]
    enc = pkg.Encoder(dm, [frames[w] for w in mine], mode) if mine else None
    stream = torch.cuda.Stream()
    ms = 0.0
    if enc is not None:
        stacked = np.ascontiguousarray(np.concatenate(mels), np.float32)
        device_view(enc.mel_ptr, stacked.shape).copy_(torch.from_numpy(stacked))
        torch.cuda.synchronize()
        for _ in range(2):
            enc.run(stream)
        stream.synchronize()
    barrier(world)
    if enc is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            enc.run(stream)
        e1.record(stream)
        e1.synchronize()
        pkg.check_device(stream)
        ms = e0.elapsed_time(e1) / steps
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    audio_s = sum(frames) * ENC_SECONDS_PER_FRAME
    # end to end through the public host API (p2_b200_encode_windows), on this rank's GPU: the windows' mel stacked in
    # page-locked host memory, the frames returned into page-locked host memory
    e2e_ms = 0.0
    n_out = sum(M.frames_after_subsampling(frames[w]) for w in mine)
    if mine:
        import ctypes as C
        mel_h = torch.empty((sum(frames[w] for w in mine), 128), dtype=torch.float32, pin_memory=True)
        mel_h.numpy()[...] = np.concatenate(mels)
        out_h = torch.empty((n_out, 640), dtype=torch.float32, pin_memory=True)
        fr = (C.c_int * len(mine))(*[frames[w] for w in mine])
        devs = (C.c_int * 1)(local)

        def call():
            rc = pkg.lib().p2_b200_encode_windows(C.addressof(sm.struct), mel_h.data_ptr(), fr, len(mine), devs, 1,
                                                  out_h.data_ptr())
            if rc != 0:
                raise pkg.Error(rc, "p2_b200_encode_windows failed (see stderr)")

        for _ in range(2):   # plan creation and its graph capture (on a plan's second run) outside the timing
            call()
        t0 = time.perf_counter()
        for _ in range(steps):
            call()
        e2e_ms = (time.perf_counter() - t0) / steps * 1e3
    barrier(world)
    e2e_max = max_over_ranks(e2e_ms, world)
    res = {"metric": "encoder audio-sec/sec", "value": audio_s / (ms_max / 1e3), "unit": "audio-s/s",
           "ms_per_step": ms_max, "steps": steps, "workload": desc, "windows": len(frames),
           "audio_seconds": audio_s, "rows_per_gpu": enc.total_frames if enc else 0, "mode": args.mode,
           "weights": args.weights, "timing": "CUDA events around graph launches, mel resident, max over ranks",
           "gpu_launches_per_step": None,
           "e2e": {"value": audio_s / (e2e_max / 1e3), "unit": "audio-s/s", "ms_per_step": e2e_max,
                   "h2d_bytes_per_step": sum(m.nbytes for m in mels), "d2h_bytes_per_step": n_out * 640 * 4,
                   "api": "p2_b200_encode_windows (page-locked host mel in, host frames out), wall clock, max over "
                          "ranks"}}
    if enc is not None:
        enc.close()
    dm.close()
    return res


# ---- the greedy TDT decoder and the whole transcription (encoder + decoder) ------------------------------------------

def decoder_frames(T, seed):
    """Joint-network input frames for the decoder workload: N(0, 1) [T, 640]. The synthetic encoder's own output
    varies too little from frame to frame to make the decoder emit tokens; on N(0, 1) frames it emits about one
    token every two frames, as speech does, so the decoder does the LSTM steps a real transcript costs."""
    return np.random.default_rng(seed).standard_normal((T, 640), dtype=np.float32)


def decoder_ours(args, world, rank, local, torch, pkg, steps=5):
    """Greedy TDT decoding of this rank's share of the config-3 windows (T'_i encoder frames each) in one launch per
    step, frames resident; then end to end through p2_greedy_decode window by window (host frames in, host tokens
    out), as the reference's engine calls it."""
    from phonon2_b200 import model as M
    frames, desc = encoder_workload("long-audio")
    T = [M.frames_after_subsampling(n) for n in frames]
    mine = shard_windows(frames, world)[rank]
    sm = M.SyntheticModel(seed=1)
    dm = pkg.DeviceModel(sm.struct)
    encs = [decoder_frames(T[w], seed=1000 + w) for w in mine]
    stream = torch.cuda.Stream()
    ms, n_tok = 0.0, 0
    dec = None
    if mine:
        x = torch.from_numpy(np.concatenate(encs)).to(f"cuda:{local}")
        dec = pkg.Decoder(dm, len(mine), sum(T[w] for w in mine))
        for _ in range(2):
            dec.decode(x.data_ptr(), [T[w] for w in mine], stream)
        n_tok = sum(len(t) for t in dec.read(stream))
    barrier(world)
    if dec is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            dec.decode(x.data_ptr(), [T[w] for w in mine], stream)
        e1.record(stream)
        e1.synchronize()
        pkg.check_device(stream)
        ms = e0.elapsed_time(e1) / steps
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    audio_s = sum(frames) * ENC_SECONDS_PER_FRAME
    e2e_ms = 0.0
    if mine:
        for e in encs[:1]:
            pkg.host_greedy_decode(sm.struct, e)   # plan creation outside the timed region
        t0 = time.perf_counter()
        for e in encs:
            pkg.host_greedy_decode(sm.struct, e)
        e2e_ms = (time.perf_counter() - t0) * 1e3
    barrier(world)
    e2e_max = max_over_ranks(e2e_ms, world)
    res = {"metric": "decoder audio-sec/sec", "value": audio_s / (ms_max / 1e3), "unit": "audio-s/s",
           "ms_per_step": ms_max, "steps": steps,
           "workload": desc + "; decoder input: N(0, 1) joint frames of each window's T' (seeded)",
           "frames": sum(T), "tokens_rank0": n_tok,
           "timing": "CUDA events around one cooperative decode launch over the rank's windows, max over ranks",
           "gpu_launches_per_step": 1,
           "e2e": {"value": audio_s / (e2e_max / 1e3), "unit": "audio-s/s", "ms_per_step": e2e_max,
                   "h2d_bytes_per_step": sum(e.nbytes for e in encs), "d2h_bytes_per_step": 12 * n_tok,
                   "api": "p2_greedy_decode window by window (host frames in, host tokens out), wall clock, "
                          "max over ranks"}}
    if dec is not None:
        dec.close()
    dm.close()
    return res


def decoder_reference(seconds=10.0):
    """phonon-2-c's own p2_greedy_decode on the host cores, on the decoder workload's windows for about `seconds`."""
    orc = ge.load_oracle()
    if not orc.ref_available():
        return None
    from phonon2_b200 import model as M
    frames, _ = encoder_workload("long-audio")
    sm = M.SyntheticModel(seed=1)
    done, t0, n = 0, time.perf_counter(), 0
    while True:
        w = n % len(frames)
        orc.ref_greedy_decode(sm.struct, decoder_frames(M.frames_after_subsampling(frames[w]), seed=1000 + w))
        done += frames[w]
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": done * ENC_SECONDS_PER_FRAME / dt, "unit": "audio-s/s", "cores": orc.ref_threads(),
            "kind": "reference",
            "sample": f"phonon-2-c p2_greedy_decode on {n} window(s) of the decoder workload in {dt:.1f} s, "
                      "P2_THREADS = all host cores"}


def mel_ours(args, world, rank, local, torch, pkg, steps=5):
    """The log-mel front end on this rank's share of the config-3 windows as 16 kHz audio (160 samples per mel frame):
    device-timed p2cu_mel_run over the rank's windows (audio resident); then the whole path from audio - log-mel,
    encoder, decoder - end to end through p2_b200_transcribe_audio_windows (host audio in, host tokens out)."""
    from phonon2_b200 import model as M
    frames, desc = encoder_workload("long-audio")
    mine = shard_windows(frames, world)[rank]
    ns = [frames[w] * 160 for w in mine]
    audios = [M.audio(n, seed=w) for n, w in zip(ns, mine)]
    stream = torch.cuda.Stream()
    ms = 0.0
    plan = None
    if mine:
        x = torch.from_numpy(np.concatenate(audios)).to(f"cuda:{local}")
        out = torch.empty((sum(n // 160 for n in ns), 128), device=f"cuda:{local}")
        plan = pkg.Mel(len(ns), sum(ns))
        for _ in range(2):
            plan.run(x.data_ptr(), ns, out.data_ptr(), stream)
        stream.synchronize()
    barrier(world)
    if plan is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            plan.run(x.data_ptr(), ns, out.data_ptr(), stream)
        e1.record(stream)
        e1.synchronize()
        pkg.check_device(stream)
        ms = e0.elapsed_time(e1) / steps
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    audio_s = sum(frames) * ENC_SECONDS_PER_FRAME
    sm = M.SyntheticModel(seed=1, attn_out_gain=M.SPEECH_ATTN_OUT_GAIN)
    e2e_ms = 0.0
    n_tok = 0
    if mine:
        import ctypes as C
        audio_h = torch.empty(sum(ns), dtype=torch.float32, pin_memory=True)
        audio_h.numpy()[...] = np.concatenate(audios)
        na = (C.c_longlong * len(ns))(*ns)
        devs = (C.c_int * 1)(local)
        toks_p = (C.c_void_p * len(ns))()
        counts = (C.c_int * len(ns))()
        libc = C.CDLL(None)
        libc.free.argtypes = [C.c_void_p]

        def call():   # p2_b200_transcribe_audio_windows, page-locked audio in, malloc'd token lists out (freed)
            rc = pkg.lib().p2_b200_transcribe_audio_windows(C.addressof(sm.struct), audio_h.data_ptr(), na, len(ns),
                                                            devs, 1, toks_p, counts)
            if rc != 0:
                raise pkg.Error(rc, "p2_b200_transcribe_audio_windows failed (see stderr)")
            total = sum(counts)
            for i in range(len(ns)):
                if toks_p[i]:
                    libc.free(toks_p[i])
            return total

        for _ in range(2):   # plans and their graph capture (on a plan's second run) outside the timing
            n_tok = call()
        t0 = time.perf_counter()
        for _ in range(2):
            call()
        e2e_ms = (time.perf_counter() - t0) / 2 * 1e3
    barrier(world)
    e2e_max = max_over_ranks(e2e_ms, world)
    res = {"metric": "log-mel audio-sec/sec", "value": audio_s / (ms_max / 1e3), "unit": "audio-s/s",
           "ms_per_step": ms_max, "steps": steps,
           "workload": desc + "; as synthetic 16 kHz audio (seeded harmonics under a syllable envelope)",
           "timing": "CUDA events around p2cu_mel_run over the rank's windows (audio resident), max over ranks",
           "gpu_launches_per_step": 2,
           "transcribe_audio": {"value": audio_s / (e2e_max / 1e3), "unit": "audio-s/s", "ms_per_step": e2e_max,
                                "tokens_rank0": n_tok, "h2d_bytes_per_step": 4 * sum(ns),
                                "d2h_bytes_per_step": 12 * n_tok,
                                "api": "p2_b200_transcribe_audio_windows: log-mel, encoder and decoder on the device "
                                       "(host audio in, host tokens out), wall clock, max over ranks"}}
    if plan is not None:
        plan.close()
    return res


def mel_reference(seconds=5.0):
    """phonon-2-c's own p2_mel_spectrogram on the host cores over the config-3 windows for about `seconds`."""
    orc = ge.load_oracle()
    if not orc.ref_available():
        return None
    from phonon2_b200 import model as M
    frames, _ = encoder_workload("long-audio")
    done, dt, n = 0.0, 0.0, 0
    while dt < seconds:
        w = n % len(frames)
        a = M.audio(frames[w] * 160, seed=w)
        t1 = time.perf_counter()
        orc.ref_mel_spectrogram(a)
        dt += time.perf_counter() - t1
        done += frames[w] * ENC_SECONDS_PER_FRAME
        n += 1
    return {"value": done / dt, "unit": "audio-s/s", "cores": orc.ref_threads(), "kind": "reference",
            "sample": f"phonon-2-c p2_mel_spectrogram on {n} window(s) of the workload, {dt:.1f} s inside the calls, "
                      "P2_THREADS = all host cores"}


def plane_bytes(sm) -> int:
    """Bytes of every five-value weight's planes and magnitudes (signs, flags, lo, hi) in a SyntheticModel: what one
    encoder pass reads from HBM at least once (230,031,360 for the 216 five-value tensors)."""
    return sum(a.nbytes for k, a in sm.arrays.items() if k.endswith((".signs", ".flags", ".lo", ".hi")))


def transcribe_reference(n_mel, reps=2):
    """phonon-2-c's p2_encoder (exact) then p2_greedy_decode on the host cores for one window of n_mel frames (the
    speech-like synthetic model, as the configs' objects use)."""
    orc = ge.load_oracle()
    if not orc.ref_available():
        return None
    from phonon2_b200 import model as M
    sm = M.SyntheticModel(seed=1, attn_out_gain=M.SPEECH_ATTN_OUT_GAIN)
    mel = M.mel(n_mel, seed=n_mel)
    t0 = time.perf_counter()
    for _ in range(reps):
        orc.ref_greedy_decode(sm.struct, orc.ref_encoder(sm.struct, mel, "exact"))
    ms = (time.perf_counter() - t0) / reps * 1e3
    return {"value": ms, "unit": "ms", "cores": orc.ref_threads(), "kind": "reference",
            "sample": f"phonon-2-c p2_encoder (exact, AVX2) + p2_greedy_decode, {reps} runs, P2_THREADS = all host "
                      "cores"}


LONG_SECONDS = 600.0


def long_audio_ours(pkg, world, rank, local, steps=3):
    """Long-form transcription (the engine's path for long audio): each rank transcribes its own 10-minute recording
    end to end through p2_b200_transcribe_long - pause-aligned windows, dropout re-decodes as one batch per split depth,
    log-mel, encoder and decoder on the device (host audio in, host tokens out). Weak scaling: every rank holds a
    recording (the same one, so that every rank has the same windows and re-decodes to do); value = all ranks' audio
    seconds / the slowest rank's wall time per recording."""
    from phonon2_b200 import model as M
    import torch
    sm = M.SyntheticModel(seed=1, attn_out_gain=M.SPEECH_ATTN_OUT_GAIN)
    x_h = torch.empty(int(LONG_SECONDS * 16000), dtype=torch.float32, pin_memory=True)   # page-locked recording
    x = x_h.numpy()
    x[...] = M.audio_with_pauses(LONG_SECONDS, 7)   # the same recording on every rank: the same work per rank
    wins, frames = pkg.host_transcribe_long(sm.struct, x, devices=[local])   # weights and plans outside the timing
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        wins, frames = pkg.host_transcribe_long(sm.struct, x, devices=[local])
    ms = (time.perf_counter() - t0) / steps * 1e3
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    depths = {}
    for w in wins:
        depths[str(w["depth"])] = depths.get(str(w["depth"]), 0) + 1
    n_tok = sum(len(w["tokens"]) for w in wins)
    return {"metric": "long-form transcription audio-sec/sec", "value": world * LONG_SECONDS / (ms_max / 1e3),
            "unit": "audio-s/s", "ms_per_step": ms_max, "steps": steps, "scaling": "weak",
            "workload": f"{LONG_SECONDS:.0f} s of synthetic long-form 16 kHz audio on each rank (bursts of 1-6 s under a "
                        "syllable envelope between pauses of 0.05-1.4 s, seeded), the speech-like synthetic model",
            "windows_by_depth_rank0": depths, "encoder_frames_rank0": frames, "tokens_rank0": n_tok,
            "h2d_bytes_per_step": 4 * int(x.shape[0]), "d2h_bytes_per_step": 12 * n_tok,
            "gpu_launches_per_step": "one mel + one encoder pass + one decoder launch per split depth and GPU, one "
                                     "block-RMS launch per planned window and per split depth",
            "api": "p2_b200_transcribe_long, wall clock (host audio -> host tokens per window), max over ranks"}


def long_audio_reference(seconds=70.0):
    """phonon-2-c's engine (p2_engine_open + p2_transcribe, exact: its x86 path) on the first `seconds` of the
    long-form recording, on the host cores."""
    orc = ge.load_oracle()
    if not orc.ref_available():
        return None
    import tempfile
    from phonon2_b200 import model as M
    from oracle import weights_file as wf
    x = M.audio_with_pauses(LONG_SECONDS, 7)[: int(seconds * 16000)]
    with tempfile.TemporaryDirectory() as d:
        wf.write_model_dir(M.SyntheticModel(seed=1, attn_out_gain=M.SPEECH_ATTN_OUT_GAIN), d)
        t0 = time.perf_counter()
        orc.ref_transcribe(d, x)
        dt = time.perf_counter() - t0
    return {"value": seconds / dt, "unit": "audio-s/s", "cores": orc.ref_threads(), "kind": "reference",
            "sample": f"phonon-2-c p2_transcribe on the first {seconds:.0f} s of the recording ({dt:.1f} s; its "
                      "windows and re-decodes one after another), exact mode, P2_THREADS = all host cores"}


ENCODER_MAX_STEPS = 20


def run_encoder_only(args, world, rank, local):
    """--workload encoder: the encoder alone, as its own line (the metric's "encoder audio-sec/sec")."""
    import torch
    pkg = ge.load_package()
    torch.cuda.set_device(local)
    steps = min(args.steps, ENCODER_MAX_STEPS)   # whole encoder passes (0.1-0.2 s each at config 3)
    enc = encoder_ours(args, world, rank, local, torch, pkg, workload=args.encoder_config, steps=steps,
                       windows=args.windows)
    if rank != 0:
        return
    line = {"metric": "encoder audio-sec/sec", "value": enc["value"], "unit": "audio-s/s", "n_gpus": world,
            "steps": steps, "warmup": 2, "ms_per_step": enc["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8" if args.mode != "exact" else "f32",
            "data": "synthetic", "config": {"workload": enc["workload"], "mode": args.mode, "weights": args.weights,
                                            "rows_per_gpu": enc["rows_per_gpu"]},
            "e2e": enc["e2e"]}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = encoder_reference(workload=args.encoder_config, windows=args.windows)
    print(json.dumps(line))


def probes_lib():
    """The hardware-rate probes (phonon-2-c_b200/libphonon2_probes.so, built beside the product library)."""
    import ctypes as C
    L = C.CDLL(str(ROOT / "phonon-2-c_b200" / "libphonon2_probes.so"))
    for name in ("p2cu_probe_int8_mma", "p2cu_probe_int8_ring", "p2cu_probe_tma_load"):
        getattr(L, name).argtypes = [C.c_int, C.c_int, C.POINTER(C.c_double)]
        getattr(L, name).restype = C.c_int
    L.p2cu_probes_last_error.restype = C.c_char_p
    return L


def probe_check(L, rc):
    if rc != 0:
        raise RuntimeError(f"probe failed ({rc}): {L.p2cu_probes_last_error().decode()}")


def measured_int8_peak(pkg, pair=False) -> float:
    """The tcgen05 int8 MMA rate measured on this GPU (p2cu_probe_int8_mma), in TMAC/s."""
    import ctypes as C
    L = probes_lib()
    v = C.c_double()
    probe_check(L, L.p2cu_probe_int8_mma(1 if pair else 0, 4000, C.byref(v)))
    return v.value / 1e12


def run_probes(args):
    """--workload probes: the hardware rates the GEMM design rests on, one JSON line each: the int8 MMA peak (one CTA
    per SM, and CTA pairs) and tiled TMA load throughput per SM by issuing warps and box size."""
    import ctypes as C
    import torch
    pkg = ge.load_package()
    torch.cuda.set_device(0)
    for pair in (False, True):
        print(json.dumps({"probe": "int8_mma", "cta_pairs": pair, "value": measured_int8_peak(pkg, pair),
                          "unit": "TMAC/s", "nominal": 2250.0,
                          "what": "tcgen05 kind::i8 MMAs from shared memory, M=%d N=256 K=32, all SMs" %
                                  (256 if pair else 128)}))
    v = C.c_double()
    for mode, what in ((0, "issued without hand-back after the first round"),
                       (1, "each stage handed back by the MMAs' commit, a producer arrive and the odd CTA's relay"),
                       (2, "each stage handed back by the MMAs' commit and producer arrives, the odd CTA's on the "
                           "even CTA's barrier")):
        probe_check(probes_lib(), probes_lib().p2cu_probe_int8_ring(mode, 4000, C.byref(v)))
        print(json.dumps({"probe": "int8_mma_ring", "mode": mode, "value": v.value / 1e12, "unit": "TMAC/s",
                          "what": "CTA-pair MMAs (M=256 N=256 K=128 per step) over a ring of six 32 KB stages, "
                                  "zero operands, no copies: " + what}))
    for box_rows in (32, 128, 256):
        for warps in (1, 2, 4):
            if 2 * warps * 128 * box_rows > 196608:
                continue
            probe_check(probes_lib(), probes_lib().p2cu_probe_tma_load(warps, box_rows, C.byref(v)))
            print(json.dumps({"probe": "tma_load", "issuing_warps": warps, "box_bytes": 128 * box_rows,
                              "value": v.value / 1e9, "unit": "GB/s per SM",
                              "what": "tiled TMA loads of 128-byte rows from an L2-resident int8 matrix, two boxes "
                                      "in flight per issuing warp"}))


def run_transcribe(args, local):
    """--workload transcribe: one window of --mel-frames mel frames (300 = configs[4], 3000 = configs[2]) from host
    mel to host tokens in int8w, the synthetic speech-like model. Prints the end-to-end time of
    p2_b200_transcribe_windows (wall clock) and its split measured with CUDA events on one stream through the plans it
    is built from: mel copy up, the encoder's graph, the decoder launch, the token read-back."""
    import torch
    pkg = ge.load_package()
    from phonon2_b200 import model as Mo
    from phonon2_b200.device import device_view
    torch.cuda.set_device(local)
    n_mel = args.mel_frames
    sm = Mo.SyntheticModel(seed=1, attn_out_gain=Mo.SPEECH_ATTN_OUT_GAIN)
    mel = Mo.mel(n_mel, seed=n_mel)
    steps = max(1, min(args.steps, 50))
    for _ in range(args.warmup):
        toks = pkg.host_transcribe_windows(sm.struct, [mel], devices=[local])
    t0 = time.perf_counter()
    for _ in range(steps):
        toks = pkg.host_transcribe_windows(sm.struct, [mel], devices=[local])
    e2e_ms = (time.perf_counter() - t0) / steps * 1e3
    dm = pkg.DeviceModel(sm.struct)
    enc = pkg.Encoder(dm, [n_mel], pkg.INT8W)
    dec = pkg.Decoder(dm, 1, enc.total_frames)
    mel_h = torch.empty(mel.shape, dtype=torch.float32, pin_memory=True)
    mel_h.numpy()[...] = mel
    dst = device_view(enc.mel_ptr, mel.shape)
    stream = torch.cuda.Stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    split = np.zeros(3)
    for it in range(args.warmup + steps):
        with torch.cuda.stream(stream):
            ev[0].record(stream)
            dst.copy_(mel_h, non_blocking=True)
            ev[1].record(stream)
        enc.run(stream)
        with torch.cuda.stream(stream):
            ev[2].record(stream)
        dec.decode(enc.out_ptr, enc.frames, stream)
        with torch.cuda.stream(stream):
            ev[3].record(stream)
        got = dec.read(stream)
        if it >= args.warmup:
            split += [ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3])]
    split /= steps
    assert len(got) == len(toks) and all(np.array_equal(a, b) for a, b in zip(got, toks)), \
        "plans and the host entry point disagree"
    dec.close()
    enc.close()
    dm.close()
    print(json.dumps({"workload": "transcribe", "mel_frames": n_mel, "encoder_frames": enc.frames[0],
                      "tokens": int(len(toks[0])), "steps": steps, "e2e_ms": round(e2e_ms, 3),
                      "split_ms": {"mel_up": round(split[0], 3), "encoder_graph": round(split[1], 3),
                                   "decoder": round(split[2], 3)},
                      "api": "p2_b200_transcribe_windows (wall clock); split by CUDA events through the plans"}))


def run_attention(args, local):
    """--workload attention: the encoder's relative-position self-attention alone (p2cu_rel_attention, one launch of
    attn_rel_tc_kernel) on the config-3 windows' encoder lengths (--windows N: the first N), synthetic N(0, 0.25)
    Q | K | V rows and positions resident on the device, CUDA events around the timed calls. Reports the reference's
    fp32 multiply-adds per call (AC, the full BD band of 2T - 1 positions, the context) and the tf32 products the
    kernel executes (three per product, 64-key chunks and 64-position pieces, rows padded to the 128-query tile)."""
    import ctypes as C
    import torch
    pkg = ge.load_package()
    from phonon2_b200 import model as Mo
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    mel_frames = Mo.long_audio_windows(0)
    if args.windows:
        mel_frames = mel_frames[:args.windows]
    Ts = [Mo.frames_after_subsampling(n) for n in mel_frames]
    Tmax, R = max(Ts), sum(Ts)
    g = torch.Generator(device=dev).manual_seed(5)
    qkv = 0.5 * torch.randn(R, 3072, device=dev, generator=g)
    P = 0.5 * torch.randn(2 * Tmax - 1, 1024, device=dev, generator=g)
    bu = 0.1 * torch.randn(1024, device=dev, generator=g)
    bv = 0.1 * torch.randn(1024, device=dev, generator=g)
    out = torch.empty(R, 1024, device=dev)
    L = pkg.lib()
    Tarr = (C.c_int * len(Ts))(*Ts)
    nws = L.p2cu_rel_attention_ws_bytes(len(Ts), Tarr)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)

    def call():
        pkg.check(L.p2cu_rel_attention(qkv.data_ptr(), P.data_ptr(), bu.data_ptr(), bv.data_ptr(), Tarr, len(Ts), Tmax,
                                       out.data_ptr(), ws.data_ptr(), nws, None))
    steps = max(1, min(args.steps, 50))
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    pkg.check_device()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    e1.synchronize()
    pkg.check_device()
    ms = e0.elapsed_time(e1) / steps
    fp32_macs = sum(8 * 128 * T * (T + (2 * T - 1) + T) for T in Ts)
    tf32_macs = 0
    for T in Ts:
        nch = (T + 63) // 64
        tf32_macs += ((T + 127) // 128) * 8 * 3 * (nch * (2 * 128 * 64 * 128 + 128 * 128 * 64) + 2 * 128 * 64 * 128)
    print(json.dumps({"workload": "attention", "windows": len(Ts), "rows": R, "Tmax": Tmax,
                      "ctas": 8 * sum((T + 127) // 128 for T in Ts), "steps": steps, "ms_per_call": round(ms, 4),
                      "fp32_macs": fp32_macs, "tf32_macs_executed": tf32_macs,
                      "tf32_tmacs_per_s": round(tf32_macs / ms / 1e9, 1),
                      "api": "p2cu_rel_attention (include/p2cuda.h), device rows, CUDA events"}))


def run_gemm_sweep(args):
    """--workload gemm-sweep: the five-value GEMM alone (quantised A resident) at growing M, K = 1024, N = 4096 (the
    north star's large-M shape) and K = 4096, N = 1024; planes and the code cache. One JSON line per case."""
    import torch
    pkg = ge.load_package()
    from phonon2_b200 import synth
    from phonon2_b200.device import DeviceFiveValue
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s = torch.cuda.Stream()
    peak = measured_int8_peak(pkg)
    shapes = [(375, 1024, 4096), (1500, 1024, 4096), (4096, 1024, 4096), (8192, 1024, 4096), (24000, 1024, 4096),
              (8192, 4096, 1024)]
    if args.gemm_shape:
        shapes = [tuple(int(x) for x in args.gemm_shape.split(","))]
    for (M, K, N) in shapes:
        w = synth.five_value(K, N, seed=1)
        for form in ((args.weights,) if args.gemm_shape else ("planes", "codes", "vindex")):
            codes = form == "codes"
            B = DeviceFiveValue(w, dev, codes=codes, vindex=form == "vindex")
            A = torch.from_numpy(synth.activations(M, K, seed=2)).to(dev)
            q = torch.empty((M, K), dtype=torch.int8, device=dev)
            sc = torch.empty(M, dtype=torch.float32, device=dev)
            pkg.quant_rows(A.data_ptr(), M, K, K, q.data_ptr(), sc.data_ptr())
            C = torch.zeros((M, N), dtype=torch.float32, device=dev)
            nws = max(pkg.q8a_workspace_bytes(M, N, K), 256)
            ws = torch.empty(nws, dtype=torch.uint8, device=dev)
            mode = pkg.MODES[args.mode if args.mode != "exact" else "int8w"]

            def run():
                pkg.sgemm_fvb_q8a(M, N, K, 1.0, q.data_ptr(), sc.data_ptr(), B.struct, mode, 0.0, C.data_ptr(), N,
                                  ws.data_ptr(), nws, s)
            with torch.cuda.stream(s):
                for _ in range(args.warmup):
                    run()
                s.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for _ in range(10):
                        run()
                g.replay()
                s.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = max(1, args.steps // 10)
                e0.record(s)
                for _ in range(reps):
                    g.replay()
                e1.record(s)
                e1.synchronize()
            pkg.check_device(s)
            us = e0.elapsed_time(e1) / (10 * reps) * 1e3
            tmacs = M * K * N / (us / 1e6) / 1e12
            print(json.dumps({"metric": "five-value int8 GEMM TMAC/s", "M": M, "K": K, "N": N, "mode": args.mode,
                              "weights": form, "us": us, "value": tmacs, "unit": "TMAC/s",
                              "frac_of_nominal_int8": tmacs / 2250.0, "measured_int8_peak": peak,
                              "frac_of_measured_int8": tmacs / peak,
                              "hbm_bound_us": (M * K + (K * N if codes else 3 * K * N // 8) + 4 * M * N) / 6534.8e3}))


def encoder_reference(seconds=15.0, workload="long-audio", windows=0):
    """phonon-2-c's own p2_encoder (exact, its only x86 path) on the host cores, on the first windows of the
    workload for about `seconds`."""
    orc = ge.load_oracle()
    if not orc.ref_available():
        return None
    from phonon2_b200 import model as M
    frames, desc = encoder_workload(workload, windows)
    sm = M.SyntheticModel(seed=1)
    done, t0, n = 0.0, time.perf_counter(), 0
    while True:
        w = n % len(frames)
        orc.ref_encoder(sm.struct, M.mel(frames[w], seed=w), "exact")
        done += frames[w] * ENC_SECONDS_PER_FRAME
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": done / dt, "unit": "audio-s/s", "cores": orc.ref_threads(), "kind": "reference",
            "sample": f"phonon-2-c p2_encoder (exact, AVX2) on {n} window(s) of the workload ({done:.0f} s of audio) "
                      f"in {dt:.1f} s, P2_THREADS = all host cores"}


def run_e2e(pkg, torch, dev, stream, gset, mode, args, seed):
    """The same step through the reference-facing C ABI: p2_sgemm_fvb (include/blas.h, csrc/blas.h:65-67) with the
    weights as host planes (uploaded by the library on first use, outside the timing) and page-locked host buffers.
    Each call uploads its fp32 activations (and C_old where beta != 0), runs the GEMM and returns with C in host
    memory, so the step is timed by the wall clock around the nine calls."""
    import ctypes as C
    from phonon2_b200 import synth
    L = pkg.lib()
    calls = []
    for i, (M, K, N, alpha, beta, _, _, _, _) in enumerate(gset.items):
        w = synth.five_value(K, N, seed=1000 * seed + i)
        a = torch.empty((M, K), dtype=torch.float32, pin_memory=True)
        a.copy_(torch.from_numpy(synth.activations(M, K, seed=2000 * seed + i)))
        c = torch.zeros((M, N), dtype=torch.float32, pin_memory=True)
        fvb = pkg.host_five_value(w)
        if args.weights == "codes":   # the code cache, as the reference's P2_CACHE_CODES selects it
            fvb = pkg.host_five_value(w, codes=L.p2_fv_pack_codes(C.byref(fvb), K, N))
        calls.append((M, K, N, alpha, beta, w, fvb, a, c))
    h2d = sum(a.numel() * 4 + (c.numel() * 4 if beta != 0 else 0) for (_, _, _, _, beta, _, _, a, c) in calls)
    d2h = sum(c.numel() * 4 for (_, _, _, _, _, _, _, _, c) in calls)
    steps = max(10, min(args.steps, 200))

    def step():
        for (M, K, N, alpha, beta, w, fvb, a, c) in calls:
            L.p2_sgemm_fvb(M, N, K, alpha, a.data_ptr(), K, C.byref(fvb), beta, c.data_ptr(), N)

    for _ in range(3):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    ms = (time.perf_counter() - t0) / steps * 1e3
    return {"value": block_macs() / (ms / 1e3) / 1e12, "unit": "TMAC/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": ms,
            "api": "p2_sgemm_fvb (include/blas.h) on page-locked host buffers, nine calls per step, wall clock"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["int8w", "int8", "exact"], default="int8w")
    ap.add_argument("--weights", choices=["planes", "codes", "vindex"], default="vindex",
                    help="vindex: the planes as the library uploads them (the reference's sign/magnitude planes plus "
                         "the value-index plane packed from them once, which the int8w GEMMs of one window read); "
                         "planes: the reference's planes alone, expanded in every GEMM; codes: the int8w code cache "
                         "(the reference's P2_CACHE_CODES), int8w only")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-config objects at the end of the line")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-encoder", action="store_true", help="skip the encoder (config 3) part of the line")
    ap.add_argument("--no-decoder", action="store_true",
                    help="skip the decoder (config 3 windows) and transcription (configs 2, 4) parts of the line")
    ap.add_argument("--workload", choices=["block-gemms", "encoder", "gemm-sweep", "probes", "transcribe",
                                           "attention"],
                    default="block-gemms",
                    help="block-gemms: configs[1] with the encoder object (default); encoder: the encoder alone; "
                         "gemm-sweep: the GEMM alone at growing M (one line per case); attention: the encoder's "
                         "attention kernel alone on the config-3 windows")
    ap.add_argument("--encoder-config", choices=["long-audio", "window", "short"], default="long-audio",
                    help="--workload encoder: configs[3] (64 windows), [2] (one 30 s window) or [4] (3 s)")
    ap.add_argument("--windows", type=int, default=0,
                    help="--workload encoder long-audio / attention: only the first N windows")
    ap.add_argument("--gemm-shape", default="", help="--workload gemm-sweep: only this M,K,N (with --weights)")
    ap.add_argument("--mel-frames", type=int, default=300, help="--workload transcribe: the window's mel frames")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "encoder":
            run_encoder_only(args, world, rank, local)
        elif args.workload == "gemm-sweep":
            if rank == 0:
                run_gemm_sweep(args)
        elif args.workload == "probes":
            if rank == 0:
                run_probes(args)
        elif args.workload == "transcribe":
            if rank == 0:
                run_transcribe(args, local)
        elif args.workload == "attention":
            if rank == 0:
                run_attention(args, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
