#!/usr/bin/env python
"""Benchmark of the RVQ encode hot path.

Workload: N = 2^20 vectors of D = 1024 (bf16, N(0,1), seeded synthetic data),
8 residual levels with K = 16384 codewords each (level l ~ N(0, 0.6^l)),
codebooks replicated, token rows sharded across the ranks (the fixed-size
config-5 problem: strong scaling), codes and reconstructions all-gathered
over NCCL after the encode. One step = one encode of the whole problem.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU runs are launched by torchrun, one rank per GPU. Rank 0 prints ONE
JSON line. `--impl reference` times the CPU restatement of the path (the
reference has no runnable implementation here) on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "rvq_encode_vectors_per_s"
UNIT = "vectors/s"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--rows", type=int, default=1 << 20)
    p.add_argument("--dim", type=int, default=1024)
    p.add_argument("--levels", type=int, default=8)
    p.add_argument("--codes", type=int, default=16384)
    p.add_argument("--cpu-rows", type=int, default=2048, help="rows per CPU-baseline sample")
    p.add_argument("--seed", type=int, default=20260)
    p.add_argument("--transport", choices=["peer", "nccl"], default="peer",
                   help="N>1: copy-engine pushes over CUDA IPC mappings (peer) or NCCL all-gather kernels")
    p.add_argument("--graph", action="store_true",
                   help="secondary workloads: replay one captured CUDA graph per step")
    p.add_argument("--upsample", choices=["nearest", "linear"], default="nearest",
                   help="tokenizer workload: upsampling mode of each scale's reconstruction")
    p.add_argument("--phi", action="store_true",
                   help="tokenizer workload: apply the quantiser's Phi convolution after each upsampling")
    p.add_argument("--workload", choices=["rvq", "tokenizer", "linear", "decoder", "aux"], default="rvq",
                   help="rvq = BASELINE config 5 (the headline); tokenizer = config 2; linear = config 3 sweep; "
                        "decoder = config 4")
    return p.parse_args()


def config_dict(a, world):
    return {
        "workload": "rvq_encode (BASELINE config 5)",
        "rows": a.rows,
        "dim": a.dim,
        "levels": a.levels,
        "codebook_size": a.codes,
        "rows_per_gpu": a.rows // world,
        "parallelism": f"row-sharded x{world}, codebooks replicated",
        "collective": (("copy-engine pushes of codes and bf16 reconstructions into every rank's output buffers over "
                        "CUDA IPC mappings, between two one-element NCCL all-reduces, on a second stream overlapping "
                        "the next step's encode") if a.transport == "peer" else
                       "NCCL all_gather of codes and bf16 reconstructions, on a second stream overlapping the "
                       "next step's encode") if world > 1 else "none (1 GPU)",
        "l2": "inputs exceed L2 (bf16 rows 2 GiB/N, f32 residual 4 GiB/N); codebooks (32 MiB/level) stay L2-resident by design",
        "data": "synthetic seeded N(0,1) rows, N(0,0.6^l) codebooks",
    }


# ---------------------------------------------------------------- clocks
_RESULT_FD = None


def _claim_stdout():
    """The JSON result line is the only thing this program writes to stdout:
    library and runtime messages (NCCL's version banner, warnings) that would
    go to file descriptor 1 are sent to stderr instead."""
    global _RESULT_FD
    if _RESULT_FD is None:
        sys.stdout.flush()
        _RESULT_FD = os.dup(1)
        os.dup2(2, 1)


def emit(line: dict) -> None:
    data = (json.dumps(line) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, data)


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = str(gpu_index)
        self.proc = None
        # raw samples: NCM_CLOCKS_DIR when set (to keep them), else the temp directory
        out_dir = os.environ.get("NCM_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = pathlib.Path(out_dir) / f"clocks_bench_{os.getpid()}.csv"

    def start(self):
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # the first sample lands before the timed region starts, so even a short
        # region (a few 30 ms steps at 8 GPUs) is covered by the sampling loop
        t0 = time.time()
        while time.time() - t0 < 2.0 and self.proc.poll() is None:
            if self.path.stat().st_size > 0:
                break
            time.sleep(0.01)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        mhz, maxmhz, reasons = [], [], set()
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9 or parts[0] != self.gpu:
                continue
            try:
                mhz.append(float(parts[1]))
                maxmhz.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxmhz), "samples": len(mhz),
                "reasons": sorted(reasons)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(rows_per_launch: int):
    """DRAM bytes per rvq_argmin launch from the committed ncu summary, scaled
    from the captured case to this launch by rows (traffic ~ rows * D * 2
    plus one codebook read)."""
    p = ROOT / "profiles" / "rvq_argmin_pair_kernel_n131072.md"
    if not p.exists():
        return None
    d = {}
    for line in p.read_text().splitlines():
        parts = line.strip().split(":")
        if len(parts) == 2 and parts[0] in ("rows", "dram_bytes_per_launch", "codebook_bytes"):
            d[parts[0]] = float(parts[1])
    if len(d) != 3:
        return None
    per_row = (d["dram_bytes_per_launch"] - d["codebook_bytes"]) / d["rows"]
    return per_row * rows_per_launch + d["codebook_bytes"]


# ------------------------------------------------------------ CPU leg
def cpu_encode_sample(a, rows: int, threads: int):
    """Times the oracle (the CPU restatement of the path) on `rows` rows of the
    same workload. Returns (seconds, rows)."""
    from oracle import pyoracle as orc
    rng = np.random.default_rng(a.seed + 99)
    x = orc.bf16_bits(rng.standard_normal((rows, a.dim)).astype(np.float32))
    cbs = np.stack([orc.bf16_bits((rng.standard_normal((a.codes, a.dim)) * 0.6 ** l).astype(np.float32))
                    for l in range(a.levels)])
    t0 = time.perf_counter()
    orc.rvq_encode(x, cbs, threads=threads)
    return time.perf_counter() - t0, rows


def cpu_leg_and_parity(a, x, cbs, codes):
    """The CPU baseline and the code parity of the headline workload, on one
    sample of the GPU's own rows: the oracle port encodes `a.cpu_rows` rows on
    its own (timed: the baseline), then once more teacher-forced by the GPU's
    codes. Reports the flip rate (codes differing from the oracle's argmin on
    the same residual), the near-tie rate (oracle top-2 gap below 1e-3 of the
    best full squared distance), flips outside near-ties (must be 0), and how
    many rows' free-running code sequences diverge."""
    import torch
    from oracle import pyoracle as orc
    threads = os.cpu_count() or 1
    n = x.shape[0]
    L, K, D = cbs.shape
    g = torch.Generator().manual_seed(a.seed + 7)
    idx = torch.sort(torch.randperm(n, generator=g)[: min(a.cpu_rows, n)]).values
    idx_d = idx.to(x.device)
    xs = x[idx_d].view(torch.int16).cpu().numpy().view(np.uint16)
    cs = codes[:, idx_d].cpu().numpy()
    cbs_np = cbs.view(torch.int16).cpu().numpy().view(np.uint16)
    rows = idx.numel()
    t0 = time.perf_counter()
    free_best, _, _, _ = orc.rvq_encode(xs, cbs_np, threads=threads)
    sec = time.perf_counter() - t0
    cpu = {"value": rows / sec, "unit": UNIT, "cores": threads, "kind": "port",
           "sample": (f"{rows} of the GPU's rows x {L} levels x K={K} x D={D}, encoded free-running by the oracle "
                      f"port (its per-level codebook transpose included)")}
    tf_best, gaps, _, _ = orc.rvq_encode(xs, cbs_np, codes_in=cs, threads=threads)
    flips = cs != tf_best
    near = gaps < 1e-3
    diverged = (cs != free_best).any(axis=0)
    parity = {"rows": rows, "codes": int(cs.size), "flip_rate": float(flips.mean()),
              "near_tie_rate": float(near.mean()), "flips_outside_near_ties": int((flips & ~near).sum()),
              "free_running_diverged_rows": int(diverged.sum()),
              "rule": ("teacher-forced: the oracle advances with the GPU's codes, so each flip is a level-local "
                       "argmin difference; near-tie = oracle top-2 gap < 1e-3 of the best full squared distance")}
    return cpu, parity


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    for _ in range(a.warmup):
        cpu_encode_sample(a, a.cpu_rows, threads)
    times = []
    for _ in range(a.steps):
        s, n = cpu_encode_sample(a, a.cpu_rows, threads)
        times.append(s)
    sec = sum(times) / len(times)
    value = a.cpu_rows / sec
    sample = (f"{a.cpu_rows} rows x {a.levels} levels x K={a.codes} x D={a.dim} per step "
              f"(oracle port, includes its per-level codebook transpose)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 operands, f32 accumulation", "data": "synthetic",
        "config": config_dict(a, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


# ------------------------------------------------------------ GPU leg
def run_ours(a):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    from ncmorph_b200 import _lib, device as ndev, vq
    import ctypes

    if a.rows % world:
        raise SystemExit("rows must divide evenly across ranks")
    n = a.rows // world
    L, K, D = a.levels, a.codes, a.dim
    g = torch.Generator(device=dev).manual_seed(a.seed + 1000 * rank)
    x = torch.randn((n, D), generator=g, device=dev).to(torch.bfloat16)
    gc = torch.Generator(device=dev).manual_seed(a.seed)  # same codebooks on every rank
    decay = torch.tensor([0.6 ** l for l in range(L)], device=dev).view(L, 1, 1)
    cbs = (torch.randn((L, K, D), generator=gc, device=dev) * decay).to(torch.bfloat16)
    sq = vq.code_sqnorm(cbs)
    codes = torch.empty((L, n), dtype=torch.int32, device=dev)
    recon = torch.empty((n, D), dtype=torch.bfloat16, device=dev)
    ctx = ndev.context(dev)
    lib = _lib.load()
    if world > 1:
        from ncmorph_b200.sharded import ShardedEncoder
        # batches stream: a step's all-gathers overlap the next step's encode
        encoder = ShardedEncoder(cbs, a.rows, torch.bfloat16, sq, overlap=True, transport=a.transport)
    result = {}

    def step():
        if world > 1:
            result["codes"], result["recon"] = encoder(x)
        else:
            vq.rvq_encode(x, cbs, sq, codes=codes, recon=recon)
            result["codes"], result["recon"] = codes, recon

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps, finish=None):
        """Device time per step, max over ranks; finish() makes the current
        stream wait for work the steps left on other streams, so the closing
        event covers it."""
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        if finish is not None:
            finish()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / steps)

    for _ in range(a.warmup):
        step()
    ndev.sync(dev)

    # ---- value: device-resident inputs; per-kernel events for the roofline
    lib.ncm_profile_read(ctx, b"*", None, None)
    lib.ncm_profile_enable(ctx, 1)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    ms = timed(step, a.steps, encoder.wait if world > 1 else None)
    clocks = sampler.stop() if sampler else None
    lib.ncm_profile_enable(ctx, 0)
    tot = ctypes.c_double()
    cnt = ctypes.c_int64()
    _lib.check(lib.ncm_profile_read(ctx, b"rvq_argmin", ctypes.byref(tot), ctypes.byref(cnt)))
    argmin_ms, argmin_launches = tot.value, cnt.value
    _lib.check(lib.ncm_profile_read(ctx, b"rvq_decode", ctypes.byref(tot), ctypes.byref(cnt)))
    decode_ms, decode_launches = tot.value, cnt.value
    other_ms = ctypes.c_double()
    other_cnt = ctypes.c_int64()
    _lib.check(lib.ncm_profile_read(ctx, b"*", ctypes.byref(other_ms), ctypes.byref(other_cnt)))
    launches = argmin_launches + decode_launches + other_cnt.value
    ndev.sync(dev)
    argmin_avg_ms = max_over_ranks(argmin_ms / max(argmin_launches, 1))
    kernel_share = argmin_ms / max(argmin_ms + decode_ms + other_ms.value, 1e-9)
    # per-step device time of each kernel family (CUDA events around every launch)
    kernels = {"rvq_argmin": {"ms_per_step": argmin_ms / a.steps, "launches": argmin_launches},
               "rvq_decode": {"ms_per_step": decode_ms / a.steps, "launches": decode_launches},
               "other": {"ms_per_step": other_ms.value / a.steps, "launches": other_cnt.value}}

    # ---- e2e: host rows in, codes and reconstructions out.
    # N=1: the host-buffer C-ABI entry (ncm_rvq_encode_host) with its chunked
    # copy/compute pipeline. N>1: rows copied in, sharded encode + all-gather;
    # every rank copies out the gathered codes and its own rows of the
    # gathered reconstruction, so the host receives the whole reconstruction
    # once across the ranks, as at N=1.
    x_host = torch.empty((n, D), dtype=torch.bfloat16).pin_memory()
    x_host.copy_(x.cpu())
    codes_host = torch.empty((L, a.rows), dtype=torch.int32).pin_memory()
    recon_host = torch.empty((n, D), dtype=torch.bfloat16).pin_memory()

    if world == 1:
        def step_e2e():
            vq.rvq_encode_host(x_host, cbs, sq, codes_host=codes_host, recon_host=recon_host)
        finish_e2e = None
    else:
        # streaming batches: step i+1's rows are copied in on a second stream
        # (into the other of two row buffers) and step i's gathered codes and
        # own reconstruction rows are copied out on a third, while the encode
        # and its all-gathers proceed
        cp, d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        xbuf = [x, torch.empty_like(x)]
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        consumed = [torch.cuda.Event(), torch.cuda.Event()]
        drained = [torch.cuda.Event(), torch.cuda.Event()]
        st = {"i": 0, "n": 1}
        own = slice(rank * n, (rank + 1) * n)

        def step_e2e():
            i = st["i"]
            b = i & 1
            cur = torch.cuda.current_stream()
            if i == 0:
                with torch.cuda.stream(cp):
                    cp.wait_stream(cur)
                    xbuf[0].copy_(x_host, non_blocking=True)
                    copied[0].record(cp)
            if i + 1 < st["n"]:
                with torch.cuda.stream(cp):  # the next step's rows
                    if i >= 1:
                        cp.wait_event(consumed[b ^ 1])
                    xbuf[b ^ 1].copy_(x_host, non_blocking=True)
                    copied[b ^ 1].record(cp)
            cur.wait_event(copied[b])
            if i >= 2:
                cur.wait_event(drained[b])   # step i-2's results (same buffer set) are copied out
            codes_d, recon_d = encoder(xbuf[b])
            consumed[b].record(cur)
            with torch.cuda.stream(d2h):
                encoder.wait()
                codes_host.copy_(codes_d, non_blocking=True)
                recon_host.copy_(recon_d[own], non_blocking=True)
                drained[b].record(d2h)
            st["i"] = i + 1

        def finish_e2e():
            torch.cuda.current_stream().wait_stream(d2h)
            torch.cuda.current_stream().wait_stream(cp)

    step_e2e()
    torch.cuda.synchronize()
    if world > 1:
        st.update(i=0, n=a.steps)
    ms_e2e = timed(step_e2e, a.steps, finish_e2e)
    ndev.sync(dev)

    value = a.rows / (ms * 1e-3)
    e2e_value = a.rows / (ms_e2e * 1e-3)
    peaks, peak_kind = measured_peaks()
    flops_per_launch = 2.0 * n * K * D
    achieved = flops_per_launch / (argmin_avg_ms * 1e-3) / 1e12
    peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
    traffic = ncu_traffic(n)

    cpu = parity = extra = None
    if rank == 0 and world == 1:
        cpu, parity = cpu_leg_and_parity(a, x, cbs, codes)
        extra = run_extras(a, dev)

    if world > 1:
        torch.cuda.synchronize()
        encoder.close()   # unmaps the peers' buffers (collective)
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 operands, f32 accumulation", "data": "synthetic", "config": config_dict(a, world),
        "e2e": {"value": e2e_value, "unit": UNIT, "ms_per_step": ms_e2e, "h2d_bytes_per_step": n * D * 2,
                "d2h_bytes_per_step": int(codes_host.numel() * 4 + recon_host.numel() * 2),
                "path": "ncm_rvq_encode_host (chunked H2D/encode/D2H pipeline)" if world == 1
                        else ("H2D rows (next step's on a copy stream), sharded encode, all-gather on a second "
                              "stream, D2H of the gathered codes and this rank's reconstruction rows on a third")},
        "roofline": {"bound": "tensor", "kernel": "rvq_argmin_kernel", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} bf16_tflops_sustained (kernel timed inside a long step)",
                     "frac_of_burst": achieved / float(peaks["bf16_tflops"]),
                     "flops_per_launch": flops_per_launch, "avg_launch_ms": argmin_avg_ms,
                     "launches": argmin_launches, "share_of_kernel_time": kernel_share,
                     "traffic": traffic},
        "kernels": kernels,
        "cpu_baseline": cpu,
        "parity": parity,
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if extra is not None:
        line["extra"] = extra
    emit(line)
    return 0


# ------------------------------------------------- secondary workloads
# Configs 1-4 are parity cases; these modes measure them on one GPU with the
# same timing rules (CUDA events, warm-up, clocks) as the headline line.

def _timed_loop(fn, steps, warmup):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / max(steps, 1)


def _tokenizer_e2e(x, x_host, codes_host, forward, steps):
    """Streaming end-to-end time per step: every step copies its input (pinned
    host -> device) and reads its codes back (device -> pinned host) inside the
    timed region; the next step's input copy runs on a second stream into the
    other of two device buffers while this step computes."""
    import torch
    cur = torch.cuda.current_stream()
    cp = torch.cuda.Stream()
    bufs = [torch.empty_like(x), torch.empty_like(x)]
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]

    def run(n):
        with torch.cuda.stream(cp):
            cp.wait_stream(cur)
            bufs[0].copy_(x_host, non_blocking=True)
            copied[0].record(cp)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                with torch.cuda.stream(cp):
                    if i >= 1:
                        cp.wait_event(consumed[b ^ 1])  # step i-1 finished reading that buffer
                    bufs[b ^ 1].copy_(x_host, non_blocking=True)
                    copied[b ^ 1].record(cp)
            cur.wait_event(copied[b])
            codes = forward(bufs[b])
            consumed[b].record(cur)
            codes_host.copy_(torch.cat([c.reshape(-1) for c in codes]), non_blocking=True)

    run(2)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    run(steps)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / max(steps, 1)


def _l2_flusher(dev):
    """Returns a function that evicts L2 between timed calls by reading a
    256 MiB buffer. L2 is left holding clean lines, so a timed call neither
    finds its data cached nor pays to write back another kernel's dirty
    lines (a written flush buffer would leave those)."""
    import torch
    buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    return lambda: buf.sum()


def _event_ms(fn, reps, flush=None):
    """Median CUDA-event time of fn over reps calls; flush() (an L2-sized
    read) runs before each call, outside the timed window."""
    import torch
    times = []
    for _ in range(reps):
        if flush is not None:
            flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return sorted(times)[len(times) // 2]


def _write_safetensors(path, tensors):
    """Minimal safetensors writer: 8-byte little-endian header length, JSON
    header with dtype/shape/data_offsets, then the raw little-endian bytes."""
    import json as _json
    import struct
    header, blobs, off = {}, [], 0
    for name, (dtype, arr) in tensors.items():
        b = arr.tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = _json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    return 8 + len(h) + off


def _aux_suite(a, dev, rnd, peaks, peak_kind):
    """The next-row pieces measured against their rooflines: the tied
    codebook head (tensor), the device loader (host-to-device copy), and the
    training-time quantiser pieces (HBM / tensor)."""
    import os
    import tempfile

    import numpy as np
    import torch

    from ncmorph_b200 import loader, ncm_model, quantizer
    hbm = float(peaks["hbm_gbs"])
    tensor = float(peaks["bf16_tflops"])
    flush = _l2_flusher(dev)
    reps = max(a.steps, 5)
    out = {}

    # (f)3 tied codebook head at the NCM shapes: T = 4096 positions, d = 1024, K = 4096 codes
    T, d, K = 4096, 1024, 4096
    z, cb = rnd((T, d)), rnd((K, d))
    bias = torch.zeros(K, dtype=torch.float32, device=dev)
    from ncmorph_b200 import vq
    esq = vq.code_sqnorm(cb)  # the codebook's norms, computed once per model as a caller would
    flops = 2.0 * T * K * d
    for name, fn in (("tied_head_logits", lambda: ncm_model.tied_head_logits(z, cb, 0.5, bias, esq)),
                     ("tied_head_argmax", lambda: ncm_model.tied_head_argmax(z, cb, 0.5, bias, esq))):
        for _ in range(3):
            fn()
        ms = _event_ms(fn, reps, flush)
        ach = flops / (ms * 1e-3) / 1e12
        out[name] = {"value": ach, "unit": "TFLOP/s", "ms": ms, "shape": [T, d, K],
                     "roofline": {"bound": "tensor", "achieved": ach, "peak": tensor, "unit": "TFLOP/s",
                                  "frac": ach / tensor, "peak_source": f"{peak_kind} bf16_tflops (burst)"}}

    # (f)2 device loader: a synthetic checkpoint (bf16, f16 and f32 tensors) read from the page cache
    rng = np.random.default_rng(a.seed)
    tmp = tempfile.mkdtemp()
    path = os.path.join(tmp, "synthetic.safetensors")
    try:
        w32 = rng.standard_normal((4096, 4096), dtype=np.float32)
        tensors = {"bf16": ("BF16", (rng.standard_normal((8192, 8192), dtype=np.float32).view(np.uint32) >> 16)
                            .astype(np.uint16)),
                   "f16": ("F16", w32[:, :].astype(np.float16).reshape(8192, 2048)),
                   "f32": ("F32", w32)}
        nbytes = _write_safetensors(path, tensors)
        loader.load_all_bf16(path, dev)               # warm the page cache and the staging buffers
        torch.cuda.synchronize()
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            loaded = loader.load_all_bf16(path, dev)
            torch.cuda.synchronize()
            times.append(time.perf_counter() - t0)
        sec = sorted(times)[1]
        host = torch.empty(nbytes // 4, dtype=torch.float32).pin_memory()
        devbuf = torch.empty_like(host, device=dev)
        h2d_ms = _event_ms(lambda: devbuf.copy_(host, non_blocking=True), 3)
        h2d = host.numel() * 4 / (h2d_ms * 1e-3) / 1e9
        gbs = nbytes / sec / 1e9
        out["loader"] = {"value": gbs, "unit": "GB/s (file bytes)", "file_bytes": nbytes,
                         "tensors": {k: list(v.shape) for k, v in loaded.items()},
                         "roofline": {"bound": "host-to-device copy", "achieved": gbs, "peak": h2d, "unit": "GB/s",
                                      "frac": gbs / h2d,
                                      "peak_source": "pinned-host to device copy of the same bytes, this run"}}
        del loaded, host, devbuf
    finally:
        if os.path.exists(path):
            os.remove(path)
        os.rmdir(tmp)

    # (f)4 pre-quant GroupNorm (8 groups) over [8, 2048, 1024] f32: read + write
    x = torch.randn((8, 2048, 1024), device=dev)
    ms = _event_ms(lambda: quantizer.group_norm(x, 8), reps, flush)
    gbs = 2 * x.numel() * 4 / (ms * 1e-3) / 1e9
    out["group_norm"] = {"value": gbs, "unit": "GB/s", "ms": ms, "shape": list(x.shape),
                         "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}}
    # one level-0 cascade stage at the tokenizer width: x [8, 2048, 1024] bf16
    xb = rnd((8, 2048, 1024))
    wd, wu = rnd((1024, 1024, 4), 0.02), rnd((1024, 1024, 4), 0.02)
    for name, fn in (("conv_down4", lambda: quantizer.conv_down4(xb, wd)),
                     ("conv_up4", lambda: quantizer.conv_up4(xb, wu))):
        f = 2.0 * 8 * 2048 * 1024 * 4096 / (4 if name == "conv_down4" else 1)
        ms = _event_ms(fn, reps, flush)
        ach = f / (ms * 1e-3) / 1e12
        out[name] = {"value": ach, "unit": "TFLOP/s", "ms": ms,
                     "roofline": {"bound": "tensor", "achieved": ach, "peak": tensor, "unit": "TFLOP/s",
                                  "frac": ach / tensor}}
    # codebook EMA of one level at scale 5 of the tokenizer: N = 16384 rows, D = 1024, K = 4096
    N, D, K = 16384, 1024, 4096
    u = torch.randn((N, D), device=dev)
    codes = torch.randint(0, K, (N,), dtype=torch.int32, device=dev)
    ema = quantizer.CodebookEMA(torch.randn((K, D), device=dev))
    ms = _event_ms(lambda: ema.stats(u, codes), reps, flush)
    byt = N * D * 4 + K * D * 4 + N * 4 * 4  # rows read once, sums written, codes/order passes
    gbs = byt / (ms * 1e-3) / 1e9
    out["ema_code_stats"] = {"value": gbs, "unit": "GB/s", "ms": ms,
                             "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                          "frac": gbs / hbm}}
    cbb = torch.empty((K, D), dtype=torch.bfloat16, device=dev)
    ms = _event_ms(lambda: ema.update(u, codes, codebook_bf16=cbb), reps, flush)
    out["ema_stats_and_update"] = {"value": ms, "unit": "ms"}

    # BASELINE config 1, the small RVQ encode: x [4096, 256], 4 levels x K = 1024.
    # Launch- and latency-bound; reported against both rooflines, eager and as
    # one CUDA-graph replay, with L2 flushed before every call.
    N, D, K, L = 4096, 256, 1024, 4
    x1 = rnd((N, D))
    decay = torch.tensor([0.5 ** l for l in range(L)], device=dev).view(L, 1, 1)
    cb1 = (rnd((L, K, D)).float() * decay).to(torch.bfloat16)
    sq1 = vq.code_sqnorm(cb1)
    codes1 = torch.empty((L, N), dtype=torch.int32, device=dev)
    recon1 = torch.empty((N, D), dtype=torch.bfloat16, device=dev)
    enc = lambda: vq.rvq_encode(x1, cb1, sq1, codes=codes1, recon=recon1)  # noqa: E731
    flops = 2.0 * L * N * K * D
    # x read, per level the f32 residual read + written, codes written and the
    # codebook read, then the bf16 reconstruction written
    byt = N * D * 2 + L * (N * D * 8 + N * 4 + K * D * 2) + N * D * 2
    for name, fn in (("rvq_small_eager", enc), ("rvq_small_graph", _graphed(enc, True))):
        for _ in range(3):
            fn()
        ms = _event_ms(fn, reps, flush)
        tf = flops / (ms * 1e-3) / 1e12
        gbs = byt / (ms * 1e-3) / 1e9
        out[name] = {"value": N / (ms * 1e-3), "unit": "vectors/s", "ms": ms, "shape": [N, D, K, L],
                     "tensor": {"achieved": tf, "peak": tensor, "unit": "TFLOP/s", "frac": tf / tensor},
                     "hbm": {"achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}}
    return {"metric": "tied_head_logits_tflops", "value": out["tied_head_logits"]["value"], "unit": "TFLOP/s",
            "config": {"workload": "next-row pieces: tied head, device loader, GroupNorm, level-0 convs, EMA; "
                                   "small RVQ encode (BASELINE config 1)"},
            "results": out, "roofline": out["tied_head_logits"]["roofline"],
            "gpu_launches": None}


def _graphed(fn, enabled):
    """Returns fn itself, or a replay of one CUDA-graph capture of fn (after a
    warm-up call, the library's calls allocate nothing and do no host sync)."""
    import torch
    if not enabled:
        return fn
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g.replay


def _profile(lib, ctx, names):
    import ctypes
    out = {}
    for n in names:
        t = ctypes.c_double()
        c = ctypes.c_int64()
        lib.ncm_profile_read(ctx, n.encode(), ctypes.byref(t), ctypes.byref(c))
        out[n] = (t.value, c.value)
    return out


def _tokenizer_setup(a, dev, rnd, g):
    """BASELINE config 2 inputs and weights (synthetic, seeded)."""
    import torch

    from ncmorph_b200 import vq
    B, T, Din, D, K, L = 8, 2048, 2048, 1024, 4096, 8
    factors = [16, 8, 4, 2, 1]
    S = len(factors)
    x = rnd((B, T, Din))
    w_in, w_out = rnd((D, Din), 0.02), rnd((Din, D), 0.02)
    decay = torch.tensor([0.6 ** l for l in range(L)], device=dev).view(1, L, 1, 1)
    cbs = (rnd((S, L, K, D)).float() * decay).to(torch.bfloat16)
    sq = vq.code_sqnorm(cbs)
    pw = pb = None
    if a.phi:
        bound = 1.0 / (3 * D) ** 0.5
        pw = ((torch.rand((S, D, D, 3), generator=g, device=dev) * 2 - 1) * bound).to(torch.bfloat16)
        pb = (torch.rand((S, D), generator=g, device=dev) * 2 - 1) * bound
    return dict(B=B, T=T, Din=Din, D=D, K=K, L=L, factors=factors, x=x, w_in=w_in, w_out=w_out, cbs=cbs, sq=sq,
                pw=pw, pb=pb)


def measure_tokenizer(a, dev, lib, ctx, rnd, g, peaks, peak_kind, steps, warmup, graph):
    """Config 2 (multiscale tokenizer forward): vectors/s, device-resident
    (eager, or one CUDA-graph replay per step with graph=True) and end to end
    from pinned host memory; per-kernel device time from the library's events."""
    import torch

    from ncmorph_b200 import vq
    c = _tokenizer_setup(a, dev, rnd, g)
    B, T, Din, D, K, L, factors = c["B"], c["T"], c["Din"], c["D"], c["K"], c["L"], c["factors"]
    S = len(factors)
    tok = dict(sqnorms=c["sq"], upsample=a.upsample, phi_weight=c["pw"], phi_bias=c["pb"], phi_ratio=0.5)
    x, w_in, cbs, w_out = c["x"], c["w_in"], c["cbs"], c["w_out"]
    step = lambda: vq.tokenizer_forward(x, w_in, cbs, w_out, factors, **tok)  # noqa: E731
    _timed_loop(step, 0, warmup)
    lib.ncm_profile_read(ctx, b"*", None, None)
    lib.ncm_profile_enable(ctx, 1)
    _timed_loop(step, steps, 0)      # per-kernel breakdown (eager launches)
    lib.ncm_profile_enable(ctx, 0)
    run = _graphed(step, graph)
    _timed_loop(run, 0, warmup)
    sampler = ClockSampler(dev.index or 0)
    sampler.start()
    ms = _timed_loop(run, steps, 0)
    clocks = sampler.stop()
    prof = _profile(lib, ctx, ["rvq_argmin", "linear_bf16", "rvq_apply", "pool_avg", "scale_update", "cast",
                               "conv_k3", "upsample", "*"])
    rows = sum(B * T // f for f in factors)
    dist_flops = 2.0 * rows * K * D * L
    proj_flops = 2 * 2.0 * B * T * Din * D
    am_ms, am_n = prof["rvq_argmin"]
    ln_ms, _ = prof["linear_bf16"]
    x_host = torch.empty_like(x, device="cpu").pin_memory()
    x_host.copy_(x.cpu())
    codes_host = torch.empty(L * rows, dtype=torch.int32).pin_memory()
    ms_e2e = _tokenizer_e2e(x, x_host, codes_host, lambda xb: vq.tokenizer_forward(xb, w_in, cbs, w_out, factors,
                                                                                   **tok)[0], steps)
    achieved = dist_flops / (am_ms / steps * 1e-3) / 1e12
    return {
        "metric": "tokenizer_vectors_per_s", "value": B * T / (ms * 1e-3), "unit": "vectors/s",
        "ms_per_step": ms, "steps": steps, "warmup": warmup, "cuda_graph": bool(graph),
        "config": {"workload": "multiscale tokenizer forward (BASELINE config 2)", "batch": B, "seq_len": T,
                   "model_width": Din, "vq_width": D, "codebook_size": K, "levels_per_scale": L,
                   "pool_factors": factors, "rows_quantised": rows, "upsample": a.upsample, "phi": bool(a.phi),
                   "l2": "inputs (64 MiB) and the f32 residual (64 MiB) are below L2; each step rewrites them"},
        "e2e": {"value": B * T / (ms_e2e * 1e-3), "unit": "vectors/s", "ms_per_step": ms_e2e,
                "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": codes_host.numel() * 4,
                "path": "vq.tokenizer_forward; the next step's input copy runs on a second stream"},
        "roofline": {"bound": "tensor", "kernel": f"rvq_argmin_kernel (all {S * L} levels)", "achieved": achieved,
                     "peak": float(peaks["bf16_tflops"]), "unit": "TFLOP/s",
                     "frac": achieved / float(peaks["bf16_tflops"]),
                     "peak_source": f"{peak_kind} bf16_tflops (burst; a 2-3 ms step)",
                     "argmin_ms_per_step": am_ms / steps, "linear_ms_per_step": ln_ms / steps,
                     "linear_tflops": proj_flops / (ln_ms / steps * 1e-3) / 1e12,
                     "conv_tflops": (2.0 * B * T * 3 * D * D * S / (prof["conv_k3"][0] / steps * 1e-3) / 1e12
                                     if a.phi and prof["conv_k3"][0] > 0 else None),
                     "share_argmin": am_ms / max(sum(v[0] for v in prof.values()), 1e-9),
                     "ms_per_step_by_kernel": {k: v[0] / steps for k, v in prof.items()}},
        "gpu_launches": int(sum(v[1] for v in prof.values())), "clocks": clocks}


def cpu_tokenizer(a, threads, rows_sample=128, proj_rows=64):
    """Config 2 on the oracle port: the RVQ cost per quantised row (all 8
    levels, K = 4096, D = 1024) from `rows_sample` rows, and the two
    projections' cost per token from `proj_rows` rows (the faithful bf16
    linear), extrapolated to the whole forward (31,744 quantised rows, 16,384
    tokens through both projections). Pooling and decode are left out."""
    from oracle import pyoracle as orc
    rng = np.random.default_rng(a.seed + 5)
    D, Din, K, L, N = 1024, 2048, 4096, 8, 8 * 2048
    rows_q = sum(N // f for f in (16, 8, 4, 2, 1))
    u = orc.bf16_bits(rng.standard_normal((rows_sample, D)).astype(np.float32))
    cbs = np.stack([orc.bf16_bits((rng.standard_normal((K, D)) * 0.6 ** l).astype(np.float32)) for l in range(L)])
    t0 = time.perf_counter()
    orc.rvq_encode(u, cbs, threads=threads)
    t_rvq = (time.perf_counter() - t0) / rows_sample
    xs = orc.round_bf16(rng.standard_normal((proj_rows, Din)).astype(np.float32))
    w_in = orc.round_bf16((rng.standard_normal((D, Din)) * 0.02).astype(np.float32))
    w_out = orc.round_bf16((rng.standard_normal((Din, D)) * 0.02).astype(np.float32))
    t0 = time.perf_counter()
    h = orc.matmul_bf16(xs, w_in, threads=threads)
    orc.matmul_bf16(orc.round_bf16(h), w_out, threads=threads)
    t_proj = (time.perf_counter() - t0) / proj_rows
    total = rows_q * t_rvq + N * t_proj
    return {"value": N / total, "unit": "vectors/s", "cores": threads, "kind": "port",
            "sample": (f"extrapolated: {rows_sample} quantised rows x {L} levels (K={K}, D={D}) and {proj_rows} tokens "
                       f"through both projections, scaled to {rows_q} quantised rows and {N} tokens")}


def measure_linear(a, dev, rnd, peaks, peak_kind, steps, warmup):
    """Config 3: the 25 Llama-3.2-1B shapes, median CUDA-event time per shape
    with L2 cleaned between calls."""
    import torch

    from ncmorph_b200 import kernels
    Ms = [1, 64, 512, 4096, 8192]
    KNs = [(2048, 2048), (2048, 512), (2048, 8192), (8192, 2048), (2048, 128256)]
    rows, tot_flops, tot_ms = [], 0.0, 0.0
    flush = _l2_flusher(dev)  # > L2: read between timed calls
    sampler = ClockSampler(dev.index or 0)
    sampler.start()
    for M in Ms:
        for (K, N) in KNs:
            xx, ww = rnd((M, K)), rnd((N, K), 0.02)
            yy = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            for _ in range(warmup):
                kernels.linear_bf16(xx, ww, out=yy)
            t = _event_ms(lambda: kernels.linear_bf16(xx, ww, out=yy), steps, flush)
            fl = 2.0 * M * N * K
            by = 2.0 * (M * K + N * K + M * N)
            tot_flops += fl
            tot_ms += t
            ai = fl / by
            roof = min(float(peaks["bf16_tflops"]) * 1e12, float(peaks["hbm_gbs"]) * 1e9 * ai)
            rows.append({"M": M, "K": K, "N": N, "us": t * 1e3, "tflops": fl / (t * 1e-3) / 1e12,
                         "gbs": by / (t * 1e-3) / 1e9, "frac_of_roofline": fl / (t * 1e-3) / roof})
            del xx, ww, yy
    clocks = sampler.stop()
    worst = min(rows, key=lambda r: r["frac_of_roofline"])
    return {
        "metric": "linear_sweep_tflops", "value": tot_flops / (tot_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
        "ms_per_step": tot_ms, "steps": steps, "warmup": warmup,
        "config": {"workload": "bf16 linear sweep, Llama-3.2-1B shapes (BASELINE config 3)",
                   "l2": "256 MiB buffer read between timed calls (L2 cold and clean)", "shapes": rows},
        "worst_shape": worst,
        "roofline": {"bound": "min(tensor, hbm x intensity) per shape",
                     "peak_source": f"{peak_kind} bf16_tflops / hbm_gbs",
                     "worst_frac": worst["frac_of_roofline"]},
        "clocks": clocks}


def cpu_linear(threads, flops_per_shape=1e9, max_outputs=4096):
    """Config 3 on the oracle port's faithful bf16 linear (matmul_bf16_impl's
    pair order, FTZ and K blocks). Its cost per output element depends only
    on K, so per (K, N) it is timed on a block of up to `max_outputs` outputs
    and about `flops_per_shape` FLOPs, and extrapolated to every M x N of the
    sweep; aggregate TFLOP/s over the 25 shapes."""
    from oracle import pyoracle as orc
    rng = np.random.default_rng(3)
    Ms = [1, 64, 512, 4096, 8192]
    KNs = [(2048, 2048), (2048, 512), (2048, 8192), (8192, 2048), (2048, 128256)]
    tot_flops = tot_sec = 0.0
    for (K, N) in KNs:
        n_sub = min(N, max_outputs)
        w = orc.round_bf16((rng.standard_normal((n_sub, K)) * 0.02).astype(np.float32))
        m = max(1, min(8192, int(flops_per_shape // (2.0 * K * n_sub))))
        xs = orc.round_bf16(rng.standard_normal((m, K)).astype(np.float32))
        t0 = time.perf_counter()
        orc.matmul_bf16(xs, w, threads=threads)
        per_elem = (time.perf_counter() - t0) / (m * n_sub)
        for M in Ms:
            tot_flops += 2.0 * M * N * K
            tot_sec += per_elem * M * N
    return {"value": tot_flops / tot_sec / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": (f"extrapolated: per (K, N) the time per output element on a block of up to {max_outputs} "
                       f"outputs and about {flops_per_shape / 1e9:g} GFLOP, scaled to the 25 shapes")}


def _decoder_setup(dev, rnd, g):
    import torch

    from ncmorph_b200 import ncm_model
    cfg = ncm_model.Config(hidden_size=2048, vq_width=1024, num_attention_heads=32, num_key_value_heads=8,
                           intermediate_size=8192, level_lengths=(256, 256, 512, 1024, 2048),
                           mask="block_causal")
    Hd, F = cfg.hidden_size, cfg.intermediate_size
    layers = [ncm_model.LayerWeights(ln_1=rnd((Hd,), 0.0) + 1, qkv=rnd((3072, Hd), 0.02), o=rnd((Hd, 2048), 0.02),
                                     ln_2=rnd((Hd,), 0.0) + 1, gate_up=rnd((2 * F, Hd), 0.02),
                                     down=rnd((Hd, F), 0.02)) for _ in range(16)]
    w = ncm_model.Weights(input_projection=rnd((Hd, cfg.vq_width), 0.02), input_projection_bias=rnd((Hd,), 0.02),
                          level_embedding=rnd((5, Hd), 0.02), final_norm=rnd((Hd,), 0.0) + 1, layers=layers)
    table = rnd((4096, cfg.vq_width))
    codes = torch.randint(0, 4096, (cfg.seq_len,), generator=g, device=dev, dtype=torch.int32)
    return cfg, w, table, codes


def measure_decoder(a, dev, lib, ctx, rnd, g, peaks, peak_kind, steps, warmup, graph):
    """Config 4 (16-layer NCM decoder forward, 4096 positions, block-causal):
    tokens/s device-resident (eager or one graph replay per step) and end to
    end (code ids in from pinned memory, hidden states back)."""
    import torch

    from ncmorph_b200 import ncm_model
    cfg, w, table, codes = _decoder_setup(dev, rnd, g)
    Hd, F = cfg.hidden_size, cfg.intermediate_size
    out = torch.empty((cfg.seq_len, Hd), dtype=torch.bfloat16, device=dev)

    def step():
        inputs = ncm_model.embedding_gather(table, codes)
        ncm_model.forward(cfg, w, inputs, out=out)

    _timed_loop(step, 0, warmup)
    lib.ncm_profile_read(ctx, b"*", None, None)
    lib.ncm_profile_enable(ctx, 1)
    _timed_loop(step, steps, 0)      # per-kernel breakdown (eager launches)
    lib.ncm_profile_enable(ctx, 0)
    run = _graphed(step, graph)
    _timed_loop(run, 0, warmup)
    sampler = ClockSampler(dev.index or 0)
    sampler.start()
    ms = _timed_loop(run, steps, 0)
    clocks = sampler.stop()
    prof = _profile(lib, ctx, ["linear_bf16", "attention", "*"])
    T = cfg.seq_len
    lin_flops = 16 * 2.0 * T * Hd * (3072 + 2048 + 3 * F) + 2.0 * T * cfg.vq_width * Hd
    lv = list(cfg.level_lengths)
    allowed = sum(n * sum(lv[: i + 1]) for i, n in enumerate(lv))
    att_flops = 16 * 4.0 * allowed * 32 * 64
    ln_ms, ln_n = prof["linear_bf16"]
    at_ms, at_n = prof["attention"]
    codes_host = codes.cpu().pin_memory()
    out_host = torch.empty((T, Hd), dtype=torch.bfloat16).pin_memory()

    def step_e2e():
        codes.copy_(codes_host, non_blocking=True)
        step()
        out_host.copy_(out, non_blocking=True)

    ms_e2e = _timed_loop(step_e2e, steps, 1)
    lin_ach = lin_flops / (ln_ms / steps * 1e-3) / 1e12
    return {
        "metric": "decoder_tokens_per_s", "value": T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
        "steps": steps, "warmup": warmup, "cuda_graph": bool(graph),
        "config": {"workload": "NCM decoder forward (BASELINE config 4)", "layers": 16, "d_model": Hd,
                   "heads": 32, "kv_heads": 8, "head_dim": 64, "ffn": F, "positions": T,
                   "levels": lv, "mask": "block_causal", "flops_linear": lin_flops, "flops_attention": att_flops,
                   "l2": "weights (1.9 GB) exceed L2 and stream every step"},
        "e2e": {"value": T / (ms_e2e * 1e-3), "unit": "tokens/s", "ms_per_step": ms_e2e,
                "h2d_bytes_per_step": T * 4, "d2h_bytes_per_step": T * Hd * 2},
        "roofline": {"bound": "tensor", "kernel": "linear_bf16_kernel", "achieved": lin_ach,
                     "peak": float(peaks["bf16_tflops"]), "unit": "TFLOP/s",
                     "frac": lin_ach / float(peaks["bf16_tflops"]), "peak_source": f"{peak_kind} bf16_tflops",
                     "linear_ms_per_step": ln_ms / steps, "attention_ms_per_step": at_ms / steps,
                     "attention_tflops": att_flops / (at_ms / steps * 1e-3) / 1e12,
                     "other_ms_per_step": prof["*"][0] / steps},
        "gpu_launches": int(ln_n + at_n + prof["*"][1]), "clocks": clocks}


def cpu_decoder(a, threads, rows_sample=32):
    """Config 4 on the oracle port: one layer's per-row work (its QKV, O,
    gate/up and down projections on the faithful bf16 linear, RMSNorms, and
    attention_impl's per-row core against all 4096 keys of the block-causal
    mask) on `rows_sample` random rows, plus the input projection, scaled to
    4096 rows x 16 layers. Each row's K/V projection is inside its QKV
    projection, so the other rows' keys and values are random stand-ins."""
    from oracle import pyoracle as orc
    rng = np.random.default_rng(a.seed + 11)
    T, Hd, V, H, Hkv, F, hd, eps = 4096, 2048, 1024, 32, 8, 8192, 64, 1e-5
    levels = [256, 256, 512, 1024, 2048]
    rb = orc.round_bf16

    def wt(o, i):
        return rb((rng.standard_normal((o, i)) * 0.02).astype(np.float32))

    w_in, qkv, wo, gu, wd = wt(Hd, V), wt((H + 2 * Hkv) * hd, Hd), wt(Hd, H * hd), wt(2 * F, Hd), wt(Hd, F)
    ln = np.ones(Hd, np.float32)
    n_all = rb(rng.standard_normal((T, Hd)).astype(np.float32))
    rows = np.sort(rng.choice(T, size=rows_sample, replace=False))
    pos = np.asarray(orc.fill_level_positions(0, levels), np.int64)
    _, c, s = orc.rope_default(hd, 500000.0, int(pos.max()) + 1)
    cos, sin = c[pos], s[pos]
    mask = orc.block_causal_mask(0, levels).astype(np.uint8)
    # K and V of every row: their projection is each row's share of its timed
    # QKV projection below, so random bf16 values stand in for them here
    k = rb(rng.standard_normal((T, Hkv * hd)).astype(np.float32))
    v = rb(rng.standard_normal((T, Hkv * hd)).astype(np.float32))
    xin = rb(rng.standard_normal((rows_sample, V)).astype(np.float32))
    t0 = time.perf_counter()
    orc.matmul_bf16(xin, w_in, threads=threads)
    t_in = time.perf_counter() - t0
    t0 = time.perf_counter()
    hs = n_all[rows]
    n1 = np.stack([orc.rms_norm(hs[i], ln, eps, bf16_mode=True) for i in range(rows_sample)])
    q = orc.matmul_bf16(n1, qkv, threads=threads)[:, : H * hd].copy()
    orc.lib().orc_rotate_rows(q, rows_sample, H, hd, np.ascontiguousarray(cos[rows]),
                              np.ascontiguousarray(sin[rows]), 1)
    ctx = np.empty((rows_sample, H * hd), np.float32)
    orc.lib().orc_attention_core_rows(q, k, v, np.ascontiguousarray(mask[rows]), rows_sample, T, H, Hkv, hd, ctx, 1,
                                      threads)
    h2 = rb(hs + orc.matmul_bf16(ctx, wo, threads=threads))
    n2 = np.stack([orc.rms_norm(h2[i], ln, eps, bf16_mode=True) for i in range(rows_sample)])
    g_u = orc.matmul_bf16(n2, gu, threads=threads)
    act = rb(orc.silu_bf16(g_u[:, :F]) * g_u[:, F:])
    rb(h2 + orc.matmul_bf16(act, wd, threads=threads))
    t_layer = time.perf_counter() - t0
    per_row = (16 * t_layer + t_in) / rows_sample
    return {"value": 1.0 / per_row, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": (f"extrapolated: one layer's per-row work on {rows_sample} random rows of 4096 (block-causal "
                       f"attention against their allowed keys) plus the input projection, scaled to 4096 rows x 16 "
                       f"layers")}


def run_extras(a, dev):
    """Configs 2-4 on the headline line (N = 1): each with its device and end-
    to-end numbers, clocks, and a CPU baseline from the oracle port."""
    import torch

    from ncmorph_b200 import _lib, device as ndev
    lib = _lib.load()
    ctx = ndev.context(dev)
    peaks, peak_kind = measured_peaks()
    g = torch.Generator(device=dev).manual_seed(a.seed + 3)

    def rnd(shape, scale=1.0):
        return (torch.randn(shape, generator=g, device=dev) * scale).to(torch.bfloat16)

    steps, warmup = max(5, min(a.steps, 20)), max(3, a.warmup)
    threads = os.cpu_count() or 1
    out = {}
    out["tokenizer"] = measure_tokenizer(a, dev, lib, ctx, rnd, g, peaks, peak_kind, steps, warmup, graph=True)
    out["tokenizer"]["cpu_baseline"] = cpu_tokenizer(a, threads)
    torch.cuda.empty_cache()
    out["decoder"] = measure_decoder(a, dev, lib, ctx, rnd, g, peaks, peak_kind, steps, warmup, graph=True)
    out["decoder"]["cpu_baseline"] = cpu_decoder(a, threads)
    torch.cuda.empty_cache()
    out["linear_sweep"] = measure_linear(a, dev, rnd, peaks, peak_kind, steps, warmup)
    out["linear_sweep"]["cpu_baseline"] = cpu_linear(threads)
    ndev.sync(dev)
    return out


def run_tokenizer_sharded(a):
    """Config 2 on N GPUs (torchrun): ShardedTokenizer with 8 batch items per
    GPU (weak scaling; weights and codebooks identical on every rank, each
    rank's items from its own seed). A step is the whole sharded forward,
    the all-gather of the codes included; timed with CUDA events between
    barriers, max over ranks."""
    import datetime

    import torch
    import torch.distributed as dist

    from ncmorph_b200 import sharded, vq

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    try:
        g = torch.Generator(device=dev).manual_seed(a.seed)

        def rnd(shape, scale=1.0):
            return (torch.randn(shape, generator=g, device=dev) * scale).to(torch.bfloat16)

        c = _tokenizer_setup(a, dev, rnd, g)
        B, T = c["B"], c["T"]
        gx = torch.Generator(device=dev).manual_seed(a.seed + 1000 + rank)
        x = torch.randn((B, T, c["Din"]), generator=gx, device=dev).to(torch.bfloat16)
        kw = dict(sqnorms=c["sq"], upsample=a.upsample, phi_weight=c["pw"], phi_bias=c["pb"], phi_ratio=0.5)
        # each rank's forward is one CUDA-graph replay on its fixed buffers, as
        # on the default line: an eager forward is about 85 launches, and a
        # rank whose host issued them slower than its GPU ran them set the
        # pace (measured: 1.5 and 3.5 ms of host time per step on two ranks
        # of one box); the code gathers stay eager
        out = {}

        def forward(xb, w_in, cbs, w_out, pf, **k):
            if "run" not in out:
                def once():
                    out["res"] = vq.tokenizer_forward(xb, w_in, cbs, w_out, pf, **k)
                out["run"] = _graphed(once, True)
            out["run"]()
            return out["res"]

        tok = sharded.ShardedTokenizer(B * world, T, c["factors"], forward=forward)

        def step():
            return tok(x, c["w_in"], c["cbs"], c["w_out"], **kw)

        for _ in range(a.warmup):
            step()
        sampler = ClockSampler(local)
        dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)
        sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(a.steps):
            step()
        e1.record()
        host_ms = (time.perf_counter() - t0) * 1e3 / a.steps  # host time to issue a step
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[local])
        clocks = sampler.stop()
        mine = torch.tensor([e0.elapsed_time(e1) / a.steps, host_ms, float(clocks.get("sm_mhz") or 0)], device=dev)
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        per_rank = [[round(float(v), 3) for v in t.tolist()] for t in every]
        ms = max(r[0] for r in per_rank)
        if rank == 0:
            emit({"metric": "tokenizer_vectors_per_s", "value": B * world * T / (ms * 1e-3), "unit": "vectors/s",
                  "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
                  "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                  "dtype": "bf16 operands, f32 accumulation", "data": "synthetic",
                  "config": {"workload": "multiscale tokenizer forward (BASELINE config 2), batch-sharded",
                             "batch_per_gpu": B, "global_batch": B * world, "seq_len": T,
                             "pool_factors": c["factors"], "parallelism": f"batch items x{world}",
                             "cuda_graph": True,
                             "collective": "NCCL all_gather of the codes of every scale (reconstructions and "
                                           "outputs stay with the rank that owns the batch items)"},
                  "e2e": None, "clocks": clocks,
                  "per_rank_ms_device_host_mhz": per_rank})
    finally:
        dist.destroy_process_group()
    return 0


def run_secondary(a):
    import torch

    from ncmorph_b200 import _lib, device as ndev

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    ctx = ndev.context(dev)
    peaks, peak_kind = measured_peaks()
    g = torch.Generator(device=dev).manual_seed(a.seed)

    def rnd(shape, scale=1.0):
        return (torch.randn(shape, generator=g, device=dev) * scale).to(torch.bfloat16)

    line = {"n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "higher_is_better": True, "scaling": "none",
            "vs_baseline": None, "dtype": "bf16 operands, f32 accumulation", "data": "synthetic"}
    threads = os.cpu_count() or 1
    if a.workload == "tokenizer":
        line.update(measure_tokenizer(a, dev, lib, ctx, rnd, g, peaks, peak_kind, a.steps, a.warmup, a.graph))
        line["cpu_baseline"] = cpu_tokenizer(a, threads)
    elif a.workload == "linear":
        line.update(measure_linear(a, dev, rnd, peaks, peak_kind, a.steps, a.warmup))
        line["cpu_baseline"] = cpu_linear(threads)
    elif a.workload == "aux":
        line.update(_aux_suite(a, dev, rnd, peaks, peak_kind))
    else:  # decoder
        line.update(measure_decoder(a, dev, lib, ctx, rnd, g, peaks, peak_kind, a.steps, a.warmup, a.graph))
        line["cpu_baseline"] = cpu_decoder(a, threads)
    ndev.sync(dev)
    emit(line)
    return 0


def main():
    _claim_stdout()
    a = parse_args()
    if a.workload == "tokenizer" and int(os.environ.get("WORLD_SIZE", "1")) > 1 and a.impl != "reference":
        return run_tokenizer_sharded(a)
    if a.workload != "rvq":
        return run_secondary(a)
    if a.impl == "reference":
        return run_reference(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())
