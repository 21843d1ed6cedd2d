"""Benchmark of the VibeKernel GEMM hot path on B200 (one JSON line on rank 0).

One GPU (default): the reference's scoring rubric: C = A*B, M=N=K=4096, fp16
A/B uniform[-1,1) seed 1, fp32 accumulation, fp16 C; 10 warm-up calls then the average of 100 timed
calls, each bracketed by CUDA events and followed by an event synchronize exactly like the reference
driver (results/naive_cycle6/src/main.cpp:52-62).  L2 is flushed (a 256 MiB write, outside the event
pair) before every timed call because the rubric's operands (96 MiB) fit in the 126 MB L2.  The same
run also times BASELINE configs[2] (fp16 accumulation), [3] (fp32 SGEMM) and [4b] (ragged) and reports
them under "workloads".

N GPUs (torchrun, one process per GPU): BASELINE configs[4a], 16384^3 fp16 (seed 4), M split into N
row blocks, B replicated, and C all-gathered on every rank -- by default through NVLink SHARP (each
GPU's GEMM epilogue stores every finished box once to the multicast view of C; NCCL after the GEMM
where the switch has no multicast).  Strong scaling; B alone (512 MiB) exceeds L2, so no flush.

Every timed output is checked against the golden rows of the reference v0 (tests/golden), and the
run fails on a mismatch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload rubric|f16acc|sgemm|ragged|shard16k]
                  [--allgather auto|none|nccl|pipelined|fused|nvls]
  python bench.py --impl reference ...   # the reference's own CPU v0 (oracle/_ref) on host cores
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (M, N, K, seed, dist, lo, hi, dtype, acc, label, golden fixture)
    "rubric": (4096, 4096, 4096, 1, "uniform", -1.0, 1.0, "f16", "f32",
               "gemm_f16_f32acc_4096^3 (BASELINE configs[1], scoring rubric)", "cfg1_4096_seed1"),
    "f16acc": (4096, 4096, 4096, 2, "uniform", -0.5, 0.5, "f16", "f16",
               "gemm_f16_f16acc_4096^3 (BASELINE configs[2])", "cfg2_4096_seed2"),
    "sgemm": (4096, 4096, 4096, 3, "normal", 0.0, 0.0, "f32", "f32",
              "sgemm_ffma_4096^3 (BASELINE configs[3])", "cfg3_sgemm_4096_seed3"),
    "ragged": (4000, 5120, 3000, 5, "uniform", -1.0, 1.0, "f16", "f32",
               "gemm_f16_f32acc_4000x5120x3000 (BASELINE configs[4b])", "cfg5_ragged_4000x5120x3000_seed5"),
    "shard16k": (16384, 16384, 16384, 4, "uniform", -1.0, 1.0, "f16", "f32",
                 "gemm_f16_f32acc_16384^3 row-sharded, C all-gathered (BASELINE configs[4a])", "cfg4a_16384_seed4"),
}
EXTRA_WORKLOADS = ("f16acc", "sgemm", "ragged")  # timed beside the rubric on one GPU

FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant kernel, from
# the ncu captures summarised under profiles/; None where no capture of the current kernel exists.
TRAFFIC = {"rubric": 136087296, "ragged": 116693248, "sgemm": 568920064}

METRIC = "sustained TFLOPS @4096^3 fp16 (10 warmup+100 iter avg), % of B200 tensor peak"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------------------------------
# Clock sampling during the timed region (NVML; same fields as the nvidia-smi clocks query)
# ------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int, interval_s: float = 0.002):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._interval = interval_s
        self._handle = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[device_index]) if vis and vis.split(",")[0].isdigit() else device_index
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable, never faked
            self._handle = None
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self._interval)

    def __enter__(self):
        if self._handle is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._handle is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------
# Output check against the golden rows of the reference v0 (tests/golden, made by oracle/_ref)
# ------------------------------------------------------------------------------------------
def check_rows(C_host_rows: np.ndarray, gold: np.ndarray, acc: str, dt: str) -> dict:
    """Parity of sampled rows with the tolerances of the parity tests: fp32-acc fp16 output, per
    element |C - G| / max(|G|, 1e-2 RMS(G)) <= 2e-3 (G and C both rounded to fp16); fp16-acc, relative
    Frobenius <= 5e-3; fp32 SGEMM, relative Frobenius <= 1e-5."""
    c = C_host_rows.astype(np.float64)
    g = gold.astype(np.float64)
    den = np.linalg.norm(g)
    frob = float(np.linalg.norm(c - g) / den) if den > 0 else float(np.linalg.norm(c))
    tau = 1e-2 * float(np.sqrt(np.mean(g * g))) if g.size else 0.0
    elem = float(np.max(np.abs(c - g) / np.maximum(np.abs(g), max(tau, 1e-300)))) if g.size else 0.0
    if dt == "f32":
        ok, rule = frob <= 1e-5, "rel_frobenius <= 1e-5"
    elif C_host_rows.shape[1] >= 16384:
        # K = 16384 (configs[4a]): the tensor cores' truncating fp32 accumulation exceeds the per-element
        # bound near zero; the fp16 output's relative Frobenius error is checked instead
        ok, rule = frob <= 1e-3 and elem <= 1e-2, "rel_frobenius <= 1e-3 and max_elem_rel <= 1e-2"
    elif acc == "f16":
        ok, rule = frob <= 5e-3, "rel_frobenius <= 5e-3"
    else:
        ok, rule = elem <= 2e-3, "max_elem_rel <= 2e-3"
    return {"ok": bool(ok and np.isfinite(c).all()), "rows": int(gold.shape[0]), "rel_frobenius": frob,
            "max_elem_rel": elem, "rule": rule}


def golden(name: str):
    z = np.load(os.path.join(ROOT, "tests", "golden", name + ".npz"))
    return z["rows"], z["C"]


# ------------------------------------------------------------------------------------------
# CPU arms: the reference's own v0 (oracle/_ref), bounded samples on the host cores
# ------------------------------------------------------------------------------------------
def cpu_v0_sample(A, B, dtype: str, budget_s: float, threads: int | None = None):
    """Times the reference v0 on a row slice of A sized to ~budget_s with `threads` OpenBLAS threads;
    returns (tflops, rows, secs)."""
    from oracle import v0
    if v0.ref_available():
        fn = v0.ref_v0_f16 if dtype == "f16" else v0.ref_v0_f32
        if threads is not None:
            v0.set_ref_threads(threads)
    else:
        fn = (lambda a, b: v0.v0_f16(a, b)[0]) if dtype == "f16" else v0.v0_f32
    n, k = B.shape[1], B.shape[0]
    rows = min(64, A.shape[0])
    t0 = time.perf_counter()
    fn(A[:rows], B)
    dt = time.perf_counter() - t0
    rows = int(min(A.shape[0], max(rows, rows * budget_s / max(dt, 1e-6))))
    rows = max(1, rows)
    t0 = time.perf_counter()
    fn(A[:rows], B)
    dt = time.perf_counter() - t0
    return 2.0 * rows * n * k / dt / 1e12, rows, dt


def run_reference(args, cfg):
    """--impl reference: the reference's CPU v0 on this box's host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import v0

    from vibekernel_b200 import testdata
    threads = os.cpu_count() or 1
    m, n, k, seed, dist, lo, hi, dt, acc, label, _ = cfg
    npdt = np.float16 if dt == "f16" else np.float32
    A, B = testdata.make_inputs(m, n, k, seed, dist, lo, hi, npdt, a_rows=(0, min(m, 4096)))
    kind = "reference" if v0.ref_available() else "port"
    if v0.ref_available():
        v0.set_ref_threads(threads)
    fn = (v0.ref_v0_f16 if dt == "f16" else v0.ref_v0_f32) if v0.ref_available() else \
        ((lambda a, b: v0.v0_f16(a, b)[0]) if dt == "f16" else v0.v0_f32)
    # Calibrate once: every step is one v0 call on a row slice of A sized so that warm-up + steps
    # finish in about two minutes (the full matrix when that fits).
    per_step = max(0.05, 120.0 / max(1, args.steps + args.warmup))
    _, rows_used, _ = cpu_v0_sample(A, B, dt, per_step)
    tfl = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        fn(A[:rows_used], B)
        dt_s = time.perf_counter() - t0
        if i >= args.warmup:
            tfl.append(2.0 * rows_used * n * k / dt_s / 1e12)
    value = statistics.mean(tfl)
    flops_full = 2.0 * m * n * k
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(flops_full / (value * 1e12) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if args.workload == "shard16k" else "weak", "vs_baseline": None, "dtype": dt,
        "data": "synthetic (seeded)",
        "config": {"workload": label, "m": m, "n": n, "k": k, "seed": seed},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOPS", "cores": threads, "kind": kind,
                         "cpu_model": cpu_model(),
                         "sample": f"v0 on a {rows_used}-row slice of A per step (x{n}x{k}), "
                                   f"OpenBLAS {threads} threads"},
        "e2e": {"value": round(value, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------
def time_workload(vk, torch, name, cfg, dev, stream, steps, warmup, flush, algo="auto", tile_n=0):
    """One GPU: the rubric loop (flush, events around each call, event synchronize) on `name`'s
    seeded inputs; returns (per-call ms list, C, A, B host arrays)."""
    from vibekernel_b200 import testdata
    m, n, k, seed, dist, lo, hi, dt, acc, label, _ = cfg
    npdt = np.float16 if dt == "f16" else np.float32
    hA, hB = testdata.make_inputs(m, n, k, seed, dist, lo, hi, npdt)
    A = torch.from_numpy(hA).to(dev)
    B = torch.from_numpy(hB).to(dev)
    C = torch.empty((m, n), dtype=A.dtype, device=dev)
    for _ in range(warmup):
        flush.fill_(1.0)
        vk.gemm(A, B, C, acc=acc, algo=algo, tile_n=tile_n, stream=stream)
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.fill_(1.0)
        ev[i][0].record(stream)
        vk.gemm(A, B, C, acc=acc, algo=algo, tile_n=tile_n, stream=stream)
        ev[i][1].record(stream)
        ev[i][1].synchronize()
    return [s.elapsed_time(e) for s, e in ev], C, hA, hB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["vk", "reference"], default="vk")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help="default: rubric on one GPU, shard16k under torchrun")
    ap.add_argument("--algo", default="auto")
    ap.add_argument("--tile-n", type=int, default=0)
    ap.add_argument("--allgather", default="auto", choices=["auto", "none", "nccl", "pipelined", "fused", "nvls"],
                    help="all-gather of C on every rank (N > 1): auto = nvls where the GPUs support NVLink "
                         "multicast, else nccl; nccl = NCCL after the GEMM; pipelined = copy-engine pushes of "
                         "finished row chunks overlapped with the GEMM; fused = the epilogue stores every box "
                         "into each peer's C; nvls = the epilogue stores every box once to the multicast view")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the extra workloads timed beside the rubric")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload is None:
        args.workload = "shard16k" if world > 1 else "rubric"
    cfg = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, cfg)
        return

    import torch
    import torch.distributed as dist

    import vibekernel_b200 as vk
    from vibekernel_b200 import dist_gemm, testdata

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)

    m_cfg, n, k, seed, distname, lo, hi, dt, acc, label, gold_name = cfg
    strong = args.workload == "shard16k"
    m_total = m_cfg if strong else m_cfg * world
    off = vk.row_blocks(m_total, world)
    rows = off[rank + 1] - off[rank]
    tdt = torch.float16 if dt == "f16" else torch.float32
    npdt = np.float16 if dt == "f16" else np.float32
    # Seeded inputs of the configuration (the golden fixtures' recipe): this rank's rows of A and all of
    # B, generated on the host and copied to the device before any timing.
    if strong:
        hA, hB = testdata.make_inputs(m_cfg, n, k, seed, distname, lo, hi, npdt, a_rows=(off[rank], off[rank + 1]))
    else:  # weak scaling (a non-default workload under torchrun): every rank the whole config
        hA, hB = testdata.make_inputs(m_cfg, n, k, seed, distname, lo, hi, npdt)
    A = torch.from_numpy(hA).to(dev)
    B = torch.from_numpy(hB).to(dev)

    mode = args.allgather if world > 1 else "none"
    if mode == "auto":
        flags = [None] * world
        dist.all_gather_object(flags, dt == "f16" and vk.mc_supported(local))
        mode = "nvls" if all(flags) else "nccl"
    gather_on = mode != "none"
    mc_gather = peer_gather = None
    if mode == "nvls":
        try:
            mc_gather = dist_gemm.McRowGather(m_total, n, off, rank, dtype=tdt)
        except dist_gemm.McSetupRefused as e:
            # a refused multicast object is reported to every rank at the same point, so all fall back
            if args.allgather != "auto":
                raise
            if rank == 0:
                print(f"warning: NVLS multicast unavailable ({e}); gathering C with NCCL", file=sys.stderr)
            mode = "nccl"
    if mc_gather is not None:
        C_full = mc_gather.C_full
    else:
        C_full = torch.empty((m_total, n), dtype=tdt, device=dev) if gather_on else None
        if mode in ("pipelined", "fused"):
            peer_gather = dist_gemm.PeerRowGather(C_full, off, rank)
    C = C_full[off[rank]:off[rank + 1]] if C_full is not None else torch.empty((rows, n), dtype=tdt, device=dev)
    # L2 (126 MB) flush between timed calls when the operands would fit in it
    in_l2 = (rows * k + k * n + rows * n) * hA.itemsize < 126e6
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev) if in_l2 else None
    stream = torch.cuda.current_stream(dev)

    def local_gemm(a, b, out, peers=None, mc=None):
        vk.gemm(a, b, out, acc=acc, algo=args.algo, tile_n=args.tile_n, stream=stream, peers=peers, mc=mc)

    launches_per_step = 1
    if mode == "pipelined":
        launches_per_step = len(dist_gemm.chunk_rows(rows, 2))

    def step():
        if mc_gather is not None:
            mc_gather.run(A, B, local_gemm)  # GEMM + every box stored once through the switch
        elif peer_gather is not None:
            peer_gather.run(A, B, local_gemm, chunks=2, mode=mode)
        else:
            local_gemm(A, B, C)
            if mode == "nccl":
                dist_gemm.allgather_rows(C_full, off, rank)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    try:
        for _ in range(args.warmup):
            if flush is not None:
                flush.fill_(1.0)
            step()
        barrier()

        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        probe = dt == "f16"  # the tensor-core kernels carry the in-kernel clock probe
        if probe:
            vk.set_option("clock_probe", 1)
            vk.read_clock_probe(local, clear=True)
        with ClockSampler(local) as clocks:
            for i in range(args.steps):
                if flush is not None:
                    flush.fill_(1.0)
                ev[i][0].record(stream)
                step()
                ev[i][1].record(stream)
                ev[i][1].synchronize()  # the reference driver synchronises every iteration
            barrier()
        kernel_mhz = None
        if probe:
            kernel_mhz, _ = vk.read_clock_probe(local, clear=True)
            vk.set_option("clock_probe", 0)
        step_ms = [s.elapsed_time(e) for s, e in ev]
        err = vk.device_error(local)
        if err:
            raise SystemExit(f"device error word {err:#x}")

        # output check: the golden rows of the reference v0 present in this rank's result
        g_rows, g_C = golden(gold_name)
        if C_full is not None:
            have = g_rows
            got = C_full[torch.from_numpy(have).to(dev)].cpu().numpy()
        else:
            sel = (g_rows >= off[rank]) & (g_rows < off[rank + 1]) if strong else np.ones(len(g_rows), bool)
            have = g_rows[sel]
            local_idx = (have - off[rank]) if strong else have
            got = C[torch.from_numpy(local_idx).to(dev)].cpu().numpy() if len(have) else np.zeros((0, n), npdt)
        chk = check_rows(got, g_C[np.isin(g_rows, have)], acc, dt)

        # compute-only steps (no exchange) for the cost of the gather, N > 1 with a gather
        compute_ms = None
        if world > 1 and gather_on:
            Cl = torch.empty((rows, n), dtype=tdt, device=dev)
            for _ in range(3):
                local_gemm(A, B, Cl)
            barrier()
            evc = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            for i in range(args.steps):
                evc[i][0].record(stream)
                local_gemm(A, B, Cl)
                evc[i][1].record(stream)
                evc[i][1].synchronize()
            barrier()
            compute_ms = sum(s.elapsed_time(e) for s, e in evc) / args.steps
            del Cl
    finally:
        if mc_gather is not None:
            mc_gather.close()  # collective: every rank detaches from the multicast buffer together
        if peer_gather is not None:
            peer_gather.close()

    total_ms = sum(step_ms)
    kernel_ms = total_ms / args.steps  # this rank's average step (one launch per step at N = 1)
    t = torch.tensor([total_ms, compute_ms or 0.0, 0.0 if chk["ok"] else 1.0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, compute_ms_max, any_bad = float(t[0]), float(t[1]), float(t[2])
    flops_step = 2.0 * m_total * n * k
    value = flops_step * args.steps / (total_ms * 1e-3) / 1e12

    # ---------------- e2e: the public host-buffer API (vk_gemm_host): every step copies this rank's A
    # rows and B in from pinned host memory and its C rows back out, pipelined with the GEMM in row
    # blocks; the call is synchronous, so host wall-clock around it covers every byte moved.
    e2e = None
    if not args.no_e2e:
        pA = torch.from_numpy(hA).pin_memory()
        pB = torch.from_numpy(hB).pin_memory()
        pC = torch.empty((rows, n), dtype=tdt).pin_memory()
        e2e_steps = max(3, min(args.steps, 20))
        for _ in range(3):
            vk.gemm_host(pA, pB, pC, acc=acc, algo=args.algo)
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            vk.gemm_host(pA, pB, pC, acc=acc, algo=args.algo)
        t_e2e = time.perf_counter() - t0
        te = torch.tensor([t_e2e], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_val = flops_step * e2e_steps / float(te[0]) / 1e12
        e2e = {"value": round(e2e_val, 3), "unit": "TFLOPS",
               "h2d_bytes_per_step": int((pA.numel() + pB.numel()) * pA.element_size() * world),
               "d2h_bytes_per_step": int(pC.numel() * pC.element_size() * world), "steps": e2e_steps,
               "api": "vk_gemm_host (pinned host A rows, B, C rows; copies pipelined with the GEMM in row blocks"
                      + ("; C stays row-sharded, no all-gather)" if world > 1 else ")"),
               "timing": "host wall clock around the synchronous call, max over ranks"}

    line = None
    if rank == 0:
        pk, pk_src = peaks()
        sm_mhz = clocks.summary()["sm_mhz"] or pk.get("sm_max_mhz", 1965.0)
        if dt == "f16":
            peak = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
            bound = "tensor"
        else:
            peak = 148 * 128 * 2 * float(sm_mhz) * 1e6 / 1e12  # FFMA peak at the sampled clock
            bound = "ffma"
        achieved = 2.0 * rows * n * k / (kernel_ms * 1e-3) / 1e12
        roof = {"bound": bound, "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": TRAFFIC.get(args.workload) if world == 1 else None,
                "traffic_unit": "bytes/launch",
                "algorithmic_bytes": int((rows * k + k * n + rows * n) * (2 if dt == "f16" else 4)),
                "peak_source": (f"MEASURED_PEAKS.json bf16_tflops (burst), of {pk_src}" if dt == "f16"
                                else "148 SMs x 128 FP32 lanes x 2 x sampled SM clock"),
                "kernel": "per-step time" + (" (GEMM + fused all-gather)" if world > 1 and gather_on else "")}
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": dt, "data": "synthetic (seeded BASELINE inputs, the golden fixtures' recipe)",
            "config": {"workload": label, "m": m_total, "n": n, "k": k, "seed": seed, "m_per_gpu": rows,
                       "acc": acc, "algo": args.algo, "tile_n": args.tile_n or 256,
                       "parallelism": f"rowshard{world}", "allgather_c": mode if gather_on else False,
                       "l2": ("flushed before every timed call (256 MiB write outside the event pair)" if in_l2
                              else "inputs larger than L2 (no flush)"),
                       "timing": "per-step CUDA events + event synchronize (reference main.cpp loop), max over ranks"},
            "roofline": roof,
            "pct_of_dense_peak_2250": round(value / world / 2250.0, 4),
            "clocks": dict(clocks.summary(), kernel_sm_mhz=(round(kernel_mhz, 1) if kernel_mhz else None)),
            "clock_true_peak_frac": (round(achieved / (148 * 8192 * kernel_mhz * 1e6 / 1e12), 4)
                                     if (kernel_mhz and dt == "f16") else None),
            "gpu_launches": args.steps * launches_per_step,
            "check": dict(chk, ok=any_bad == 0.0, golden=gold_name),
            "process_group": ({"backend": "nccl", "ranks": dist.get_world_size(),
                               "nccl_version": ".".join(str(x) for x in torch.cuda.nccl.version())}
                              if world > 1 else None),
            "e2e": e2e,
        }
        if compute_ms is not None:
            line["compute_ms_per_step"] = round(compute_ms_max, 5)
            line["gather_ms_per_step"] = round(total_ms / args.steps - compute_ms_max, 5)
            line["compute_only_tflops"] = round(flops_step / (compute_ms_max * 1e-3) / 1e12, 3)

    if world == 1 and not args.no_extra:
        # BASELINE configs[2], [3], [4b] in the same run: same loop, fewer steps, each checked
        flush1 = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
        extra = {}
        for name in EXTRA_WORKLOADS:
            wc = WORKLOADS[name]
            st = max(3, min(args.steps, 30))
            ms, Cw, _, _ = time_workload(vk, torch, name, wc, dev, stream, st, 3, flush1)
            g_rows, g_C = golden(wc[10])
            wchk = check_rows(Cw[torch.from_numpy(g_rows).to(dev)].cpu().numpy(), g_C, wc[8], wc[7])
            fl = 2.0 * wc[0] * wc[1] * wc[2]
            tf = fl * st / (sum(ms) * 1e-3) / 1e12
            if wc[7] == "f16":
                wpeak, wbound = float(peaks()[0].get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])), "tensor"
            else:
                wpeak, wbound = 148 * 128 * 2 * float(line["clocks"]["sm_mhz"] or 1965.0) * 1e6 / 1e12, "ffma"
            extra[name] = {"workload": wc[9], "value": round(tf, 3), "unit": "TFLOPS", "steps": st, "warmup": 3,
                           "ms_per_step": round(sum(ms) / st, 5), "roofline": {"bound": wbound, "peak": round(wpeak, 2),
                                                                              "frac": round(tf / wpeak, 4),
                                                                              "traffic": TRAFFIC.get(name)},
                           "check": dict(wchk, golden=wc[10])}
            any_bad = any_bad or (0.0 if wchk["ok"] else 1.0)
            del Cw
        line["workloads"] = extra
        line["gpu_launches"] += sum(v["steps"] for v in extra.values())
        line["check"]["ok"] = line["check"]["ok"] and all(v["check"]["ok"] for v in extra.values())

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import v0
        threads = os.cpu_count() or 1
        tfl, rws, secs = cpu_v0_sample(hA, hB, dt, 10.0, threads)
        tfl1, rws1, secs1 = cpu_v0_sample(hA, hB, dt, 10.0, 1) if v0.ref_available() else (None, 0, 0.0)
        if v0.ref_available():
            v0.set_ref_threads(threads)
        line["cpu_baseline"] = {
            "value": round(tfl, 4), "unit": "TFLOPS", "cores": threads,
            "kind": "reference" if v0.ref_available() else "port", "cpu_model": cpu_model(),
            "sample": f"reference v0 (oracle/_ref) on {rws} of {m_cfg} rows ({secs:.2f} s), OpenBLAS {threads} threads",
            "one_core": ({"value": round(tfl1, 5), "unit": "TFLOPS", "cores": 1,
                          "sample": f"{rws1} of {m_cfg} rows ({secs1:.2f} s), OpenBLAS 1 thread"}
                         if tfl1 is not None else None)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ok_all = line["check"]["ok"] if rank == 0 else any_bad == 0.0
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if not ok_all:
        raise SystemExit("output check against the golden rows failed")


if __name__ == "__main__":
    main()
