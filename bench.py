"""Benchmark of the VibeKernel GEMM hot path on B200 (one JSON line on rank 0).

Default workload = the reference's scoring rubric: C = A*B, M=N=K=4096,
fp16 A/B uniform[-1,1) seed 1, fp32 accumulation, fp16 C; 10 warm-up calls then the average of
100 timed calls, each bracketed by CUDA events and followed by an event synchronize exactly like
the reference driver (results/naive_cycle6/src/main.cpp:52-62).  L2 is flushed (a 256 MiB
write, outside the event pair) before every timed call because the rubric's operands (96 MiB)
fit in the 126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload rubric|f16acc|sgemm|ragged|shard16k]
  python bench.py --impl reference ...   # the reference's own CPU v0 (oracle/_ref) on host cores

Multi-GPU (torchrun, one process per GPU): every rank computes its own 4096-row block of a
(4096*N) x 4096 x 4096 GEMM with B replicated (row-block sharding, weak scaling, no exchange on
the data path); `--allgather` adds the NCCL all-gather of C after the GEMM, `--allgather pipelined`
the copy-engine gather overlapped with it (row chunks pushed into the peers' C as they finish).
`--workload shard16k` is the
16384^3 strong-scaling case (M split across ranks).
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
    # name: (M per rank, N, K, seed, dist, lo, hi, dtype, acc, label)
    "rubric": (4096, 4096, 4096, 1, "uniform", -1.0, 1.0, "f16", "f32",
               "gemm_f16_f32acc_4096^3 (BASELINE configs[1], scoring rubric)"),
    "f16acc": (4096, 4096, 4096, 2, "uniform", -0.5, 0.5, "f16", "f16",
               "gemm_f16_f16acc_4096^3 (BASELINE configs[2])"),
    "sgemm": (4096, 4096, 4096, 3, "normal", 0.0, 0.0, "f32", "f32",
              "sgemm_ffma_4096^3 (BASELINE configs[3])"),
    "ragged": (4000, 5120, 3000, 5, "uniform", -1.0, 1.0, "f16", "f32",
               "gemm_f16_f32acc_4000x5120x3000 (BASELINE configs[4b])"),
    "shard16k": (16384, 16384, 16384, 4, "uniform", -1.0, 1.0, "f16", "f32",
                 "gemm_f16_f32acc_16384^3 row-sharded (BASELINE configs[4a])"),
}

FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


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
# CPU arms: the reference's own v0 (oracle/_ref), bounded samples on the host cores
# ------------------------------------------------------------------------------------------
def cpu_v0_sample(A, B, dtype: str, budget_s: float):
    """Times the reference v0 on a row slice of A sized to ~budget_s; returns (tflops, rows, secs)."""
    from oracle import v0
    fn = v0.ref_v0_f16 if dtype == "f16" else v0.ref_v0_f32
    if not v0.ref_available():
        fn = (lambda a, b: v0.v0_f16(a, b)[0]) if dtype == "f16" else v0.v0_f32
    n, k = B.shape[1], B.shape[0]
    rows = min(256, A.shape[0])
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
    threads = os.cpu_count() or 1
    os.environ.setdefault("OPENBLAS_NUM_THREADS", str(threads))
    m, n, k, seed, dist, lo, hi, dt, acc, label = cfg
    npdt = np.float16 if dt == "f16" else np.float32
    A, B = v0.make_inputs(m, n, k, seed, dist, lo, hi, npdt)
    kind = "reference" if v0.ref_available() else "port"
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
        "scaling": "weak", "vs_baseline": None, "dtype": dt, "data": "synthetic (seeded)",
        "config": {"workload": label, "m": m, "n": n, "k": k, "seed": seed},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOPS", "cores": threads, "kind": kind,
                         "sample": f"v0 on a {rows_used}-row slice of A per step (x{n}x{k}), "
                                   f"OpenBLAS {threads} threads"},
        "e2e": {"value": round(value, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "sustained TFLOPS @4096^3 fp16 (10 warmup+100 iter avg), % of B200 tensor peak"


# ------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["vk", "reference"], default="vk")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="rubric")
    ap.add_argument("--algo", default="auto")
    ap.add_argument("--tile-n", type=int, default=0)
    ap.add_argument("--allgather", nargs="?", const="nccl", default=None, choices=["nccl", "pipelined", "fused"],
                    help="all-gather C on every rank: nccl = NCCL after the GEMM (default when given); "
                         "pipelined = copy-engine peer pushes of finished row chunks overlapped with the GEMM; "
                         "fused = the GEMM epilogue stores every C box into the peers' C as well")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    cfg = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, cfg)
        return

    import torch
    import torch.distributed as dist
    import vibekernel_b200 as vk
    from vibekernel_b200 import dist_gemm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)

    m_cfg, n, k, seed, distname, lo, hi, dt, acc, label = cfg
    strong = args.workload == "shard16k"
    m_total = m_cfg if strong else m_cfg * world
    off = vk.row_blocks(m_total, world)
    rows = off[rank + 1] - off[rank]
    tdt = torch.float16 if dt == "f16" else torch.float32
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed * 1000 + rank)

    def rand(shape):
        if distname == "normal":
            return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).to(tdt)
        return (torch.rand(shape, generator=gen, device=dev, dtype=torch.float32) * (hi - lo) + lo).to(tdt)

    A = rand((rows, k))
    g_b = torch.Generator(device=dev)
    g_b.manual_seed(seed * 1000 + 999)  # B identical on every rank (replicated)
    B = (torch.randn((k, n), generator=g_b, device=dev, dtype=torch.float32) if distname == "normal" else
         torch.rand((k, n), generator=g_b, device=dev, dtype=torch.float32) * (hi - lo) + lo).to(tdt)
    C_full = torch.empty((m_total, n), dtype=tdt, device=dev) if (args.allgather and world > 1) else None
    C = C_full[off[rank]:off[rank + 1]] if C_full is not None else torch.empty((rows, n), dtype=tdt, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def local_gemm(a, b, out, peers=None):
        vk.gemm(a, b, out, acc=acc, algo=args.algo, tile_n=args.tile_n, stream=stream, peers=peers)

    peer_gather = None
    launches_per_step = 1
    if C_full is not None and args.allgather in ("pipelined", "fused"):
        peer_gather = dist_gemm.PeerRowGather(C_full, off, rank)
        launches_per_step = len(dist_gemm.chunk_rows(rows, 2)) if args.allgather == "pipelined" else 1

    def step():
        if peer_gather is not None:
            peer_gather.run(A, B, local_gemm, chunks=2, mode=args.allgather)  # GEMM + overlapped peer stores
        else:
            local_gemm(A, B, C)

    def gather():
        if C_full is not None and peer_gather is None:
            dist_gemm.allgather_rows(C_full, off, rank)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        flush.fill_(1.0)
        step()
        gather()
    barrier()

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    evg = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    probe = dt == "f16"  # the tensor-core kernels carry the in-kernel clock probe
    if probe:
        vk.set_option("clock_probe", 1)
        vk.read_clock_probe(local, clear=True)
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.fill_(1.0)
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
            evg[i][0].record(stream)
            gather()
            evg[i][1].record(stream)
            ev[i][1].synchronize()  # the reference driver synchronises every iteration
        barrier()
    kernel_mhz = None
    if probe:
        kernel_mhz, _ = vk.read_clock_probe(local, clear=True)
        vk.set_option("clock_probe", 0)
    gemm_ms = sum(s.elapsed_time(e) for s, e in ev)
    gather_ms = sum(s.elapsed_time(e) for s, e in evg) if C_full is not None else 0.0
    err = vk.device_error(local)
    if err:
        raise SystemExit(f"device error word {err:#x}")
    total_ms = gemm_ms + gather_ms
    t = torch.tensor([total_ms, gemm_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, gemm_ms_max = float(t[0]), float(t[1])
    flops_step = 2.0 * m_total * n * k
    value = flops_step * args.steps / (total_ms * 1e-3) / 1e12
    kernel_ms = gemm_ms / args.steps  # this rank's average launch duration

    # ---------------- e2e: the public host-buffer API (vk_gemm_host): every step copies A and B in
    # from pinned host memory and C back out, pipelined with the GEMM in row blocks; the call is
    # synchronous, so host wall-clock around it covers every byte moved.
    e2e = None
    if not args.no_e2e:
        hA = torch.empty(A.shape, dtype=tdt, pin_memory=True)
        hB = torch.empty(B.shape, dtype=tdt, pin_memory=True)
        hC = torch.empty(C.shape, dtype=tdt, pin_memory=True)
        hA.copy_(A)
        hB.copy_(B)
        e2e_steps = max(3, min(args.steps, 20))
        for _ in range(3):
            vk.gemm_host(hA, hB, hC, acc=acc, algo=args.algo)
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            vk.gemm_host(hA, hB, hC, acc=acc, algo=args.algo)
        t_e2e = time.perf_counter() - t0
        te = torch.tensor([t_e2e], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_val = flops_step * e2e_steps / float(te[0]) / 1e12
        e2e = {"value": round(e2e_val, 3), "unit": "TFLOPS",
               "h2d_bytes_per_step": int((hA.numel() + hB.numel()) * hA.element_size() * world),
               "d2h_bytes_per_step": int(hC.numel() * hC.element_size() * world), "steps": e2e_steps,
               "api": "vk_gemm_host (pinned host A, B, C; copies pipelined with the GEMM in row blocks)",
               "timing": "host wall clock around the synchronous call, max over ranks"}

    if rank == 0:
        pk, pk_src = peaks()
        if dt == "f16":
            peak = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
            roof_unit, bound = "TFLOP/s", "tensor"
        else:
            sm_mhz = clocks.summary()["sm_mhz"] or pk.get("sm_max_mhz", 1965.0)
            peak = 148 * 128 * 2 * float(sm_mhz) * 1e6 / 1e12  # FFMA peak at the sampled clock
            roof_unit, bound = "TFLOP/s", "ffma"
        achieved = 2.0 * rows * n * k / (kernel_ms * 1e-3) / 1e12
        roof = {"bound": bound, "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": roof_unit,
                "frac": round(achieved / peak, 4), "traffic": TRAFFIC.get(args.workload),
                "traffic_unit": "bytes/launch",
                "algorithmic_bytes": int((rows * k + k * n + rows * n) * (2 if dt == "f16" else 4)),
                "peak_source": (f"MEASURED_PEAKS.json bf16_tflops (burst), of {pk_src}" if dt == "f16"
                                else "148 SMs x 128 FP32 lanes x 2 x sampled SM clock")}
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": dt, "data": "synthetic (seeded uniform/normal inputs, BASELINE shapes)",
            "config": {"workload": label, "m": m_total, "n": n, "k": k, "m_per_gpu": rows, "acc": acc,
                       "algo": args.algo, "tile_n": args.tile_n or 256, "parallelism": f"rowshard{world}",
                       "allgather_c": (args.allgather if C_full is not None else False),
                       "l2": "flushed before every timed call (256 MiB write outside the event pair)",
                       "timing": "per-call CUDA events + event synchronize (reference main.cpp loop)"},
            "roofline": roof,
            "pct_of_dense_peak_2250": round(value / world / 2250.0, 4),
            "clocks": dict(clocks.summary(), kernel_sm_mhz=(round(kernel_mhz, 1) if kernel_mhz else None)),
            "clock_true_peak_frac": (round(achieved / (148 * 8192 * kernel_mhz * 1e6 / 1e12), 4)
                                     if (kernel_mhz and dt == "f16") else None),
            "gpu_launches": args.steps * launches_per_step,
            "e2e": e2e,
        }
        if C_full is not None:
            line["gather_ms_per_step"] = round(gather_ms / args.steps, 4)
        if world == 1 and not args.no_cpu_baseline:
            from oracle import v0
            npdt = np.float16 if dt == "f16" else np.float32
            hA_np, hB_np = v0.make_inputs(m_cfg, n, k, seed, distname, lo, hi, npdt)
            threads = os.cpu_count() or 1
            tfl, rws, secs = cpu_v0_sample(hA_np, hB_np, dt, 10.0)
            line["cpu_baseline"] = {
                "value": round(tfl, 4), "unit": "TFLOPS", "cores": threads,
                "kind": "reference" if v0.ref_available() else "port",
                "sample": f"reference v0 (oracle/_ref) on {rws} of {m_cfg} rows ({secs:.2f} s), OpenBLAS {threads} threads"}
        print(json.dumps(line), flush=True)
    if peer_gather is not None:
        peer_gather.close()
    if world > 1:
        dist.destroy_process_group()


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant kernel, from
# the ncu captures summarised in profiles/tc_gemm_pair_rubric4096.md and profiles/sgemm_ffma_4096.md;
# None where no capture of the current kernel exists.
TRAFFIC = {"rubric": 136087296, "ragged": 116693248, "sgemm": 568920064}

if __name__ == "__main__":
    main()
