"""The task-1 C++ driver (task-1/): builds, keeps the reference's CLI and result line, and its GPU
versions pass the error check through libvkgemm.so.  Also the anti-library scan of
scripts/check_handwritten.sh (restated here, and the reference's own script when its tree is present)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TASK = os.path.join(ROOT, "task-1")
BUILD = os.path.join(TASK, "build")
RESULT = re.compile(r"\[Playground\] Result >>> TFLOPS: ([0-9.eE+-]+); Average Error: ([0-9.eE+-]+)")
EXTRA = re.compile(r"RelFrobenius\(fp32 copy\): ([0-9.eE+-]+); MaxElemRel\(tau=1e-2\*RMS\): ([0-9.eE+-]+); "
                   r"KernelSmMHz: ([0-9.]+)")
# scripts/check_handwritten.sh:18 -- case-insensitive, lines starting with // or * are skipped
BANNED = re.compile(r"cutlass|cute/|#include[ ]*<cute|cublas|cublasLt|cudnn", re.I)


@pytest.fixture(scope="module")
def built():
    res = subprocess.run(["make", "-C", TASK, "-j4"], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    return BUILD


def _run(binary, *args, timeout=600):
    return subprocess.run([os.path.join(BUILD, binary), *args], capture_output=True, text=True, timeout=timeout)


def test_v0_cpu_paths_and_result_line(built):
    for b in ("task1_float16_v0", "task1_float32_v0"):
        r = _run(b, "-m", "96", "-n", "80", "-k", "72", "--seed", "5")
        assert r.returncode == 0, r.stderr
        m = RESULT.search(r.stdout)
        assert m and float(m.group(2)) == 0.0  # v0 against itself
        assert "Start Testing for GEMM Version 0" in r.stdout


SHARDED = re.compile(r"Sharded >>> GPUs: (\d+); AllGather: (\w+); AllGpusEqual: (\d)")


def test_gpus_option_needs_a_gpu_version(built):
    r = _run("task1_float16_v0", "--gpus", "2", "-m", "64", "-n", "64", "-k", "64")
    assert r.returncode == 2 and "GPU version" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("gpus,mode", [(1, "none"), (1, "nccl"), (2, "none"), (2, "nccl"), (2, "pipelined"),
                                       (2, "fused"), (2, "nvls")])
def test_sharded_driver(built, gpus, mode):
    """--gpus: the driver's row-sharded mode through vk_gemm_sharded, error check against v0."""
    import torch
    if torch.cuda.device_count() < gpus:
        pytest.skip(f"needs {gpus} GPUs")
    r = _run("task1_float16_v1", "-m", "1024", "-n", "768", "-k", "512", "-w", "2", "-t", "5", "--seed", "0",
             "--dist", "uniform", "--gpus", str(gpus), "--allgather", mode)
    if mode == "nvls" and r.returncode != 0 and "multicast" in r.stderr + r.stdout:
        pytest.skip("no NVLS multicast on these GPUs")
    assert r.returncode == 0, r.stdout + r.stderr
    res, sh = RESULT.search(r.stdout), SHARDED.search(r.stdout)
    assert res and sh, r.stdout
    assert float(res.group(1)) > 0 and float(res.group(2)) <= 2e-3
    assert int(sh.group(1)) == gpus and sh.group(2) == mode and sh.group(3) == "1"


def test_cli_help_and_errors(built):
    r = _run("task1_float16_v1", "-h")
    assert r.returncode == 0 and "-m arg" in r.stdout and "--n_warmup" in r.stdout
    r = _run("task1_float16_v1", "-m")
    assert r.returncode == 2
    r = _run("task1_float16_v1", "--dist", "cauchy")
    assert r.returncode == 2


def _scan_files():
    out = []
    for base in ("task-1/src", "task-1/include", "include"):
        for dp, _, fs in os.walk(os.path.join(ROOT, base)):
            for f in fs:
                if f.endswith((".cu", ".cuh", ".cpp", ".hpp", ".h")) and not re.search(r"_v0(_|\.)", f):
                    out.append(os.path.join(dp, f))
    return out


def test_handwritten_scan_restated():
    hits = []
    for path in _scan_files():
        for i, line in enumerate(open(path, encoding="utf-8"), 1):
            if BANNED.search(line) and not re.match(r"\s*(//|\*)", line):
                hits.append(f"{os.path.relpath(path, ROOT)}:{i}: {line.strip()}")
    assert not hits, "\n".join(hits)
    assert len(_scan_files()) >= 12


@pytest.mark.gpu
@pytest.mark.parametrize("binary,frob_tol,avg_tol", [
    ("task1_float16_v1", 1e-4, 2e-3), ("task1_float16_v2", 5e-3, 5e-2), ("task1_float16_v3", 1e-4, 2e-3),
    ("task1_float16_v4", 1e-4, 2e-3), ("task1_float32_v1", 1e-5, 1e-3)])
def test_gpu_versions(built, binary, frob_tol, avg_tol):
    r = _run(binary, "-m", "1024", "-n", "1024", "-k", "1024", "-w", "3", "-t", "10", "--seed", "0",
             "--dist", "uniform")
    assert r.returncode == 0, r.stdout + r.stderr
    res = RESULT.search(r.stdout)
    extra = EXTRA.search(r.stdout)
    assert res and extra, r.stdout
    assert float(res.group(1)) > 0
    assert float(res.group(2)) <= avg_tol
    assert float(extra.group(1)) <= frob_tol
    assert float(extra.group(2)) <= (2e-3 if frob_tol <= 1e-4 else 1.0)
