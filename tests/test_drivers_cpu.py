"""Drop-in build interfaces on CPU: every driver builds from the reference's make
variables, and a main run without a GPU fails the way the reference's mains do
(non-zero exit, an error line), which its drivers turn into a skipped row.

When the reference tree is present, its own tcgen05_sparse_mma/benchmark.py is
run unchanged against our Makefile with --build-only (the mode its authors used
on machines without sm_100, tcgen05_sparse_mma/REPORT.md:136-174)."""
import csv
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRV = os.path.join(ROOT, "microbench-blackwell_b200", "drivers")
# the reference checkout: $REFERENCE_DIR, else `reference` beside this repository
REF = os.environ.get("REFERENCE_DIR", os.path.abspath(os.path.join(ROOT, "..", "reference")))


def make(d, *args):
    return subprocess.run(["make", "-s"] + list(args), cwd=d, capture_output=True, text=True)


@pytest.mark.parametrize("d,target,vars_", [
    ("umma_throughput", "umma_tput.out", ["MMA_FORMAT=4", "MMA_M=256", "MMA_N=256", "MMA_K=32",
                                           "MMA_DEPTH=64", "CTA_GROUP=2", "AB_LAYOUT=1"]),
    ("tcgen05_sparse_mma", "tcgen05_sparse_mma.out", ["KIND=mxf4nvf4", "A_TYPE=nvf4",
                                                      "B_TYPE=nvf4", "SPARSITY=1",
                                                      "SCALE_TYPE=ue4m3", "CTA_GROUP=2",
                                                      "MMA_M=256", "MMA_K=128"]),
    ("tma2d_throughput", "tma2d_tput.out", ["NUM_STAGES=2", "SMEM_HEIGHT=64"]),
    ("cutlass_gemm_mainloop", "cutlass_gemm_bench.out", ["TILE_M=128", "TILE_N=256", "TILE_K=128",
                                                         "DTYPE_ID=1"]),
    ("umma_latency", "umma_lat.out", ["MMA_FORMAT=1", "MMA_M=256", "MMA_N=128", "MMA_K=32",
                                      "CTA_GROUP=2", "AB_LAYOUT=0"]),
    ("tma_throughput", "tma_tput.out", ["NUM_STAGES=4", "LOAD_SIZE=16384"]),
    ("tma2d_latency", "tma2d_lat.out", ["SMEM_WIDTH=128", "SMEM_HEIGHT=16"]),
])
def test_driver_builds_and_fails_cleanly_without_gpu(d, target, vars_):
    path = os.path.join(DRV, d)
    assert make(path, "clean").returncode == 0
    b = make(path, target, *vars_)
    assert b.returncode == 0, b.stderr
    if torch.cuda.is_available():
        pytest.skip("GPU present: run behaviour covered by tests/test_zperf_drivers_gpu.py")
    r = subprocess.run([f"./{target}"], cwd=path, capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    assert "Error" in r.stdout + r.stderr or "failed" in r.stderr
    assert make(path, "clean").returncode == 0
    assert not os.path.exists(os.path.join(path, target))


def test_cutlass_mainloop_rejects_shapes_the_engine_does_not_build():
    # like the reference main when CUTLASS cannot implement a configuration:
    # a "Cannot implement" line and exit 1 (before any device call)
    path = os.path.join(DRV, "cutlass_gemm_mainloop")
    for vars_ in (["TILE_N=16"], ["TILE_M=256"], ["TILE_K=32"], ["DTYPE_ID=1", "TILE_K=64"]):
        make(path, "clean")
        b = make(path, "cutlass_gemm_bench.out", *vars_)
        assert b.returncode == 0, b.stderr
        r = subprocess.run(["./cutlass_gemm_bench.out"], cwd=path, capture_output=True, text=True,
                           timeout=60)
        assert r.returncode == 1 and "Cannot implement" in r.stderr, (vars_, r.stderr)
    make(path, "clean")


def test_compile_time_guards():
    path = os.path.join(DRV, "tcgen05_sparse_mma")
    b = make(path, "tcgen05_sparse_mma.out", "INSTRUCTION=ws", "CTA_GROUP=2")
    assert b.returncode != 0 and "CTA_GROUP=1" in b.stderr
    make(path, "clean")


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference tree not present")
def test_reference_sparse_driver_runs_unchanged_build_only(tmp_path):
    out = tmp_path / "rows.csv"
    d = os.path.join(DRV, "tcgen05_sparse_mma")
    r = subprocess.run([sys.executable, os.path.join(REF, "tcgen05_sparse_mma", "benchmark.py"),
                        "--build-only", "--preset", "smoke", "--max-configs", "6",
                        "--output", str(out), "--overwrite"],
                       cwd=d, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    assert "BUILD_FAILED" not in r.stderr
    rows = list(csv.DictReader(open(out)))
    assert len(rows) == 6
    assert list(rows[0].keys())[:3] == ["PairID", "Instruction", "Kind"]
    make(d, "clean")


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference tree not present")
def test_reference_tma2d_latency_driver_builds_unchanged(tmp_path):
    # the reference's own tma2d_latency/benchmark.py drives this directory's Makefile
    # (make clean; make tma2d_lat.out CTAS_PER_SM= SMEM_WIDTH= SMEM_HEIGHT=; run); without
    # a GPU the run step fails, so the check is that every build succeeded
    d = os.path.join(DRV, "tma2d_latency")
    r = subprocess.run([sys.executable, os.path.join(REF, "tma2d_latency", "benchmark.py"),
                        "--heights", "1", "64", "--output", str(tmp_path / "lat.csv"), "--overwrite"],
                       cwd=d, capture_output=True, text=True, timeout=600)
    assert "Build failed" not in r.stderr, r.stderr
    if not torch.cuda.is_available():
        assert r.stderr.count("Run failed") == 2, r.stderr
    make(d, "clean")


UMMA_TPUT_HEADER = ["Format", "ABLayout", "CTAGroup", "M", "N", "K", "PipelineDepth", "Cycles",
                    "CyclesPerMMA", "FLOPsPerCycle"]  # umma_throughput/benchmark.py:46-49
UMMA_LAT_HEADER = ["Format", "ABLayout", "CTAGroup", "M", "N", "K", "MedianCycles"]


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference tree not present")
@pytest.mark.parametrize("d,script,header,n_runs", [
    # one N, cta_group 1 (M 64 and 128), bf16 SS: 2 x 5 pipeline depths / 2 latency points
    ("umma_throughput", "benchmark.py", UMMA_TPUT_HEADER, 10),
    ("umma_latency", "benchmark.py", UMMA_LAT_HEADER, 2),
])
def test_reference_umma_drivers_run_unchanged(tmp_path, d, script, header, n_runs):
    # the reference's own umma_throughput / umma_latency benchmark.py drive this
    # directory's Makefile (make clean; make <x>.out MMA_FORMAT= MMA_M= ...; ./<x>.out)
    # and write their CSV header; without a GPU every run step fails after its build
    out = tmp_path / "rows.csv"
    path = os.path.join(DRV, d)
    r = subprocess.run([sys.executable, os.path.join(REF, d, script), "0", "--cta-group", "1",
                        "--mode", "ss", "--n-sweep", "256:256:16", "-o", str(out), "--overwrite"],
                       cwd=path, capture_output=True, text=True, timeout=900)
    assert "Build failed" not in r.stderr, r.stderr
    with open(out) as f:
        assert next(csv.reader(f)) == header
    if not torch.cuda.is_available():
        assert r.stderr.count("Run failed") == n_runs, r.stderr
        assert r.returncode == 1  # "No successful results"
    else:
        assert r.returncode == 0, r.stderr
    make(path, "clean")
