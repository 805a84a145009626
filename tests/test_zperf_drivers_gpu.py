"""The drop-in benchmark mains on the GPU: build with the reference's make
variables, run, and parse the RESULT line the way the reference's drivers do
(umma_throughput/benchmark.py:109-128, tcgen05_sparse_mma/benchmark.py:283-310).

Issue rates are compared with the reference's own published measurements
(tests/golden/umma_tput_reference_rows.csv, extracted from
umma_throughput/tput_results_max.csv by tests/golden/make_umma_golden.py): the
engine's probe must issue within 10 % of the reference's cycles per MMA.

Every test here asserts a rate, a latency or a bandwidth.  The file name sorts
after every parity file (and before test_zz_no_alloc.py), so that under
`pytest -x` a slow or busy GPU can stop the run only after all correctness
results are in."""
import csv
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRV = os.path.join(ROOT, "microbench-blackwell_b200", "drivers")
GOLD = os.path.join(ROOT, "tests", "golden", "umma_tput_reference_rows.csv")
GOLD_LAT = os.path.join(ROOT, "tests", "golden", "umma_lat_reference_rows.csv")
GOLD_TMA_LAT = os.path.join(ROOT, "tests", "golden", "tma2d_lat_reference_rows.csv")
FMT_ID = {"BF16": 0, "E4M3": 1, "S8": 2, "F4": 3, "MXF8": 4, "MXF4": 5}
FMT_K = {0: 16, 1: 32, 2: 32, 3: 64, 4: 32, 5: 64}


def build_run(d, target, variables):
    subprocess.run(["make", "-s", "clean"], cwd=d, check=True, capture_output=True)
    b = subprocess.run(["make", "-s", target] + [f"{k}={v}" for k, v in variables.items()], cwd=d,
                       capture_output=True, text=True)
    assert b.returncode == 0, b.stderr
    r = subprocess.run([f"./{target}"], cwd=d, capture_output=True, text=True, timeout=180)
    return r


def result_line(out):
    for line in out.splitlines():
        if line.startswith("RESULT,"):
            return line.split(",")
    raise AssertionError(f"no RESULT line in: {out!r}")


@pytest.mark.parametrize("row", list(csv.DictReader(open(GOLD))),
                         ids=lambda r: f"{r['Format']}-{r['ABLayout']}-cg{r['CTAGroup']}-{r['M']}x{r['N']}")
def test_umma_tput_matches_reference_rates(row):
    fmt = FMT_ID[row["Format"]]
    v = dict(MMA_FORMAT=fmt, MMA_M=row["M"], MMA_N=row["N"], MMA_K=FMT_K[fmt],
             MMA_DEPTH=row["PipelineDepth"], CTA_GROUP=row["CTAGroup"],
             AB_LAYOUT=1 if row["ABLayout"] == "TS" else 0)
    r = build_run(os.path.join(DRV, "umma_throughput"), "umma_tput.out", v)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Done!" in r.stdout
    p = result_line(r.stdout)
    assert len(p) >= 8
    M, N, K = int(p[1]), int(p[2]), int(p[3])
    cpm = float(p[7])
    assert (M, N, K) == (int(row["M"]), int(row["N"]), FMT_K[fmt])
    assert int(p[6]) == int(row["PipelineDepth"]) * 1000
    ref = float(row["CyclesPerMMA"])
    # (cta_group::2 M=128 N=128 executes in 32.7 cycles, less than a rolled issue
    # loop took per MMA: the probe unrolls its depth loop, as the reference's
    # compile-time depth is, and measures 32.9)
    assert abs(cpm - ref) / ref < 0.10, f"{cpm:.2f} cycles/MMA vs reference {ref:.2f}"


SPARSE_CASES = [
    # forms whose semantics this repository validates end to end elsewhere
    # (bf16 sparse / dense: tests/test_sparse_gpu.py; NVFP4 block16:
    # tests/test_nvfp4_gpu.py).  Other kinds are built and shape-checked but not
    # run by the test suite.
    dict(KIND="f16", A_TYPE="bf16", B_TYPE="bf16", SPARSITY=0, CTA_GROUP=1, MMA_M=128, MMA_N=256, MMA_K=16),
    dict(KIND="f16", A_TYPE="bf16", B_TYPE="bf16", SPARSITY=1, CTA_GROUP=1, MMA_M=128, MMA_N=256, MMA_K=32),
    dict(KIND="f16", A_TYPE="bf16", B_TYPE="bf16", SPARSITY=1, CTA_GROUP=2, MMA_M=256, MMA_N=256, MMA_K=32),
    dict(KIND="f16", A_TYPE="bf16", B_TYPE="bf16", SPARSITY=1, CTA_GROUP=2, MMA_M=256, MMA_N=128, MMA_K=32),
    dict(KIND="mxf4nvf4", A_TYPE="nvf4", B_TYPE="nvf4", SPARSITY=0, CTA_GROUP=1, MMA_M=128, MMA_N=256,
         MMA_K=64, SCALE_TYPE="ue4m3"),
]


@pytest.mark.parametrize("case", SPARSE_CASES, ids=lambda c: "-".join(str(v) for v in c.values()))
def test_sparse_driver_throughput_and_latency(case):
    d = os.path.join(DRV, "tcgen05_sparse_mma")
    v = dict(case, MMA_DEPTH=128, MODE="throughput")
    r = build_run(d, "tcgen05_sparse_mma.out", v)
    assert r.returncode == 0, r.stdout + r.stderr
    p = result_line(r.stdout)
    assert p[1] == "throughput" and len(p) == 18
    cycles, total, cpm = int(p[13]), int(p[14]), float(p[15])
    assert total == 128 * 1000 and cycles > 0
    n = case["MMA_N"]
    ii = n / 2 if case["CTA_GROUP"] == 1 or case["MMA_M"] == 256 else n / 4
    assert 0.8 * ii < cpm < 1.6 * ii, f"{cpm:.1f} cycles/MMA, expected about {ii}"
    lat = build_run(d, "tcgen05_sparse_mma.out", dict(case, MMA_DEPTH=1, MODE="latency"))
    assert lat.returncode == 0, lat.stdout + lat.stderr
    q = result_line(lat.stdout)
    assert q[1] == "latency" and len(q) == 15 and int(q[12]) > 0


def test_tma2d_stream_bandwidth():
    r = build_run(os.path.join(DRV, "tma2d_throughput"), "tma2d_tput.out",
                  dict(CTAS_PER_SM=1, NUM_STAGES=4, SMEM_WIDTH=128, SMEM_HEIGHT=32))
    assert r.returncode == 0, r.stdout + r.stderr
    line = [l for l in r.stdout.splitlines() if l.startswith("streamed")][0]
    gbs = float(line.split(":")[1].split("GB/s")[0])
    # reference: 7.22 TB/s for this configuration by ncu's kernel-only DRAM rate
    # (tma2d_tput_results.csv:19); this stager measures 7.14 TB/s by the same
    # counter and 7.14 by CUDA events.  The GPUs are shared, so the floor is about
    # half of that: it catches a broken stager, not a slow neighbour
    assert gbs > 3500, line


def test_probe_rejects_shapes_outside_the_tables(engine):
    import b2g

    with pytest.raises(b2g.B2GError) as e:
        engine.probe_mma(kind=1, a_type=1, b_type=1, cta_group=1, m=96, n=128, depth=4)
    assert e.value.status == 1
    with pytest.raises(b2g.B2GError):
        engine.probe_mma(kind=4, a_type=0, b_type=0, cta_group=1, m=128, n=128, depth=4,
                         instruction=1)
    # a type code outside the kind's element types (kind::mxf4 takes e2m1 as code 1,
    # not kind::f8f6f4's 5) is refused on the host: on the device it is an illegal
    # instruction
    with pytest.raises(b2g.B2GError) as e:
        engine.probe_mma(kind=5, a_type=5, b_type=5, cta_group=2, m=256, n=256, depth=4,
                         scale_type=1)
    assert e.value.status == 1


# The reference's per-CTA CUTLASS mainloop numbers (one CTA, M = TILE_M, N =
# TILE_N, K = 131072): cutlass_gemm_mainloop/results.csv:461 (BF16 128x256x64,
# 10.4596 TFLOPS) and :938 (FP8_E4M3 128x256x128, 20.6377 TFLOPS), the best rows
# of its sweep for those tiles.
CUTLASS_PER_CTA = [
    (dict(TILE_M=128, TILE_N=256, TILE_K=64, STAGES=0, DTYPE_ID=0), "BF16", 10.4596),
    (dict(TILE_M=128, TILE_N=256, TILE_K=128, STAGES=0, DTYPE_ID=1), "FP8_E4M3", 20.6377),
]


@pytest.mark.parametrize("v,dtype,ref", CUTLASS_PER_CTA, ids=["bf16-128x256", "fp8-128x256"])
def test_cutlass_mainloop_dropin_beats_reference_published_per_cta(v, dtype, ref):
    r = build_run(os.path.join(DRV, "cutlass_gemm_mainloop"), "cutlass_gemm_bench.out", v)
    assert r.returncode == 0, r.stdout + r.stderr
    p = r.stdout.strip().splitlines()[-1].split(",")
    assert len(p) == 10 and p[7] == dtype
    assert [int(x) for x in p[:7]] == [v["TILE_M"], v["TILE_N"], 131072, v["TILE_M"], v["TILE_N"],
                                       v["TILE_K"], v["STAGES"]]
    tflops = float(p[9])
    assert tflops > ref, f"{tflops:.2f} TFLOPS per CTA vs the reference's CUTLASS {ref:.2f}"


@pytest.mark.parametrize("row", list(csv.DictReader(open(GOLD_LAT))),
                         ids=lambda r: f"{r['Format']}-{r['ABLayout']}-cg{r['CTAGroup']}-{r['M']}x{r['N']}")
def test_umma_latency_matches_reference(row):
    # reference: umma_latency/lat_results_full.csv (tests/golden/make_umma_lat_golden.py);
    # single-MMA issue -> commit -> wait round trip, median of 100
    fmt = FMT_ID[row["Format"]]
    v = dict(MMA_FORMAT=fmt, MMA_M=row["M"], MMA_N=row["N"], MMA_K=FMT_K[fmt],
             CTA_GROUP=row["CTAGroup"], AB_LAYOUT=1 if row["ABLayout"] == "TS" else 0)
    r = build_run(os.path.join(DRV, "umma_latency"), "umma_lat.out", v)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Done!" in r.stdout
    p = result_line(r.stdout)
    assert len(p) == 5
    assert (int(p[1]), int(p[2]), int(p[3])) == (int(row["M"]), int(row["N"]), FMT_K[fmt])
    med, ref = int(p[4]), int(row["MedianCycles"])
    assert abs(med - ref) / ref < 0.25, f"{med} cycles vs reference {ref}"


@pytest.mark.parametrize("v,floor_gbs", [
    (dict(CTAS_PER_SM=1, NUM_STAGES=1, LOAD_SIZE=32768), 1800.0),   # the reference's defaults
    (dict(CTAS_PER_SM=1, NUM_STAGES=4, LOAD_SIZE=32768), 2000.0),
    (dict(CTAS_PER_SM=2, NUM_STAGES=2, LOAD_SIZE=49152), 2000.0),
], ids=["defaults", "4x32k", "2cta-2x48k"])
def test_tma_1d_stream_bandwidth(v, floor_gbs):
    # 1D cp.async.bulk streaming of about 2 GB (tma_throughput/tma_tput.cu; the
    # reference publishes no figure for it).  Measured by CUDA events on a B200:
    # 3.7 TB/s at the defaults, 4.5-4.6 TB/s from 4 slots of 32 KB on (2.99 TB/s on
    # one busy box); the assertions are floors at about half of those, since the
    # GPUs are shared
    r = build_run(os.path.join(DRV, "tma_throughput"), "tma_tput.out", v)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [l for l in r.stdout.splitlines() if l.startswith("streamed")][-1]
    gbs = float(line.split(":")[1].split("GB/s")[0])
    assert gbs > floor_gbs, line


TMA_LAT_ROWS = {int(r["SmemHeight"]): r for r in csv.DictReader(open(GOLD_TMA_LAT))}


@pytest.mark.parametrize("h", [1, 8, 32, 128, 256])
def test_tma2d_load_latency_against_reference(h):
    # one 128 x h fp32 TMA 2D load per CTA from DRAM (tma2d_latency/tma2d_lat.cu): the
    # median of the launch medians, parsed from SUMMARY,<med>,<min>,<max> as the
    # reference's driver parses it, against the reference's published medians
    r = build_run(os.path.join(DRV, "tma2d_latency"), "tma2d_lat.out",
                  dict(CTAS_PER_SM=1, SMEM_WIDTH=128, SMEM_HEIGHT=h))
    assert r.returncode == 0, r.stdout + r.stderr
    line = [l for l in r.stdout.splitlines() if l.startswith("SUMMARY,")][-1].split(",")
    med, lo, hi = int(line[1]), int(line[2]), int(line[3])
    # (the median is over the 10 launches' medians, min / max over one more launch, so
    # the median need not lie between them: the reference's own row for 2 rows has
    # median 1413 below min 1521)
    assert 0 < lo <= hi and med > 0
    ref = float(TMA_LAT_ROWS[h]["LatencyCyclesMedian"])
    # measured on a B200: 0.56-1.02 x the reference's medians over 1-256 rows
    assert 0.4 < med / ref < 2.0, f"{h} rows: {med} cycles vs reference {ref}"


# The reference's own CUTLASS comparator (cutlass_gemm_mainloop/cutlass_gemm_bench.cu),
# built unchanged into oracle/_ref/ by `make -C oracle cutlass`, at the reference's
# best stage count of each 128 x N tile; run on the same GPU as the engine's drop-in
# main with the same variables.
REF_BIN = os.path.join(ROOT, "oracle", "_ref")
SAME_BOX = [(0, 64, 64, 6), (0, 128, 64, 7), (0, 192, 64, 5), (0, 256, 64, 4),
            (1, 64, 128, 7), (1, 128, 128, 6), (1, 192, 128, 4), (1, 256, 128, 0)]


def _tflops(line_out):
    p = line_out.strip().splitlines()[-1].split(",")
    assert len(p) == 10, line_out
    return float(p[9])


@pytest.mark.parametrize("dt,n,k,stages", SAME_BOX,
                         ids=[f"{'bf16' if d == 0 else 'fp8'}-128x{n}" for d, n, _, _ in SAME_BOX])
def test_cutlass_mainloop_against_reference_binary_same_box(dt, n, k, stages):
    ref = os.path.join(REF_BIN, f"cutlass_{dt}_{n}_{k}_{stages}.out")
    if not os.path.exists(ref):
        pytest.skip("reference CUTLASS comparator not built (make -C oracle cutlass)")
    r_ref = subprocess.run([ref], capture_output=True, text=True, timeout=180)
    assert r_ref.returncode == 0, r_ref.stdout + r_ref.stderr
    # the engine's drop-in main, best of its own stage counts at this tile
    best = 0.0
    for st in (0, 4):
        r = build_run(os.path.join(DRV, "cutlass_gemm_mainloop"), "cutlass_gemm_bench.out",
                      dict(TILE_M=128, TILE_N=n, TILE_K=k, STAGES=st, DTYPE_ID=dt))
        assert r.returncode == 0, r.stdout + r.stderr
        best = max(best, _tflops(r.stdout))
    ref_tf = _tflops(r_ref.stdout)
    print(f"128x{n} {'bf16' if dt == 0 else 'fp8'}: engine {best:.2f} / CUTLASS {ref_tf:.2f} TFLOPS "
          f"per CTA = {best / ref_tf:.2f}")
    # Same box, CUTLASS 4.5 headers: the reference's kernel runs 1.3-1.4x its own
    # published figures; the engine measured 0.98-1.01x of it at 128 x 192 and
    # 128 x 256, 0.70-0.75x at 128 x 64 and 128 x 128 (issue-bound narrow tiles)
    assert best > (0.9 if n >= 192 else 0.6) * ref_tf, (best, ref_tf)
