#!/usr/bin/env python
"""bench.py -- headline benchmark of the B200 tensor-core GEMM engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference]

One "step" is one GEMM C = alpha * A . B^T of the configured workload over
inputs already resident in HBM.  The default workload is BASELINE config 2,
the configuration the headline metric is quoted on: dense fp8 e4m3,
M = N = K = 8192 per GPU, per-tensor scales 1/64 (alpha = 1/4096), fp32
accumulate, bf16 C, cta_group::2 with 256 x 256 pair tiles.

Multi-GPU (torchrun, one process per GPU, NCCL): M-row shards of one global
A of N*8192 rows, B replicated -- weak scaling, no collective on the data path.
After timing, C is all-gathered over NCCL once for verification (timed
separately, not part of `value`).

Printed on rank 0: ONE JSON line with value (whole-box TFLOP/s), the kernel's
roofline, the CPU baseline, the end-to-end number through b2g_gemm_host (host
buffers, copies inside the timed region), clocks sampled during the timed
region and the number of libb2g kernel launches timed.  The same run also
measures, each as its own short burst after the headline:

  sustained   the headline GEMM back to back for >= 2 s of device time (one GPU),
              with its own clock samples: the power-capped figure;
  secondary   the north star's other targets: bf16 8192^3, cfg1, cfg3 beside the
              same-shape dense kernel (sparse_over_dense) and cfg4 on one GPU; on
              N GPUs, cfg4 as one 16384^3 problem split into M-row shards (strong
              scaling), with per-GPU waves and the all-gather of C timed apart.

`--impl reference` times the CPU implementation of the path (the reference has
none of its own -- its kernels never read a GEMM result back -- so this is the
repository's CPU restatement, oracle/liboracle.so) on the host cores, on a
bounded row slab of the same workload per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "microbench-blackwell_b200"))

WORKLOADS = {
    "cfg2": dict(
        desc="BASELINE cfg2: dense fp8 e4m3 GEMM M=N=K=8192 per GPU, A row-major, B column-major, "
             "per-tensor scales 1/64, fp32 accumulate, bf16 C, cta_group::2 256x256 MMAs, two "
             "per CTA pair and K step (two 128-row A sub-tiles per CTA share one B tile: "
             "512x256 pair tiles)",
        fmt="e4m3", M=8192, N=8192, K=8192, cta_group=2, tile_n=256, m_sub=2, alpha=1.0 / 4096.0,
        dist=1,
        dtype="e4m3"),
    "cfg3": dict(
        desc="BASELINE cfg3: 2:4 structured-sparse bf16 GEMM M=N=8192, K=16384 per GPU; 2 of "
             "every 4 K elements of A zeroed at seeded positions; compressed A and metadata from "
             "b2g_compress_24, metadata prepared once (static operand); B uniform[-1,1]; "
             "TFLOP/s counted at logical (dense-equivalent) 2MNK; cta_group::2 512x224 pair tiles "
             "(two 128-row A sub-tiles per CTA share one B tile)",
        fmt="bf16", sparse=True, M=8192, N=8192, K=16384, cta_group=2, tile_n=224, m_sub=2,
        alpha=1.0, dist=0, dtype="bf16"),
    "cfg4": dict(
        desc="BASELINE cfg4: block-scaled NVFP4 GEMM M=N=K=16384 per GPU; e2m1 operands, one "
             "ue4m3 scale per 16-element K block (e4m3(amax/6)), values normal(0,1) quantised "
             "per block; fp32 accumulate, bf16 C; kind::mxf4nvf4.block16, cta_group::2 "
             "512x224 pair tiles (two 128-row A sub-tiles per CTA share one B tile and its "
             "scale factors)",
        fmt="nvfp4", M=16384, N=16384, K=16384, cta_group=2, tile_n=224, m_sub=2, alpha=1.0, dist=1,
        dtype="e2m1"),
    "mxf8": dict(
        desc="OCP MXFP8 GEMM M=N=K=8192 per GPU (not a BASELINE config): e4m3 operands, one "
             "E8M0 scale per 32-element K block, values normal(0,1) quantised per block; fp32 "
             "accumulate, bf16 C; kind::mxf8f6f4.block_scale, cta_group::2 512x224 pair tiles",
        fmt="mxf8", M=8192, N=8192, K=8192, cta_group=2, tile_n=224, m_sub=2, alpha=1.0, dist=1,
        dtype="e4m3"),
    "mxf4": dict(
        desc="OCP MXFP4 GEMM M=N=K=16384 per GPU (not a BASELINE config): packed e2m1 operands, "
             "one E8M0 scale per 32-element K block, values normal(0,1) quantised per block; fp32 "
             "accumulate, bf16 C; kind::mxf4.block_scale.block32, cta_group::2 512x224 pair tiles",
        fmt="mxf4", M=16384, N=16384, K=16384, cta_group=2, tile_n=224, m_sub=2, alpha=1.0, dist=1,
        dtype="e2m1"),
    "cfg3_e4m3": dict(
        desc="2:4 structured-sparse fp8 e4m3 GEMM M=N=8192, K=16384 (cfg3's shape on "
             "kind::f8f6f4 .sp), normal(0,1) operands, scales 1/64, 2 of every 4 K elements of A "
             "zeroed at seeded positions; TFLOP/s at logical 2MNK; cta_group::2 512x224 pair tiles",
        fmt="e4m3", sparse=True, M=8192, N=8192, K=16384, cta_group=2, tile_n=224, m_sub=2,
        alpha=1.0 / 4096.0, dist=1, dtype="e4m3"),
    "cfg4_sparse": dict(
        desc="structured-sparse NVFP4 GEMM M=N=K=16384 per GPU (not a BASELINE config: cfg4's "
             "shape and values, A sparse 4:8 in pairs at seeded positions, kind::mxf4nvf4 block16 "
             ".sp): one ue4m3 scale per 32 K (the sparse MMA's scale block); TFLOP/s at logical "
             "2MNK; cta_group::2 512x192 pair tiles (two 128-row A sub-tiles per CTA)",
        fmt="nvfp4", sparse=True, M=16384, N=16384, K=16384, cta_group=2, tile_n=192, m_sub=2,
        alpha=1.0, dist=1, dtype="e2m1"),
    "cfg5": dict(
        desc="BASELINE cfg5: UMMA shape and pipeline sweep of the GEMM at M=N=K=8192: cta_group "
             "1/2 (tile M 128/256), tile N 64/128/224/256, SS vs TS operands, ring stages 2/4/deepest, "
             "bf16 (K slot 64), fp8 e4m3 (K slot 128), fp4 e2m1 on kind::f8f6f4 (K slot 128, "
             "packed in HBM, unpacked by the TMA) and as MXFP4 (K slot 256)",
        fmt="sweep", M=8192, N=8192, K=8192, cta_group=0, tile_n=0, alpha=1.0, dist=1,
        dtype="mixed"),
    "cfg1": dict(
        desc="BASELINE cfg1: dense bf16 GEMM M=N=K=4096 per GPU, A row-major, B column-major, "
             "uniform[-1,1] from seed 0 (A: rows [0, M), B: rows [2^20, 2^20 + N) of the seed-0 "
             "stream), fp32 accumulate, bf16 C",
        fmt="bf16", M=4096, N=4096, K=4096, cta_group=2, tile_n=192, alpha=1.0, dist=0,
        dtype="bf16", seed_a=0, seed_b=0, b_row0=1 << 20),
}
# operand seeds of the workloads that name none (cfg1 overrides them: "from seed 0")
SEED_A, SEED_B, SEED_PRUNE = 11, 22, 33


def seeds(wl):
    """(seed of A, seed of B, first generator row of B) of a workload."""
    return wl.get("seed_a", SEED_A), wl.get("seed_b", SEED_B), wl.get("b_row0", 0)
L2_FLUSH_BYTES = 256 << 20  # 2x the 126 MB L2


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--config", default="cfg2", choices=sorted(WORKLOADS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="target CPU time of the cpu_baseline sample")
    p.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    p.add_argument("--no-secondary", action="store_true",
                   help="skip the secondary targets and the sustained loop")
    p.add_argument("--sustained-seconds", type=float, default=2.0,
                   help="device time of the back-to-back loop of the headline GEMM (one GPU)")
    p.add_argument("--sweep-csv", default=None, help="cfg5: also write every sweep point to this CSV")
    p.add_argument("--shape", default=None,
                   help="MxNxK: run the configured workload at another size (profiling a "
                        "smaller case of the same kernel); the line's config says so")
    return p.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def measured_peaks():
    """(bf16 burst TF/s, bf16 sustained TF/s, HBM GB/s, "measured" | "fallback")."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        burst = float(d["bf16_tflops"])
        return (burst, float(d.get("bf16_tflops_sustained", burst)),
                float(d.get("hbm_gbs", 6650.0)), "measured")
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def ncu_traffic(cfg_name: str):
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", f"gemm_{cfg_name}_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self, gpus: int):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.strip()]
        os.unlink(self.out.name)
        sm, mx, reasons, pw = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                idx = int(r[0])
                if idx >= gpus:
                    continue
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                pw.append(float(r[3]))
                for name, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        # samples taken while the GPU was busy: power at least half the peak seen
        # (the sampler also records the idle lead-in and tail around the region)
        pmax = max(pw) if pw else 0.0
        busy = [c for c, p in zip(sm, pw) if p >= 0.5 * pmax] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm), "samples_under_load": len(busy),
                "power_w_max": pmax or None}


# ---------------------------------------------------------------------------- CPU leg
def cpu_gemm_rate(A_rows, B, alpha, seconds_target, threads):
    """Time the oracle FP32 GEMM on row slabs; returns (tflops, rows, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402  (test / baseline infrastructure only)

    K = B.shape[1]
    N = B.shape[0]
    rows = min(64, A_rows.shape[0])
    t0 = time.perf_counter()
    oracle.gemm(A_rows[:rows], B, alpha, threads)
    dt = time.perf_counter() - t0
    rate = 2.0 * rows * N * K / max(dt, 1e-6)
    want = int(seconds_target * rate / (2.0 * N * K))
    rows = max(64, min(A_rows.shape[0], want))
    t0 = time.perf_counter()
    oracle.gemm(A_rows[:rows], B, alpha, threads)
    dt = time.perf_counter() - t0
    return 2.0 * rows * N * K / dt / 1e12, rows, dt


# ---------------------------------------------------------------------------- reference arm
def run_reference(args, wl):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    if wl["fmt"] == "sweep":
        # the CPU GEMM has no tile shapes to sweep: time it on the sweep's e4m3 point
        wl = dict(WORKLOADS["cfg2"], desc=wl["desc"] + " (CPU arm: the e4m3 8192^3 GEMM)")
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np  # noqa: F401
    import oracle  # noqa: E402

    threads = host_cores()
    M, N, K = wl["M"], wl["N"], wl["K"]
    # operands of the workload from the oracle's own generator (bit-identical to the device's)
    seed_a, seed_b, b_row0 = seeds(wl)
    B = oracle.operand(wl["fmt"], N, K, seed_b, wl["dist"], b_row0)[1]
    # Per-step row slab: sized so that warmup + steps fit in about two minutes, but
    # at least 256 rows, so that every host thread gets a block of rows to work on
    # (thin slabs measure thread start-up instead of the GEMM).
    budget_s = 120.0
    probe_rows = 128
    prune = SEED_PRUNE if wl.get("sparse") else None
    Ap = oracle.operand(wl["fmt"], probe_rows, K, seed_a, wl["dist"], prune_seed=prune)[1]
    oracle.gemm(Ap[:16], B, wl["alpha"], threads)  # warm the threads and caches
    t0 = time.perf_counter()
    oracle.gemm(Ap, B, wl["alpha"], threads)
    rate = 2.0 * probe_rows * N * K / (time.perf_counter() - t0)
    per_step = budget_s / max(1, args.steps + args.warmup)
    rows = int(max(min(M, 256), min(M, per_step * rate / (2.0 * N * K))))
    A = oracle.operand(wl["fmt"], rows, K, seed_a, wl["dist"], prune_seed=prune)[1]
    for _ in range(args.warmup):
        oracle.gemm(A, B, wl["alpha"], threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.gemm(A, B, wl["alpha"], threads)
    dt = time.perf_counter() - t0
    flops = 2.0 * rows * N * K * args.steps
    tflops = flops / dt / 1e12
    sample = (f"{rows} rows of C ({rows}x{N}x{K} per step, of the {M}x{N}x{K} GEMM), "
              f"fp32 oracle GEMM over dequantised operands, {threads} threads")
    line = {
        "impl": "reference",
        "metric": "GEMM TFLOP/s (whole box)",
        "value": tflops,
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded generator of the oracle)",
        "config": {"workload": wl["desc"], "M": M, "N": N, "K": K, "sample_rows": rows},
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def peak_multiple(wl):
    """(multiple of the bf16 tensor peak that bounds this workload, why)."""
    sp, why_sp = ((2.0, "; 2:4 sparse MMA retires twice the dense-equivalent FLOPs per cycle")
                  if wl.get("sparse") else (1.0, ""))
    if wl["fmt"] in ("e4m3", "mxf8"):
        return 2.0 * sp, "fp8 issues at twice the bf16 rate per SM cycle" + why_sp
    if wl["fmt"] in ("nvfp4", "mxf4"):
        return 4.0 * sp, "e2m1 issues at four times the bf16 rate per SM cycle" + why_sp
    return sp, ("dense bf16" if sp == 1.0 else why_sp[2:])


def strong_rows(M: int, ws: int, rank: int, granule: int = 512):
    """Rows [row0, row0 + rows) of a global M-row problem that rank `rank` of `ws`
    owns under the strong split: equal shards of whole `granule`-row blocks (one
    512-row pair tile of two sub-tiles), the last shard taking what is left.  Every
    shard is padded to `per` rows for the all-gather of C.  Returns (row0, rows, per)."""
    per = -(-M // ws)
    per = -(-per // granule) * granule
    row0 = min(M, rank * per)
    return row0, min(M, row0 + per) - row0, per


class Problem:
    """One GEMM of a workload on this GPU: rows [a_row0, a_row0 + a_rows) of the
    global A (generated by counter, so a shard is the exact slice of the whole
    matrix), all of B, and C -- built on the device by libb2g's generator and
    quantisers."""

    def __init__(self, eng, dev, wl, a_row0, a_rows):
        import torch

        import b2g

        self.torch, self.eng, self.dev, self.wl = torch, eng, dev, wl
        self.fmt = fmt = wl["fmt"]
        self.code = {"bf16": b2g.FMT_BF16, "e4m3": b2g.FMT_E4M3, "nvfp4": b2g.FMT_NVFP4,
                     "mxf8": b2g.FMT_MXF8, "mxf4": b2g.FMT_MXF4}[fmt]
        self.scaled = fmt in ("nvfp4", "mxf8", "mxf4")  # operands carry scale factors
        self.packed4 = fmt in ("nvfp4", "mxf4")
        self.sparse = bool(wl.get("sparse"))
        # scale block: NVFP4 16 (32 for 4:8-sparse NVFP4, whose MMA reads four scales per
        # 128 dense K), MX 32
        self.sf_block = (32 if self.sparse else 16) if fmt == "nvfp4" else 32
        self.M, self.N, self.K = a_rows, wl["N"], wl["K"]
        self.a_row0 = a_row0
        self.sfs = {}
        seed_a, seed_b, b_row0 = seeds(wl)
        self.seed_a = seed_a
        M, K = self.M, self.K
        A = self.operand(M, K, seed_a, a_row0)
        kw = {}
        if self.sparse:  # 2:4-sparse A: bf16 (kind::f16) or e4m3 (kind::f8f6f4); NVFP4 4:8
            # in pairs (kind::mxf4nvf4): a byte of packed e2m1 is the unit
            eng.prune_24(A, SEED_PRUNE, row0=a_row0, fmt=self.code)
            pairs = self.packed4
            comp = torch.empty(M, K // 4 if pairs else K // 2, dtype=A.dtype, device=dev)
            meta = torch.empty(M, K // 64 if pairs else K // 32, dtype=torch.int32, device=dev)
            eng.compress_24(A, comp, meta, fmt=self.code)
            ready = torch.empty(eng.sparse_meta_bytes(M, K, fmt=self.code) // 4, dtype=torch.int32,
                                device=dev)
            eng.sparse_meta_prepare(meta, M, K, ready, fmt=self.code)
            eng.check()
            self.A_op, kw = comp, dict(sparse=1, meta=ready, meta_layout=1, K=K)
            self.meta = meta
        else:
            self.A_op = A
        self.A = A  # dense (for sparse: pruned) A, for checks and the dense comparison
        self.B = self.operand(self.N, K, seed_b, b_row0)
        if self.scaled:
            kw.update(sfa=self.sfs[A.data_ptr()], sfb=self.sfs[self.B.data_ptr()])
        self.C = torch.empty(M, self.N, dtype=torch.bfloat16, device=dev)
        self.kw = dict(alpha=wl["alpha"], cta_group=wl["cta_group"], tile_n=wl["tile_n"],
                       m_sub=wl.get("m_sub", 0), **kw)
        self.flops = 2.0 * M * self.N * K

    def operand(self, rows, cols, seed, row0):
        torch, eng = self.torch, self.eng
        x = torch.empty(rows, cols, dtype=torch.float32, device=self.dev)
        eng.fill(x, seed, self.wl["dist"], row0=row0)
        if self.scaled:
            q = torch.empty(rows, cols // 2 if self.packed4 else cols, dtype=torch.uint8,
                            device=self.dev)
            sf = torch.empty(rows, cols // self.sf_block, dtype=torch.uint8, device=self.dev)
            if self.fmt == "nvfp4":
                eng.quantize_nvfp4(x, q, sf, block=self.sf_block)
            else:
                eng.quantize(self.code, x, q, sf)
            self.sfs[q.data_ptr()] = sf
        else:
            q = torch.empty(rows, cols, dtype=torch.bfloat16 if self.fmt == "bf16" else torch.uint8,
                            device=self.dev)
            eng.quantize(self.code, x, q)
        del x
        return q

    def dequant(self, q, rows=None):
        """First `rows` rows of a stored operand -> fp64 values on the device
        (verification and the CPU-baseline operands only)."""
        torch = self.torch
        rows = q.shape[0] if rows is None else rows
        if self.fmt == "e4m3":
            return q[:rows].view(torch.float8_e4m3fn).double()
        if self.scaled:
            qr = q[:rows]
            if self.packed4:
                lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6],
                                   dtype=torch.float64, device=self.dev)
                v = torch.stack([lut[(qr & 15).long()], lut[(qr >> 4).long()]], dim=2).flatten(1)
            else:
                v = qr.view(torch.float8_e4m3fn).double()
            raw = self.sfs[q.data_ptr()][:rows]
            sc = (raw.view(torch.float8_e4m3fn).double() if self.fmt == "nvfp4"
                  else torch.pow(2.0, raw.double() - 127.0))  # ue4m3 / E8M0
            return v * sc.repeat_interleave(self.sf_block, dim=1)
        return q[:rows].double()

    def gemm(self):
        self.eng.gemm(self.A_op, self.B, self.C, self.code, **self.kw)

    def waves(self, max_clusters=0):
        """(tiles, clusters, waves) of the launch b2g_gemm plans for this problem."""
        import b2g

        opts = {k: v for k, v in self.kw.items()
                if k in ("cta_group", "tile_n", "m_sub", "meta_layout")}
        p = b2g.plan_gemm(self.code, self.M, self.N, self.K, sm_count=self.eng.sm_count,
                          max_clusters=max_clusters, sparse=1 if self.sparse else 0, **opts)
        tiles = p["num_m_tiles"] * p["num_n_tiles"]
        return tiles, p["clusters"], tiles / p["clusters"]

    def linearity(self, C=None, A=None, row_blocks=None):
        """Relative residual of C . x against alpha * A . (B^T . x), fp64, for a
        seeded x: a size-independent check of the whole product."""
        torch = self.torch
        x = torch.empty(1, self.N, dtype=torch.float32, device=self.dev)
        self.eng.fill(x, 99, 0)
        x = x[0].double()
        C = self.C if C is None else C
        A = self.A if A is None else A
        bx = self.dequant(self.B).t() @ x
        lhs = C.double() @ x
        rhs = self.wl["alpha"] * (self.dequant(A) @ bx)
        return float((lhs - rhs).norm() / rhs.norm())


def dense_tile(code, M, N, K, kw):
    """'tile_m x tile_n' of the launch b2g_gemm plans for these options (the pair's
    output tile: 128 rows x A sub-tiles x cta_group)."""
    import b2g

    opts = {k: v for k, v in kw.items()
            if k in ("cta_group", "tile_n", "m_sub", "meta_layout", "sparse")}
    pl = b2g.plan_gemm(code, M, N, K, **opts)
    return f"{pl['tile_m']}x{pl['tile_n']}"


def time_steps(run, steps, warmup, flush, stream):
    """Device time (ms) of each of `steps` calls of run() after `warmup` untimed
    ones, the L2 flushed (an untimed 256 MiB write) before every call; CUDA events
    on the launching stream."""
    import torch

    for _ in range(warmup):
        flush.zero_()
        run()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    torch.cuda.synchronize()
    for e0, e1 in ev:
        flush.zero_()
        e0.record(stream)
        run()
        e1.record(stream)
    torch.cuda.synchronize()
    return [e0.elapsed_time(e1) for e0, e1 in ev]


def max_over_ranks(x, ws, dev):
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# Secondary targets measured in the same run as the headline (BASELINE cfg1, cfg3,
# cfg4 and the north star's bf16 8192^3), each as its own short burst.
SECONDARY = {
    "bf16_8192": dict(
        desc="dense bf16 GEMM M=N=K=8192 (the north star's bf16 target size), uniform[-1,1], "
             "fp32 accumulate, bf16 C, cta_group::2, planner's tile",
        fmt="bf16", M=8192, N=8192, K=8192, cta_group=2, tile_n=0, alpha=1.0, dist=0, dtype="bf16"),
}
# selectable with --config as well (its own line, profiling of the same kernel)
WORKLOADS["bf16_8192"] = SECONDARY["bf16_8192"]


def run_secondary(args, eng, dev, ws, rank, flush, stream, peaks, main_config):
    """The other BASELINE targets, timed in this run: on one GPU bf16 8192^3, cfg1,
    cfg3 with its same-shape dense kernel, and cfg4; on N GPUs the strong split of
    cfg4 (one 16384^3 problem in M-row shards) with its all-gather timed apart."""
    import torch
    import torch.distributed as dist

    burst, sust = peaks
    steps = max(10, min(args.steps, 100))
    warm = max(3, min(args.warmup, 10))
    names = (["bf16_8192", "cfg1", "cfg3", "cfg3_e4m3", "cfg4", "cfg4_sparse"] if ws == 1
             else ["cfg4"])
    out = {}
    for name in names:
        if name == main_config and ws == 1:
            continue
        wl = SECONDARY.get(name) or WORKLOADS[name]
        M_glob = wl["M"]
        row0, rows, per = strong_rows(M_glob, ws, rank) if ws > 1 else (0, M_glob, M_glob)
        p = Problem(eng, dev, wl, row0, rows)
        ms = time_steps(p.gemm, steps, warm, flush, stream)
        eng.check()
        tot = max_over_ranks(sum(ms), ws, dev)
        mean = tot / steps
        flops = 2.0 * M_glob * wl["N"] * wl["K"]
        tf = flops / (mean * 1e-3) / 1e12
        mult, _ = peak_multiple(wl)
        tiles, clusters, waves = p.waves()
        e = {"workload": wl["desc"], "M": M_glob, "N": wl["N"], "K": wl["K"],
             "rows_per_gpu": rows, "steps": steps, "warmup": warm, "ms_per_step": mean,
             "tflops": tf, "peak_multiple": mult,
             "frac_of_burst": tf / ws / (mult * burst), "frac_of_sustained": tf / ws / (mult * sust),
             "tiles_per_gpu": tiles, "clusters": clusters, "waves_per_gpu": waves,
             "l2": "flushed before every step"}
        if ws > 1:
            e["split"] = (f"strong: one {M_glob}x{wl['N']}x{wl['K']} problem, M-row shards of "
                          f"{per} rows on {ws} GPUs, B replicated")
            # verification only, timed apart: all-gather of the padded C shards
            Cp = torch.zeros(per, wl["N"], dtype=torch.bfloat16, device=dev)
            Cp[:rows] = p.C
            Cg = torch.empty(ws * per, wl["N"], dtype=torch.bfloat16, device=dev)
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            dist.barrier()
            g0.record(stream)
            dist.all_gather_into_tensor(Cg, Cp)
            g1.record(stream)
            torch.cuda.synchronize()
            e["allgather_ms"] = max_over_ranks(g0.elapsed_time(g1), ws, dev)
            e["allgather_bytes"] = ws * per * wl["N"] * 2
            if rank == 0:
                x = torch.empty(1, wl["N"], dtype=torch.float32, device=dev)
                eng.fill(x, 99, 0)
                x = x[0].double()
                bx = p.dequant(p.B).t() @ x
                num = den = 0.0
                for r in range(ws):
                    r0, nr, _ = strong_rows(M_glob, ws, r)
                    if nr == 0:
                        continue
                    Ar = p.operand(nr, wl["K"], p.seed_a, r0)
                    if p.sparse:
                        eng.prune_24(Ar, SEED_PRUNE, row0=r0, fmt=p.code)
                    lhs = Cg[r * per:r * per + nr].double() @ x
                    rhs = wl["alpha"] * (p.dequant(Ar) @ bx)
                    num += float((lhs - rhs).norm() ** 2)
                    den += float(rhs.norm() ** 2)
                    del Ar
                e["linearity_residual"] = (num / den) ** 0.5
            del Cg, Cp
        else:
            e["linearity_residual"] = p.linearity()
        if p.sparse and p.scaled:
            # block-scaled: the dense kernel of the format on cfg4-style operands of the
            # same shape (its scale block differs from the sparse one): equal logical FLOPs
            del p
            torch.cuda.empty_cache()
            pd = Problem(eng, dev, WORKLOADS["cfg4"], 0, M_glob)
            dms = time_steps(pd.gemm, steps, warm, flush, stream)
            eng.check()
            dtf = flops / (max_over_ranks(sum(dms), ws, dev) / steps * 1e-3) / 1e12
            e["dense_same_shape_tflops"] = dtf
            e["sparse_over_dense"] = tf / dtf
            e["dense_kernel"] = "gemm_tn_kernel nvfp4 cta_group::2 512x224 (cfg4's dense kernel)"
            p = pd
        elif p.sparse:
            # the dense kernel on the pruned A, same shape: equal logical FLOPs
            dkw = dict(alpha=wl["alpha"], cta_group=2, tile_n=256)
            Cd = torch.empty_like(p.C)
            dms = time_steps(lambda: eng.gemm(p.A, p.B, Cd, p.code, **dkw), steps, warm, flush,
                             stream)
            eng.check()
            dtf = flops / (max_over_ranks(sum(dms), ws, dev) / steps * 1e-3) / 1e12
            e["dense_same_shape_tflops"] = dtf
            e["sparse_over_dense"] = tf / dtf
            e["dense_kernel"] = (f"gemm_tn_kernel {wl['fmt']} cta_group::2 "
                                 f"{dense_tile(p.code, p.M, p.N, p.K, dkw)} on the pruned A")
            # the two kernels step by step in alternation, so that both run in the same
            # power state (the bursts above run one after the other, and under the 1 kW
            # cap the later one can meet a lower clock)
            sp_ms, de_ms = [], []
            for _ in range(steps):
                sp_ms += time_steps(p.gemm, 1, 0, flush, stream)
                de_ms += time_steps(lambda: eng.gemm(p.A, p.B, Cd, p.code, **dkw), 1, 0, flush,
                                    stream)
            eng.check()
            sp_t, de_t = max_over_ranks(sum(sp_ms), ws, dev), max_over_ranks(sum(de_ms), ws, dev)
            e["sparse_over_dense_interleaved"] = de_t / sp_t
            e["interleaved_steps"] = steps
            del Cd
        out[name] = e
        del p
        torch.cuda.empty_cache()
    if ws == 1:
        out["cublas_fp8_same_box"] = library_fp8(eng, dev, flush, stream, steps, warm)
    return out


def library_fp8(eng, dev, flush, stream, steps, warm):
    """The vendor library on the same box, for comparison only (never the reported
    value): cuBLASLt's fp8 e4m3 GEMM through torch._scaled_mm at the headline's
    8192^3 on the same seeded operands and per-tensor scales, L2 flushed between
    steps like every other entry.  Returns its TFLOP/s, or why it is unavailable."""
    import torch

    wl = WORKLOADS["cfg2"]
    try:
        p = Problem(eng, dev, wl, 0, wl["M"])
        a = p.A.view(torch.float8_e4m3fn)
        b = p.B.view(torch.float8_e4m3fn).t()  # [K][N] column-major: B as stored
        sa = torch.tensor(1.0 / 64, dtype=torch.float32, device=dev)
        sb = torch.tensor(1.0 / 64, dtype=torch.float32, device=dev)
        out = torch.empty(wl["M"], wl["N"], dtype=torch.bfloat16, device=dev)

        def run():
            torch._scaled_mm(a, b, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16, out=out)

        ms = time_steps(run, steps, warm, flush, stream)
        tf = p.flops / (sum(ms) / steps * 1e-3) / 1e12
        # same values as the engine's C (fp32 accumulate of the same products)
        p.gemm()
        torch.cuda.synchronize()
        rel = float((out.float() - p.C.float()).norm() / p.C.float().norm())
        del p
        torch.cuda.empty_cache()
        return {"workload": "cuBLASLt fp8 e4m3 GEMM (torch._scaled_mm) on cfg2's operands, "
                            "per-tensor scales 1/64, bf16 out", "steps": steps,
                "ms_per_step": sum(ms) / steps, "tflops": tf,
                "rel_diff_vs_engine_C": rel, "l2": "flushed before every step"}
    except Exception as ex:  # a library or torch build without the fp8 path
        return {"unavailable": f"{type(ex).__name__}: {ex}"[:200]}


def run_sustained(args, p, flush, stream, seconds, peaks):
    """The headline GEMM back to back for at least `seconds` of device time (L2
    flushed between steps), with its own clock samples: the power-capped figure
    beside the short burst of the headline."""
    import torch

    burst, sust = peaks
    ms = time_steps(p.gemm, 3, 3, flush, stream)
    n = int(seconds * 1e3 / max(1e-3, statistics.median(ms))) + 1
    sampler = ClockSampler()
    sampler.start()
    time.sleep(0.3)
    ms = time_steps(p.gemm, n, 0, flush, stream)
    clocks = sampler.stop(1)
    p.eng.check()
    mean = sum(ms) / n
    tf = p.flops / (mean * 1e-3) / 1e12
    mult, _ = peak_multiple(p.wl)
    return {"steps": n, "seconds": sum(ms) / 1e3, "ms_per_step": mean, "tflops": tf,
            "frac_of_sustained": tf / (mult * sust), "frac_of_burst": tf / (mult * burst),
            "clocks": clocks, "l2": "flushed before every step"}


# ---------------------------------------------------------------------------- our arm
def run_ours(args, wl):
    import torch
    import torch.distributed as dist

    import b2g

    ws, rank, local = dist_env()
    if ws != args.gpus:
        print(f"warning: WORLD_SIZE={ws} but --gpus {args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    eng = b2g.Engine(local)
    M, N, K = wl["M"], wl["N"], wl["K"]
    # M-row shard `rank` of the global (ws*M) x K matrix A (weak split); B replicated
    p = Problem(eng, dev, wl, rank * M, M)
    fmt, FMT, sparse, nvfp4 = p.fmt, p.code, p.sparse, p.scaled
    A_op, A, B, C, kw = p.A_op, p.A, p.B, p.C, p.kw
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    for _ in range(args.warmup):
        flush.zero_()
        p.gemm()
    eng.check()

    # ---- timed region: exactly K GEMMs, L2 flushed (untimed) before each
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler() if rank == 0 else None
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        p.gemm()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    clocks = sampler.stop(ws) if sampler else None
    eng.check()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(sum(step_ms), ws, dev)
    flops_step = p.flops
    value = ws * flops_step * args.steps / (total_ms * 1e-3) / 1e12
    mean_ms = total_ms / args.steps
    achieved = flops_step / (mean_ms * 1e-3) / 1e12

    # ---- sparse only: the dense kernel on the pruned A, same shape (equal logical FLOPs)
    dense_cmp = None
    if sparse and nvfp4:
        # block-scaled: the format's dense kernel on cfg4-style operands of the same shape
        # (the sparse scale block differs from the dense one)
        pd = Problem(eng, dev, dict(WORKLOADS["cfg4"], M=M, N=N, K=K), 0, M)
        n_d = max(3, args.steps // 4)
        d_ms = time_steps(pd.gemm, n_d, 3, flush, stream)
        eng.check()
        dense_tf = flops_step / (sum(d_ms) / n_d * 1e-3) / 1e12
        dense_cmp = {"dense_tflops_same_shape": dense_tf, "dense_steps": n_d,
                     "sparse_over_dense": achieved / dense_tf,
                     "dense_kernel": "gemm_tn_kernel nvfp4 cta_group::2 (cfg4's dense kernel)"}
        del pd
        torch.cuda.empty_cache()
    elif sparse:
        dkw = dict(alpha=wl["alpha"], cta_group=2, tile_n=256)
        n_d = max(3, args.steps // 4)
        d_ms = time_steps(lambda: eng.gemm(A, B, C, FMT, **dkw), n_d, 3, flush, stream)
        dense_ms = sum(d_ms) / n_d
        dense_tf = flops_step / (dense_ms * 1e-3) / 1e12
        dense_cmp = {"dense_tflops_same_shape": dense_tf, "dense_steps": n_d,
                     "sparse_over_dense": achieved / dense_tf,
                     "dense_kernel": "gemm_tn_kernel bf16 cta_group::2 "
                                     f"{dense_tile(FMT, M, N, K, dkw)} on the pruned A"}
        p.gemm()  # restore the sparse result for verification

    # ---- end to end through b2g_gemm_host: pinned host A/B/C, copies inside the timed region
    hA = A_op.cpu().pin_memory()
    hB = B.cpu().pin_memory()
    hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    hkw = dict(kw)
    if not sparse and not nvfp4:
        # dense: each block of C (a quarter of the rows and columns) takes the planner's
        # sub-tile choice; the whole-problem tile of two A sub-tiles would leave half the
        # clusters of a block's launch idle
        hkw["m_sub"] = 0
    if sparse:
        hkw["meta"] = kw["meta"].cpu().pin_memory()
    if nvfp4:
        hkw["sfa"] = kw["sfa"].cpu().pin_memory()
        hkw["sfb"] = kw["sfb"].cpu().pin_memory()
    h2d = [hA, hB] + ([hkw["meta"]] if sparse else []) + ([hkw["sfa"], hkw["sfb"]] if nvfp4 else [])
    h2d_bytes = sum(t.numel() * t.element_size() for t in h2d)
    for _ in range(2):
        eng.gemm_host(hA, hB, hC, FMT, **hkw)
    e_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.e2e_steps)]
    e_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.e2e_steps)]
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.e2e_steps):
        e_s[i].record(stream)
        eng.gemm_host(hA, hB, hC, FMT, **hkw)
        e_e[i].record(stream)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e2e_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(e_s, e_e)), ws, dev)
    e2e_value = ws * flops_step * args.e2e_steps / (e2e_ms * 1e-3) / 1e12
    e2e_match = bool(torch.equal(hC.to(dev), C))
    # split tails change the fp32 summation order of the device run only
    e2e_rel = float(((hC.to(dev).float() - C.float()).norm() / C.float().norm().clamp_min(1e-30)).item())
    del hA, hB, hC, hkw

    # ---- verification: all-gather of C over NCCL (timed separately), linearity check
    gather_ms = None
    verify = None
    if ws > 1:
        Cg = torch.empty(ws * M, N, dtype=torch.bfloat16, device=dev)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        g0.record(stream)
        dist.all_gather_into_tensor(Cg, C)
        g1.record(stream)
        torch.cuda.synchronize()
        gather_ms = g0.elapsed_time(g1)
        if rank == 0:
            x = torch.empty(1, N, dtype=torch.float32, device=dev)
            eng.fill(x, 99, 0)
            x = x[0].double()
            bx = p.dequant(B).t() @ x
            num = den = 0.0
            for r in range(ws):  # every shard's slice of the gathered C
                Ar = p.operand(M, K, p.seed_a, r * M)
                if sparse:
                    eng.prune_24(Ar, SEED_PRUNE, row0=r * M, fmt=p.code)
                lhs = Cg[r * M:(r + 1) * M].double() @ x
                rhs = wl["alpha"] * (p.dequant(Ar) @ bx)
                num += float((lhs - rhs).norm() ** 2)
                den += float(rhs.norm() ** 2)
                del Ar
            verify = (num / den) ** 0.5
        del Cg
    elif rank == 0:
        verify = p.linearity()

    # ---- CPU baseline (rank 0, N = 1 only): the oracle GEMM on a row slab
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        threads = host_cores()
        Bh = p.dequant(B).float().cpu().numpy()
        Ah = p.dequant(A, min(M, 4096)).float().cpu().numpy()
        tf, rows, secs = cpu_gemm_rate(Ah, Bh, wl["alpha"], args.cpu_seconds, threads)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{rows} rows of C ({rows}x{N}x{K}, {secs:.1f} s) of the {M}x{N}x{K} "
                         f"GEMM, fp32 oracle GEMM over the dequantised operands"}
        del Bh, Ah

    burst_bf16, sust_bf16, _, peak_kind = measured_peaks()
    # ---- the other targets of the north star, each a short burst in this run (before
    # the sustained loop, whose power-capped clocks would carry over into them)
    secondary = None
    if not args.no_secondary:
        secondary = run_secondary(args, eng, dev, ws, rank, flush, stream,
                                  (burst_bf16, sust_bf16), args.config)
    # ---- the headline GEMM for >= 2 s back to back (one GPU): the power-capped figure
    sustained = None
    if ws == 1 and not args.no_secondary and args.sustained_seconds > 0:
        sustained = run_sustained(args, p, flush, stream, args.sustained_seconds,
                                  (burst_bf16, sust_bf16))

    if ws > 1:
        dist.barrier()
    if rank == 0:
        # Power-capped run (SM clock under load below max with sw_power_cap active):
        # the denominator is the sustained cuBLAS figure, else the burst one.
        capped = bool(clocks and "sw_power_cap" in clocks["reasons"]
                      and clocks["sm_mhz"] < 0.95 * clocks["sm_max_mhz"])
        bf16_peak = sust_bf16 if capped else burst_bf16
        which = "sustained (power-capped run)" if capped else "burst"
        mult, why = peak_multiple(wl)
        peak = mult * bf16_peak
        peak_note = (f"{mult:g} x {peak_kind} cuBLAS bf16 {which} {bf16_peak:.0f} TF/s ({why}: "
                     f"the multiple is the per-SM-cycle issue ratio the reference measures, "
                     f"umma_throughput/tput_results_max.csv; no fp8 or fp4 peak is measured on "
                     f"this pool); of {peak_kind}")
        # (the committed traffic figures are for the configurations' own sizes)
        traffic = None if args.shape else ncu_traffic(args.config)
        line = {
            "metric": "GEMM TFLOP/s (whole box)",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": mean_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": wl["dtype"],
            "data": "synthetic (seeded on-device generator, bit-identical to the CPU oracle's)",
            "config": {"workload": wl["desc"], "M_per_gpu": M, "N": N, "K": K,
                       "cta_group": wl["cta_group"],
                       "tile": dense_tile(p.code, M, N, K, p.kw),
                       "l2": "flushed (256 MiB write, untimed) before every timed step",
                       "parallelism": f"M-row shards x{ws}, B replicated, no data-path collective"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                         "peak_source": peak_note,
                         "frac_of_burst": achieved / (mult * burst_bf16),
                         "frac_of_sustained": achieved / (mult * sust_bf16),
                         "algorithmic_flops_per_launch": flops_step},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d_bytes,
                    "d2h_bytes_per_step": M * N * 2, "steps": args.e2e_steps,
                    "ms_per_step": e2e_ms / args.e2e_steps, "matches_device_C": e2e_match,
                    "rel_diff_vs_device_C": e2e_rel,
                    "api": "b2g_gemm_host (C ABI, pinned host buffers)"},
            "sparse_vs_dense": dense_cmp,
            "gpu_launches": args.steps,
            "clocks": clocks,
            "verify": {"linearity_residual": verify, "allgather_ms": gather_ms},
            "sustained": sustained,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if ws > 1:
        dist.destroy_process_group()
    return 0


def run_sweep(args, wl):
    """BASELINE cfg5 on one GPU: every point is the full 8192^3 GEMM, timed by CUDA
    events over `--steps` launches (L2 flushed before each) after `--warmup`; the
    JSON line carries every point, the value is the best point."""
    import torch

    import b2g

    ws, rank, local = dist_env()
    if rank != 0:
        return 0  # one-GPU sweep: the other ranks of a torchrun launch have no work
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    eng = b2g.Engine(local)
    S = wl["M"]
    steps, warm = max(1, min(args.steps, 20)), max(3, min(args.warmup, 5))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    C = torch.empty(S, S, dtype=torch.bfloat16, device=dev)

    def operand(fmt, seed):
        x = torch.empty(S, S, dtype=torch.float32, device=dev)
        eng.fill(x, seed, 0 if fmt == "bf16" else 1)
        if fmt == "bf16":
            q = torch.empty(S, S, dtype=torch.bfloat16, device=dev)
            eng.quantize(b2g.FMT_BF16, x, q)
            return q, None
        if fmt == "e4m3":
            q = torch.empty(S, S, dtype=torch.uint8, device=dev)
            eng.quantize(b2g.FMT_E4M3, x, q)
            return q, None
        if fmt == "e2m1":  # packed two per byte, unpacked by the TMA for kind::f8f6f4
            q = torch.empty(S, S // 2, dtype=torch.uint8, device=dev)
            eng.quantize(b2g.FMT_E2M1, x, q)
            return q, None
        q = torch.empty(S, S // 2, dtype=torch.uint8, device=dev)
        sf = torch.empty(S, S // 32, dtype=torch.uint8, device=dev)
        eng.quantize(b2g.FMT_MXF4, x, q, sf)
        return q, sf

    formats = (("bf16", b2g.FMT_BF16, 64, "kind::f16", 1.0),
               ("e4m3", b2g.FMT_E4M3, 128, "kind::f8f6f4", 1.0 / 4096.0),
               ("e2m1", b2g.FMT_E2M1, 128, "kind::f8f6f4 (e2m1, no scales)", 1.0),
               ("mxf4", b2g.FMT_MXF4, 256, "kind::mxf4.block_scale.block32 (MXFP4)", 1.0))
    points = []
    for name, fmt, kslot, kind, alpha in formats:
        (A, sfa), (B, sfb) = operand(name, 11), operand(name, 22)
        extra = dict(sfa=sfa, sfb=sfb) if sfa is not None else {}
        for cg in (1, 2):
            for tn in (64, 128, 224, 256):  # 224: the widest tile with TMEM for TS / scales
                for ab in ((0, 1) if name in ("bf16", "e4m3") else (0,)):
                    for stages in (2, 4, 0):
                        p = {"format": name, "instruction": kind, "cta_group": cg,
                             "tile_m": 128 * cg, "tile_n": tn, "k_slot": kslot,
                             "ab": "TS" if ab else "SS", "stages": stages or "deepest"}
                        kw = dict(alpha=alpha, cta_group=cg, tile_n=tn, ab_mode=ab, stages=stages,
                                  **extra)
                        try:  # the pair's output tile as planned (A sub-tiles per CTA included)
                            pl = b2g.plan_gemm(fmt, S, S, S, cta_group=cg, tile_n=tn, ab_mode=ab,
                                               stages=stages)
                            p["tile_m"], p["m_sub"] = pl["tile_m"], pl["m_sub"]
                        except b2g.B2GError:
                            pass
                        try:
                            for _ in range(warm):
                                flush.zero_()
                                eng.gemm(A, B, C, fmt, **kw)
                            eng.check()
                            ev = [(torch.cuda.Event(enable_timing=True),
                                   torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
                            for e0, e1 in ev:
                                flush.zero_()
                                e0.record()
                                eng.gemm(A, B, C, fmt, **kw)
                                e1.record()
                            torch.cuda.synchronize()
                            eng.check()
                            ms = statistics.median([e0.elapsed_time(e1) for e0, e1 in ev])
                            p["ms"] = ms
                            p["tflops"] = 2.0 * S ** 3 / (ms * 1e-3) / 1e12
                        except b2g.B2GError as e:
                            p["unsupported"] = str(e).split(": ", 1)[-1][:120]
                        points.append(p)
        del A, B
    if args.sweep_csv:
        import csv

        keys = ["format", "instruction", "cta_group", "tile_m", "m_sub", "tile_n", "k_slot", "ab",
                "stages",
                "ms", "tflops", "unsupported"]
        with open(args.sweep_csv, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=keys)
            w.writeheader()
            for p in points:
                w.writerow({k: p.get(k, "") for k in keys})
    ok = [p for p in points if "tflops" in p]
    best = max(ok, key=lambda p: p["tflops"])
    print(json.dumps({
        "metric": "GEMM TFLOP/s over the UMMA shape / pipeline sweep (best point)",
        "value": best["tflops"], "unit": "TFLOP/s", "n_gpus": 1, "steps": steps, "warmup": warm,
        "ms_per_step": best["ms"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "mixed",
        "data": "synthetic (seeded on-device generator, bit-identical to the CPU oracle's)",
        "config": {"workload": wl["desc"], "M": S, "N": S, "K": S,
                   "l2": "flushed (256 MiB write, untimed) before every timed launch",
                   "best": {k: best.get(k) for k in ("format", "cta_group", "tile_m", "tile_n", "ab",
                                                     "stages")}},
        "points": points, "gpu_launches": steps * len(ok),
    }), flush=True)
    eng.close()
    return 0


def main():
    args = parse()
    wl = WORKLOADS[args.config]
    if args.shape:
        M, N, K = (int(v) for v in args.shape.lower().split("x"))
        wl = dict(wl, M=M, N=N, K=K,
                  desc=wl["desc"] + f" -- run at M={M}, N={N}, K={K} (--shape)")
    if args.config == "cfg5" and args.impl != "reference":
        return run_sweep(args, wl)
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_ours(args, wl)


if __name__ == "__main__":
    sys.exit(main())
