"""Extract the reference's published tcgen05 issue rates used as golden values
by tests/test_zperf_drivers_gpu.py, from the reference's committed result CSV
umma_throughput/tput_results_max.csv (one row per format, layout, cta_group, M,
N at the largest pipeline depth).

    python tests/golden/make_umma_golden.py /path/to/reference
"""
import csv
import os
import sys


def reference_dir() -> str:
    """The reference checkout: $REFERENCE_DIR, else `reference` beside this repository."""
    here = os.path.dirname(os.path.abspath(__file__))
    return os.environ.get("REFERENCE_DIR",
                          os.path.abspath(os.path.join(here, "..", "..", "..", "reference")))


HERE = os.path.dirname(os.path.abspath(__file__))
KEEP = {("BF16", "SS", "1", "128", "256"), ("BF16", "SS", "2", "256", "256"),
        ("BF16", "TS", "1", "128", "256"), ("BF16", "SS", "1", "128", "128"),
        ("E4M3", "SS", "2", "256", "256"), ("E4M3", "SS", "1", "128", "256"),
        ("S8", "SS", "1", "128", "256"), ("F4", "SS", "2", "256", "256"),
        ("MXF8", "SS", "2", "256", "256"), ("MXF4", "SS", "2", "256", "256"),
        ("BF16", "SS", "1", "64", "128"), ("BF16", "SS", "2", "128", "128")}


def main(ref):
    rows = list(csv.DictReader(open(os.path.join(ref, "umma_throughput", "tput_results_max.csv"))))
    best = {}
    for r in rows:
        key = (r["Format"], r["ABLayout"], r["CTAGroup"], r["M"], r["N"])
        if key in KEEP:
            if key not in best or int(r["PipelineDepth"]) > int(best[key]["PipelineDepth"]):
                best[key] = r
    out = os.path.join(HERE, "umma_tput_reference_rows.csv")
    with open(out, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=rows[0].keys())
        w.writeheader()
        for k in sorted(best):
            w.writerow(best[k])
    print(f"{len(best)} rows -> {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else reference_dir())
