"""Extract the reference's published TMA 2D load latencies used as golden values by
tests/test_zperf_drivers_gpu.py, from the reference's committed result CSV
tma2d_latency/tma2d_lat_results.csv (one row per box height at width 128, one CTA
per SM).

    python tests/golden/make_tma2d_lat_golden.py /path/to/reference
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


def main(ref):
    rows = list(csv.DictReader(open(os.path.join(ref, "tma2d_latency", "tma2d_lat_results.csv"))))
    out = os.path.join(HERE, "tma2d_lat_reference_rows.csv")
    with open(out, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=rows[0].keys())
        w.writeheader()
        for r in rows:
            w.writerow(r)
    print(f"{len(rows)} rows -> {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else reference_dir())
