"""Generate tests/golden/idesc_reference.json from the reference's OWN descriptor
encoders, compiled from their sources where they lie by `make -C oracle ref`
(oracle/ref_idesc_umma.cu, oracle/ref_idesc_sparse.cu -> oracle/_ref/).

    make -C oracle ref && python tests/golden/make_idesc_golden.py

Each record is what the reference's make_i_desc emits for one configuration:
umma_throughput/umma_tput.cu:190-255 (per MMA_FORMAT, MMA_M, MMA_N) and
tcgen05_sparse_mma/tcgen05_sparse_mma.cu:191-228 (per KIND_ID, type codes,
SPARSITY, MMA_M, MMA_N, SCALE_TYPE_ID).
"""
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "..", "..", "oracle", "_ref", "idesc_reference.txt")


def main():
    umma, sparse = [], []
    with open(SRC) as f:
        for line in f:
            p = line.split()
            if p[0] == "umma":
                umma.append({"format": int(p[1]), "M": int(p[2]), "N": int(p[3]),
                             "idesc": int(p[4], 16)})
            elif p[0] == "sparse":
                sparse.append({"kind": int(p[1]), "a_type": int(p[2]), "b_type": int(p[3]),
                               "sparse": int(p[4]), "M": int(p[5]), "N": int(p[6]),
                               "scale_type": int(p[7]), "idesc": int(p[8], 16)})
    out = {"source": "reference make_i_desc compiled from umma_throughput/umma_tput.cu and "
                     "tcgen05_sparse_mma/tcgen05_sparse_mma.cu by `make -C oracle ref`",
           "umma": umma, "sparse": sparse}
    with open(os.path.join(HERE, "idesc_reference.json"), "w") as f:
        json.dump(out, f, indent=0)
    print(f"{len(umma)} umma + {len(sparse)} sparse records")


if __name__ == "__main__":
    main()
