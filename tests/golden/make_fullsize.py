"""Digests of the full-size permutation and BCSR structure, for the GPU parity tests at the sizes
the oracle cannot run inside a test (python tests/golden/make_fullsize.py; minutes on 8 cores).

For the banded (2,000,000 rows) and R-MAT (2^20 rows) configs, the fast exact clustering of the
oracle (oracle.cluster_fast, pinned to the compiled reference's loop at 2^13-2^15 rows in
tests/test_oracle.py) gives the permutation, and the oracle's CSR->BCSR (pinned the same way) the
permuted matrix's block structure. The file keeps their SHA-256 digests (int32 little-endian
arrays) so that a test compares the GPU's outputs bit for bit without shipping the arrays."""
import hashlib
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from xspmm_b200 import synth  # noqa: E402


def digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<i4").tobytes()).hexdigest()


def main():
    out = {}
    for name, make in (("cfg4_banded_2M", lambda: synth.cfg4_banded(N=8)),
                       ("cfg5_rmat_2^20", lambda: synth.cfg5_rmat(N=8))):
        t0 = time.time()
        P = make()
        perm = oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K)
        prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values, perm)
        brp, bci, _ = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
        out[name] = {"M": P.M, "K": P.K, "nnz": P.nnz, "nnzb": int(brp[-1]),
                     "perm_sha256": digest(perm), "bcsr_row_ptr_sha256": digest(brp),
                     "bcsr_col_ind_sha256": digest(bci),
                     "source": "oracle.cluster_fast + oracle.permute_rows + oracle.csr_to_bcsr"}
        print(name, f"{time.time() - t0:.0f} s", out[name], flush=True)
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "fullsize.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
