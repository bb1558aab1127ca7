"""xspmm_b200 -- B200-native (sm_100a) xSpMM hot path.

Tier-1 BCSR 16x16 block SpMM on tensor cores and the Tier-2 pipeline around it (exact greedy
Jaccard row clustering, CSR row permutation, CSR->BCSR conversion, unpermute), all on the device,
behind the C ABI in include/xspmm_b200.h (libxspmm_b200.so). This package is the Python view of
that ABI, mirroring the reference's API names.
"""
from .api import (  # noqa: F401
    BCSRMatrix,
    CSRMatrix,
    CudaExecutor,
    SpMMPlan,
    SpMMTimings,
    apply_permutation,
    compute_1d_jaccard_clustering,
    csr_to_bcsr,
    spmm,
    unpermute_dense_matrix,
)
from ._lib import XSpMMError, lib  # noqa: F401
