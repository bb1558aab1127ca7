"""CPU tests of the boundary: the C-ABI library loads, exports every symbol include/*.h declares,
and its host-side argument handling answers without a GPU. No kernel is launched."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from xspmm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    declared = _lib.declared_symbols()
    assert len(declared) >= 38
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert getattr(L, s) is not None


def test_status_strings():
    L = _lib.lib()
    assert L.xspmm_status_string(0) == b"ok"
    assert L.xspmm_status_string(2) == b"unsupported"


def test_null_handle_is_rejected_without_a_gpu():
    L = _lib.lib()
    rc = L.xspmm_bcsr_spmm_f16f32_i32(None, 1, 1, 1, 16, 16, None, None, None, None, None, 16,
                                      16, 8, None)
    assert rc == 1  # INVALID_ARGUMENT
    assert b"null handle" in L.xspmm_last_error()
    c = ctypes.c_uint64()
    assert L.xspmm_get_launch_count(None, ctypes.byref(c)) == 1


def test_plan_entry_points_reject_null_arguments_without_a_gpu():
    L = _lib.lib()
    plan = ctypes.c_void_p(123)
    rc = L.xspmm_plan_csr_f16f32_i32(None, 16, 16, 0, None, None, None, 16, 1,
                                     ctypes.byref(plan), None)
    assert rc == 1 and plan.value is None  # output cleared before the handle is checked
    assert L.xspmm_plan_bcsr_f32f32_i64(None, 1, 1, 0, 16, 16, None, None, None, 16, 16,
                                        None) == 1
    assert L.xspmm_plan_execute(None, None, None, 8) == 1
    assert b"null plan" in L.xspmm_last_error()
    info = _lib.PlanInfo()
    assert L.xspmm_plan_get_info(None, ctypes.byref(info)) == 1
    assert L.xspmm_plan_destroy(None) == 0  # destroying nothing is a no-op
    assert ctypes.sizeof(_lib.PlanInfo) == 72


def test_create_reports_a_status_instead_of_crashing():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present: creation is covered by the GPU tests")
    L = _lib.lib()
    h = ctypes.c_void_p()
    rc = L.xspmm_create(0, None, ctypes.byref(h))
    assert rc in (1, 3)  # no device: invalid ordinal or CUDA error


def test_cpp_api_header_compiles_against_the_abi():
    """include/xspmm/xspmm.hpp (the reference-shaped C++ API) compiles with the host compiler."""
    src = os.path.join(ROOT, "tests", "cpp", "pipeline_example.cpp")
    if not os.path.exists(src):
        pytest.skip("no C++ compile check source")
    cuda_inc = "/usr/local/cuda/include"
    r = subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-I" + os.path.join(ROOT, "include"),
                        "-I" + cuda_inc, src], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


_ALL_TYPES_SRC = r"""
#include "xspmm/xspmm.hpp"
#include "xspmm/clustering.hpp"
#include "xspmm/plan.hpp"
#include "xspmm/dist.hpp"
template <typename V, typename I>
void use(std::shared_ptr<const xspmm::Executor> exec, const xspmm::DistComm& comm, V* B, float* C) {
    xspmm::CSRMatrix<V, I> A(exec, 4, 4, 1);
    xspmm::SpMMTimings t;
    xspmm::spmm(exec, A, B, C, I(8), I(8), true, &t);
    auto Ab = xspmm::csr_to_bcsr(exec, A, I(3), I(5));
    xspmm::spmm(Ab, B, C, I(8));
    I* perm = nullptr;
    xspmm::compute_1d_jaccard_clustering(exec, A, 0.5f, I(16), perm);
    auto Ap = xspmm::apply_permutation(exec, A, perm);
    xspmm::unpermute_dense_matrix(exec, B, B, perm, I(4), I(8));
    xspmm::SpMMPlan<V, I> plan(exec, A, I(16), true, &t);
    xspmm::DistPlan<V, I> dp(comm, exec, A, I(16), true);
}
template void use<__half, int32_t>(std::shared_ptr<const xspmm::Executor>, const xspmm::DistComm&, __half*, float*);
template void use<__half, int64_t>(std::shared_ptr<const xspmm::Executor>, const xspmm::DistComm&, __half*, float*);
template void use<__nv_bfloat16, int32_t>(std::shared_ptr<const xspmm::Executor>, const xspmm::DistComm&, __nv_bfloat16*, float*);
template void use<__nv_bfloat16, int64_t>(std::shared_ptr<const xspmm::Executor>, const xspmm::DistComm&, __nv_bfloat16*, float*);
template void use<float, int32_t>(std::shared_ptr<const xspmm::Executor>, const xspmm::DistComm&, float*, float*);
template void use<float, int64_t>(std::shared_ptr<const xspmm::Executor>, const xspmm::DistComm&, float*, float*);
"""


def test_cpp_api_instantiates_every_value_and_index_type(tmp_path):
    """Every C++ entry (Tier 1 on any block shape, Tier 2, clustering, permutation, unpermute,
    plans, distributed plans) compiles for fp16, bf16 and fp32 values with int32 and int64
    indices, i.e. each maps onto a declared C entry point."""
    src = tmp_path / "all_types.cpp"
    src.write_text(_ALL_TYPES_SRC)
    r = subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-I" + os.path.join(ROOT, "include"),
                        "-I/usr/local/cuda/include", str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
