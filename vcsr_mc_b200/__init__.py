"""B200-native VCSR-MC SpMM: C (+)= A * B with A sparse (CSR -> VCSR-MC), B and C dense.

The compute path is libvcsrmc.so (hand-written sm_100a CUDA + host C++), bound through the
C ABI in include/vcsrmc.h. This package is the Python mirror of the reference's host
interface; see vcsr_mc_b200.api.
"""
from ._lib import F16, F32, PLAN_AUTO, PLAN_BAND, PLAN_HYBRID, PLAN_ROWS, PLAN_SEGMENT, GEN_RMAT, GEN_STENCIL27, GEN_STENCIL27_LINKS, GEN_UNIFORM_POISSON, GEN_ZIPF, VcsrmcError, lib
from .api import (CSR, VCSRMC, DeviceVCSRMC, apply_column_permutation, build_vcsr_mc_device, coo_to_csr, csr_to_vcsr_mc,
                  destroy_vcsr_mc_device, gen_dense_device, gen_dense_host, half_scale, load_csr, partition_rows,
                  SHARD_ROW_WEIGHT, rcm_column_order, read_matrix_market, run_vcsr_mc_spmm_gpu, spmm, upload_vcsr_mc_device)

__all__ = [
    "CSR", "VCSRMC", "DeviceVCSRMC", "VcsrmcError", "build_vcsr_mc_device", "F16", "F32", "PLAN_AUTO", "PLAN_BAND", "PLAN_HYBRID", "PLAN_ROWS", "PLAN_SEGMENT", "GEN_RMAT", "GEN_STENCIL27", "GEN_STENCIL27_LINKS",
    "GEN_UNIFORM_POISSON", "GEN_ZIPF", "apply_column_permutation", "coo_to_csr", "csr_to_vcsr_mc",
    "destroy_vcsr_mc_device", "gen_dense_device", "gen_dense_host", "half_scale", "lib", "load_csr", "partition_rows",
    "SHARD_ROW_WEIGHT",
    "rcm_column_order", "read_matrix_market", "run_vcsr_mc_spmm_gpu", "spmm", "upload_vcsr_mc_device",
]
