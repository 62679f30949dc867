"""Device-allocation failure: with almost all device memory taken, an upload fails with
VCSRMC_OOM, releases everything it had allocated, and the context stays usable (a later upload
and SpMM succeed). The failure is an ordinary cudaMalloc error, not a GPU fault."""
import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob
from tests.helpers import check_fp16

pytestmark = pytest.mark.gpu


def test_upload_out_of_memory_cleans_up(cuda):
    torch = cuda
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 18, seed=3)  # ~2.6 M entries: a few tens of MB per layout
    V = vm.csr_to_vcsr_mc(A, fp32=False, segw=32)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    free0, _ = torch.cuda.mem_get_info()
    hog = torch.empty(max(0, free0 - (8 << 20)), dtype=torch.uint8, device="cuda")  # leave 8 MB
    try:
        free_hog, _ = torch.cuda.mem_get_info()
        with pytest.raises(vm.VcsrmcError) as e:
            vm.upload_vcsr_mc_device(V, device=0)
        assert e.value.status == 3, e.value  # VCSRMC_OOM
        free_after_fail, _ = torch.cuda.mem_get_info()
        assert free_after_fail == free_hog  # nothing left allocated by the failed upload
    finally:
        del hog
        torch.cuda.empty_cache()
    # the context is still usable
    dV = vm.upload_vcsr_mc_device(V, device=0, plans=[vm.PLAN_ROWS])
    B = torch.from_numpy(vm.gen_dense_host(A.N, 64, seed=3)).cuda().half()
    C = torch.empty((A.M, 64), device="cuda")
    vm.spmm(dV, B, C, accumulate=False)
    torch.cuda.synchronize()
    assert dV.status() == 0
    rows = np.arange(0, A.M, 997)
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64_rows(rp, col, val, B.float().cpu().numpy(), rows, with_abs=True)
    check_fp16(C[torch.from_numpy(rows).cuda()].cpu().numpy(), ref, ab)
    dV.free()


def test_build_device_out_of_memory_cleans_up(cuda):
    torch = cuda
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 18, seed=4)
    rp, col, val = (torch.from_numpy(np.asarray(x)).cuda() for x in A.arrays())
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    free0, _ = torch.cuda.mem_get_info()
    hog = torch.empty(max(0, free0 - (8 << 20)), dtype=torch.uint8, device="cuda")
    try:
        free_hog, _ = torch.cuda.mem_get_info()
        with pytest.raises(vm.VcsrmcError) as e:
            vm.build_vcsr_mc_device(rp, col, val, A.M, A.N, fp32=False, segw=32)
        assert e.value.status == 3, e.value
        free_after_fail, _ = torch.cuda.mem_get_info()
        assert free_after_fail == free_hog
    finally:
        del hog
        torch.cuda.empty_cache()
    dV = vm.build_vcsr_mc_device(rp, col, val, A.M, A.N, fp32=False, segw=32)
    assert dV.status() == 0 and dV.info()["n_units"] > 0
    dV.free()
