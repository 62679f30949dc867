"""A bounded device wait that runs out, through the C ABI, without a GPU fault.

vcsrmc_device_wait_check makes one CTA hold tensor memory and wait on an mbarrier phase that can
never complete (its transaction count waits for copies that are never issued), with a short
budget. The wait must give up, report VCSRMC_TIMEOUT through the format's status word, and free its
tensor memory; nothing is in flight when it does. Afterwards the blocking SpMM call reports the
flag as VCSRMC_TIMEOUT until the flag is cleared, and SpMMs on the tensor cores (BAND, SEGMENT) and
on the CUDA cores (ROWS) still run and match the fp64 oracle, on the same format and on a new one.
"""
import ctypes

import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob
from tests.helpers import check_fp16

TIMEOUT = 4
PLANS = [vm.PLAN_ROWS, vm.PLAN_SEGMENT, vm.PLAN_BAND]


def wait_check(dV, budget: int) -> int:
    done = ctypes.c_int(-1)
    vm._lib.call("vcsrmc_device_wait_check", dV.handle, budget, None, ctypes.byref(done))
    return done.value


def test_rejects_a_null_format_without_a_device():
    done = ctypes.c_int()
    with pytest.raises(vm.VcsrmcError) as e:
        vm._lib.call("vcsrmc_device_wait_check", None, 1000, None, ctypes.byref(done))
    assert e.value.status == 1


def spmm_matches_oracle(torch, A, dV, plan):
    rp, col, val = A.arrays()
    B = torch.from_numpy(vm.gen_dense_host(A.N, 128, seed=1)).cuda().half()
    C = torch.full((A.M, 128), 5.0, device="cuda")
    vm.spmm(dV, B, C, accumulate=False, plan=plan)
    torch.cuda.synchronize()
    assert dV.status() == 0
    ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
    check_fp16(C.cpu().numpy(), ref, ab)


@pytest.mark.gpu
@pytest.mark.parametrize("budget", [10_000, 1_000_000], ids=["1e4-cycles", "1e6-cycles"])
def test_expired_wait_reports_timeout_and_the_context_stays_usable(cuda, budget):
    torch = cuda
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 2048, seed=2)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0, plans=PLANS)
    assert dV.status() == 0
    assert wait_check(dV, budget) == 0          # the phase never completed: the wait gave up
    assert dV.status() == 1                     # ... and said so in the format's status word
    B = torch.zeros((A.N, 128), dtype=torch.float32, device="cuda")
    C = torch.zeros((A.M, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(vm.VcsrmcError) as e:    # the blocking call reports the flag
        vm.run_vcsr_mc_spmm_gpu(dV, B, 128, 128, C)
    assert e.value.status == TIMEOUT
    assert dV.status(clear=True) == 1
    assert dV.status() == 0
    for plan in PLANS:                          # same format, after the expiry
        spmm_matches_oracle(torch, A, dV, plan)
    dV.free()
    fresh = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0, plans=PLANS)
    for plan in PLANS:
        spmm_matches_oracle(torch, A, fresh, plan)
    fresh.free()


@pytest.mark.gpu
def test_budget_out_of_range(cuda):
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 256, seed=3)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0, plans=[vm.PLAN_ROWS])
    for budget in (0, -5, 3_000_000_000):
        with pytest.raises(vm.VcsrmcError) as e:
            wait_check(dV, budget)
        assert e.value.status == 1
    assert dV.status() == 0
    dV.free()
