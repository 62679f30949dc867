"""vcsrmc_half_scale_device: the fp16 range scale of values already in device memory, for callers
that cannot allocate device memory (a fixed memory budget, their own pool allocator). The call makes
no allocation: its reduction's scratch word is a file-scope device array, cleared before every call.
Its result is checked against the oracle's scale of the same values, and device free memory must not
change over repeated calls."""
import ctypes

import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob


def half_scale_device(torch, values: np.ndarray) -> float:
    d = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).cuda()
    out = ctypes.c_float()
    vm._lib.call("vcsrmc_half_scale_device", ctypes.c_void_p(d.data_ptr()), int(d.numel()), None, ctypes.byref(out))
    return out.value


def test_rejects_bad_arguments_without_a_device():
    out = ctypes.c_float()
    with pytest.raises(vm.VcsrmcError) as e:
        vm._lib.call("vcsrmc_half_scale_device", None, -1, None, ctypes.byref(out))
    assert e.value.status == 1
    with pytest.raises(vm.VcsrmcError) as e:
        vm._lib.call("vcsrmc_half_scale_device", None, 5, None, ctypes.byref(out))  # NULL values
    assert e.value.status == 1


@pytest.mark.gpu
@pytest.mark.parametrize("amax", [1e6, 26.0, 1e-6, 0.0], ids=["large", "in-range", "tiny", "zero"])
def test_matches_the_oracle(cuda, amax):
    rng = np.random.default_rng(3)
    v = (rng.uniform(-1, 1, 100_003) * amax).astype(np.float32)
    if amax:
        v[777] = -amax  # the extreme is reached exactly
    assert half_scale_device(cuda, v) == ob.half_scale(v)


@pytest.mark.gpu
def test_empty_values(cuda):
    assert half_scale_device(cuda, np.zeros(0, np.float32)) == 1.0


@pytest.mark.gpu
def test_allocates_nothing(cuda):
    torch = cuda
    v = np.random.default_rng(5).uniform(-7e4, 7e4, 1 << 20).astype(np.float32)
    d = torch.from_numpy(v).cuda()
    out = ctypes.c_float()
    call = lambda: vm._lib.call("vcsrmc_half_scale_device", ctypes.c_void_p(d.data_ptr()), int(d.numel()), None,
                                ctypes.byref(out))
    call()  # loads the module (and its static scratch) on first use
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(200):
        call()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    assert out.value == ob.half_scale(v)
