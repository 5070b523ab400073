"""The allocation-free ZO-Muon update (dsmz_zo_muon_update_noalloc) through the C ABI.

It serves callers that cannot allocate device memory while they update an adapter (a
rollout engine that reserved nearly all of HBM up front, or a C host without a device
allocator). Its results must equal those of dsmz_zo_muon_update with a caller workspace,
call after call, although every call reuses the same built-in scratch array. This file
is collected last so a failure here comes after every other test has run.
"""
import ctypes

import pytest
import torch

from step_harness import rel

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _with_workspace(L, p, b, s, eta, sched, stream):
    M, N = p.shape
    ws = torch.empty(L.dsmz_zo_muon_update_workspace_bytes(M, N), dtype=torch.uint8, device=DEV)
    rc = L.dsmz_zo_muon_update(1 if p.dtype == torch.bfloat16 else 0, p.data_ptr(), p.stride(0), p.stride(1),
                               b.data_ptr(), b.stride(0), b.stride(1), s.data_ptr(), s.stride(0), s.stride(1),
                               M, N, eta, 1e-38, sched, ws.data_ptr(), ws.numel(), stream)
    assert rc == 0, L.dsmz_last_error()


def _noalloc(L, p, b, s, eta, sched, stream):
    M, N = p.shape
    return L.dsmz_zo_muon_update_noalloc(1 if p.dtype == torch.bfloat16 else 0, p.data_ptr(), p.stride(0),
                                         p.stride(1), b.data_ptr(), b.stride(0), b.stride(1), s.data_ptr(),
                                         s.stride(0), s.stride(1), M, N, eta, 1e-38, sched, stream)


@pytest.mark.parametrize("M,N,dt", [(3584, 64, torch.float32), (64, 3584, torch.bfloat16), (300, 5, torch.float32),
                                    (18944, 64, torch.bfloat16), (8192, 128, torch.float32)])
def test_noalloc_matches_workspace_entry_on_consecutive_calls(M, N, dt):
    from dsmezo_b200 import _lib
    L = _lib.lib()
    sched = _lib.schedule("cubic")
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=DEV)
    g.manual_seed(M + N)
    for call in range(2):                       # the second call sees the first call's leftovers
        param = torch.randn(M, N, generator=g, device=DEV).to(dt)
        buf = torch.randn(M, N, generator=g, device=DEV) * (1.0 + call)
        p_ref, s_ref = param.clone(), torch.zeros(M, N, device=DEV)
        _with_workspace(L, p_ref, buf, s_ref, 0.01, sched, stream)
        p_na, s_na = param.clone(), torch.full((M, N), float("nan"), device=DEV)
        rc = _noalloc(L, p_na, buf, s_na, 0.01, sched, stream)
        assert rc == 0, L.dsmz_last_error()
        torch.cuda.synchronize()
        assert rel(s_na, s_ref) < 1e-5           # the Newton-Schulz output tolerance of the suite
        assert rel(p_na.float(), p_ref.float()) < 1e-6


def test_noalloc_takes_no_device_memory():
    """Device-wide free memory (cudaMemGetInfo) is the same before and after calls of the
    entry point, once its inputs exist and a first call has looked up the scratch array."""
    from dsmezo_b200 import _lib
    L = _lib.lib()
    sched = _lib.schedule("cubic")
    stream = torch.cuda.current_stream().cuda_stream
    M, N = 8192, 128                            # close to the scratch size (~1.66 MiB)
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    param = torch.randn(M, N, generator=g, device=DEV)
    buf = torch.randn(M, N, generator=g, device=DEV)
    out = torch.zeros(M, N, device=DEV)
    assert _noalloc(L, param, buf, out, 0.01, sched, stream) == 0, L.dsmz_last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _noalloc(L, param, buf, out, 0.01, sched, stream) == 0, L.dsmz_last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from dsmezo_b200 import _lib
    L = _lib.lib()
    M, N = 1_000_000, 128
    assert L.dsmz_zo_muon_update_workspace_bytes(M, N) > 2 * 1024 * 1024
    rc = L.dsmz_zo_muon_update_noalloc(0, ctypes.c_void_p(16), N, 1, ctypes.c_void_p(16), N, 1, None, 0, 0, M, N,
                                       0.01, 1e-38, None, torch.cuda.current_stream().cuda_stream)
    assert rc == 4
    assert b"scratch bytes" in L.dsmz_last_error()
