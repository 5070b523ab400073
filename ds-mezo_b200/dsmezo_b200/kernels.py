"""Drop-in replacement for the reference module ``ds_mezo.kernels``.

Same four functions, same arguments and results as ds_mezo/kernels.py:167, :249, :371
and :415, imported by ds_mezo/controller.py:11. Each runs hand-written sm_100a kernels
of libdsmezo.so through its C ABI on the current CUDA stream. There is no CPU path:
CPU tensors or a missing library raise.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import DSMZ_BF16, DSMZ_F32, check, lib

__all__ = ["zo_muon_update", "fused_power_iter", "fused_agzo_perturbation", "fused_perturb_dual"]

_DT = {torch.float32: DSMZ_F32, torch.bfloat16: DSMZ_BF16}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise ValueError("dsmezo_b200 kernels take CUDA tensors only (no CPU fallback)")


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def zo_muon_update(param, buf, scratch, eta, norm_floor, schedule="cubic"):
    """ds_mezo/kernels.py:167-186: scratch <- NS(buf); param -= eta * scratch (in place).

    ``schedule`` extends the reference: 'cubic' (the reference's 12 steps), 'quintic', or
    explicit (c0, c1, c2) triples for S = c0 I + c1 G + c2 G^2.
    """
    _need_cuda(param, buf, scratch)
    if param.dim() != 2 or buf.shape != param.shape or scratch.shape != param.shape:
        raise ValueError("zo_muon_update: param, buf and scratch must be 2-D of one shape")
    if param.dtype not in _DT or buf.dtype != torch.float32 or scratch.dtype != torch.float32:
        raise ValueError("zo_muon_update: param fp32/bf16, buf and scratch fp32")
    M, N = param.shape
    # The kernels index buf and scratch with param's strides (as the reference does); give
    # them that layout when the caller's tensors differ.
    b = buf if buf.stride() == param.stride() else torch.empty_strided(param.shape, param.stride(), dtype=buf.dtype,
                                                                       device=buf.device).copy_(buf)
    s = scratch if scratch.stride() == param.stride() else torch.empty_strided(
        param.shape, param.stride(), dtype=scratch.dtype, device=scratch.device)
    ws = _workspace(lib().dsmz_zo_muon_update_workspace_bytes(M, N), param.device)
    sched = _lib.schedule(schedule)
    check(lib().dsmz_zo_muon_update(_DT[param.dtype], param.data_ptr(), param.stride(0), param.stride(1),
                                    b.data_ptr(), b.stride(0), b.stride(1), s.data_ptr(), s.stride(0), s.stride(1),
                                    M, N, float(eta), float(norm_floor), sched, ws.data_ptr(), ws.numel(),
                                    _stream(param)), "zo_muon_update")
    if s is not scratch:
        scratch.copy_(s)


def fused_power_iter(H, V, num_iters, norm_floor):
    """ds_mezo/kernels.py:249-265: ``num_iters`` x {W = H^T (H V); V = QR(W)}; new D x R fp32."""
    _need_cuda(H, V)
    if H.dim() != 2 or V.dim() != 2 or V.shape[0] != H.shape[1]:
        raise ValueError("fused_power_iter: H is T x D and V is D x R")
    if H.dtype not in _DT:
        H = H.float()
    if V.dtype != torch.float32:
        V = V.float()
    T, D = H.shape
    R = V.shape[1]
    out = torch.empty(D, R, device=H.device, dtype=torch.float32)
    ws = _workspace(lib().dsmz_power_iter_workspace_bytes(T, D, R), H.device)
    check(lib().dsmz_power_iter(_DT[H.dtype], H.data_ptr(), T, D, H.stride(0), H.stride(1),
                                V.data_ptr(), R, V.stride(0), V.stride(1), out.data_ptr(), int(num_iters),
                                float(norm_floor), ws.data_ptr(), ws.numel(), _stream(H)), "fused_power_iter")
    return out


def fused_agzo_perturbation(B, V, z_coeff_B, z_coeff_A, eps, norm_floor):
    """ds_mezo/kernels.py:371-397: returns (z_A [d_out x R], z_B [R x d_in]) fp32."""
    assert z_coeff_B.is_contiguous() and z_coeff_A.is_contiguous(), (
        "z_coeff tensors must be C-contiguous (kernel uses hardcoded stride=RC)"
    )
    _need_cuda(B, V, z_coeff_B, z_coeff_A)
    if B.dtype != torch.float32:
        B = B.float()
    if V.dtype != torch.float32:
        V = V.float()
    R, d_in = B.shape
    RC = V.shape[1]
    d_out = z_coeff_A.shape[0]
    if V.shape[0] != d_in or tuple(z_coeff_B.shape) != (R, RC) or z_coeff_A.shape[1] != min(R, RC):
        raise ValueError("fused_agzo_perturbation: inconsistent shapes")
    z_A = torch.empty(d_out, R, device=B.device, dtype=torch.float32)
    z_B = torch.empty(R, d_in, device=B.device, dtype=torch.float32)
    ws = _workspace(lib().dsmz_agzo_perturbation_workspace_bytes(R, d_in, RC, d_out), B.device)
    check(lib().dsmz_agzo_perturbation(B.data_ptr(), R, d_in, B.stride(0), B.stride(1),
                                       V.data_ptr(), RC, V.stride(0), V.stride(1),
                                       z_coeff_B.float().data_ptr(), z_coeff_A.float().data_ptr(), d_out,
                                       z_A.data_ptr(), z_B.data_ptr(), float(eps), float(norm_floor),
                                       ws.data_ptr(), ws.numel(), _stream(B)), "fused_agzo_perturbation")
    return z_A, z_B


def fused_perturb_dual(base, z, pos, neg):
    """ds_mezo/kernels.py:415-422: pos = base + z, neg = base - z (flat, contiguous)."""
    _need_cuda(base, z, pos, neg)
    if not (base.is_contiguous() and z.is_contiguous() and pos.is_contiguous() and neg.is_contiguous()):
        raise ValueError("fused_perturb_dual: tensors must be contiguous (flat kernel)")
    n = base.numel()
    if z.numel() != n or pos.numel() != n or neg.numel() != n:
        raise ValueError("fused_perturb_dual: size mismatch")
    if base.dtype not in _DT or pos.dtype != base.dtype or neg.dtype != base.dtype or z.dtype != torch.float32:
        raise ValueError("fused_perturb_dual: base/pos/neg fp32 or bf16 (one dtype), z fp32")
    check(lib().dsmz_perturb_dual(_DT[base.dtype], base.data_ptr(), z.data_ptr(), pos.data_ptr(), neg.data_ptr(), n,
                                  _stream(base)), "fused_perturb_dual")
