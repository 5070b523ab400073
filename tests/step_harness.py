"""Builds matching adapter sets for the CUDA grouped step and the CPU oracle.

Test infrastructure: the oracle replays the reference controller on CPU with the Gaussian
draws the reference would take from a torch CUDA generator (per module Zc_B then Zc_A,
ds_mezo/controller.py:184-191), so both sides consume identical random numbers.
"""
from __future__ import annotations

import math

import torch

from oracle import reference_ops as ref


def make_inputs(layers, hidden, inter, kv, rank, tokens, seed, copy_dtype=torch.float32, act_dtype=torch.float32):
    """Seeded synthetic adapter set: factors and momentum N(0,1) (momentum 0 for a fresh
    start is a separate case), activations N(0,1) x lognormal(0,1) channel scales,
    bases = QR of a Gaussian."""
    from dsmezo_b200 import transformer_adapter_shapes
    mods, bases = transformer_adapter_shapes(layers, hidden, inter, kv, tokens)
    g = torch.Generator().manual_seed(seed)
    A = [torch.randn(m.d_out, rank, generator=g).to(copy_dtype) for m in mods]
    B = [torch.randn(rank, m.d_in, generator=g).to(copy_dtype) for m in mods]
    V0 = [torch.linalg.qr(torch.randn(b.D, rank, generator=g))[0].contiguous() for b in bases]
    H = []
    for b in bases:
        scale = torch.exp(torch.randn(b.D, generator=g))
        H.append((torch.randn(b.T, b.D, generator=g) * scale).to(act_dtype))
    return mods, bases, A, B, V0, H


def cuda_draws(mods, rank, basis_width, seed, offset, device):
    """The draws the reference controller takes for one step from a CUDA generator at
    (seed, offset), in controller order; returns (list of CPU tensors, end offset)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    gen.set_offset(offset)
    out = []
    rca = min(rank, basis_width)
    for m in mods:
        out.append(torch.randn(rank, basis_width, device=device, generator=gen).cpu())
        out.append(torch.randn(m.d_out, rca, device=device, generator=gen).cpu())
    return out, gen.get_offset()


def oracle_state(mods, A, B, V0, eps, total_steps, mu=None, var=None, schedule=None, dtype=torch.float32):
    """Oracle step state; dtype float32 follows the reference's rounding, float64 gives the
    same algorithm without it (the exact value the reference approximates)."""
    modules = []
    for i, m in enumerate(mods):
        a = A[i].to(dtype).clone()
        b = B[i].to(dtype).clone()
        modules.append(ref.Module(m.layer, m.name, a, b,
                                  torch.zeros_like(a) if mu is None else mu[i][0].to(dtype).clone(),
                                  torch.zeros_like(b) if mu is None else mu[i][1].to(dtype).clone(),
                                  torch.full_like(a, eps ** 2) if var is None else var[i][0].to(dtype).clone(),
                                  torch.full_like(b, eps ** 2) if var is None else var[i][1].to(dtype).clone(),
                                  basis=m.basis))
    st = ref.StepState(modules, [v.to(dtype).clone() for v in V0], eps=eps, total_steps=total_steps,
                       schedule=ref.ns_cubic_schedule() if schedule is None else schedule, dtype=dtype)
    return st


def rel(a, b):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))
