"""Contrastive scoring loss on the device (ds_mezo/controller.py:14-15, 194-201, 307).

The reference pulls every scored token's logprob from vLLM into Python lists and forms
``sum_i adv_i * mean NLL(sequence i)`` for the + and - adapters on the host. Here the
logits rows that predict the scored tokens (or their logprobs) stay on the GPU and one
fused pass (log-sum-exp per row, target pick, advantage-weighted mean per sequence, fixed
summation order) returns the loss as a device fp64 scalar.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from ._lib import check, lib

SCORE_LOGITS_F32, SCORE_LOGITS_BF16, SCORE_LOGPROBS_F32 = 0, 1, 2


def contrastive_loss(src: torch.Tensor, seq_tokens: Sequence[int], advantages: Sequence[float],
                     targets: Optional[torch.Tensor] = None) -> torch.Tensor:
    """sum_i advantages[i] * mean over sequence i's scored tokens of -logprob(token).

    src: the logits rows that predict the scored tokens (ntok x V, fp32 or bf16, unit
    column stride; sequence i owns the next seq_tokens[i] rows) with `targets` (ntok int32
    token ids), or the scored tokens' logprobs (ntok fp32) with targets None. Returns a
    one-element fp64 tensor on src's device, written on the current stream; NaN if a
    target lies outside the vocabulary."""
    n = len(seq_tokens)
    if n != len(advantages):
        raise ValueError("contrastive_loss: one advantage per sequence")
    ntok = int(sum(seq_tokens))
    if targets is None:
        if src.dtype != torch.float32 or src.dim() != 1 or src.numel() != ntok:
            raise ValueError("contrastive_loss: logprobs must be a 1-D fp32 tensor of sum(seq_tokens) entries")
        kind, V, ld, tp = SCORE_LOGPROBS_F32, 1, 1, None
    else:
        if src.dim() != 2 or src.shape[0] != ntok or src.stride(1) != 1:
            raise ValueError("contrastive_loss: logits must be ntok x V with unit column stride")
        if src.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError("contrastive_loss: logits must be float32 or bfloat16")
        if targets.dtype != torch.int32 or targets.numel() != ntok or targets.device != src.device:
            raise ValueError("contrastive_loss: targets must be ntok int32 token ids on the logits' device")
        kind = SCORE_LOGITS_F32 if src.dtype == torch.float32 else SCORE_LOGITS_BF16
        tgt = targets.contiguous()
        V, ld, tp = src.shape[1], src.stride(0), tgt.data_ptr()
    start = (ctypes.c_int64 * (n + 1))()
    o = 0
    for i, k in enumerate(seq_tokens):
        start[i] = o
        o += int(k)
    start[n] = o
    adv = (ctypes.c_double * n)(*[float(a) for a in advantages])
    L = lib()
    wsb = int(L.dsmz_contrastive_loss_workspace_bytes(ntok))
    ws = torch.empty(wsb, dtype=torch.uint8, device=src.device)
    out = torch.empty(1, dtype=torch.float64, device=src.device)
    check(L.dsmz_contrastive_loss(kind, src.data_ptr(), V, ld, tp, ntok, start, adv, n, out.data_ptr(),
                                  ws.data_ptr(), wsb, torch.cuda.current_stream(src.device).cuda_stream),
          "dsmz_contrastive_loss")
    return out


def projected_gradient(loss_pos: float, loss_neg: float, eps: float) -> float:
    """dd = (L+ - L-) / (2 eps), ds_mezo/controller.py:307."""
    return float(loss_pos - loss_neg) / (2.0 * eps)
