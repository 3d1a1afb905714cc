"""EXL3 trellis layers beside the routed experts, on the same sm_100a kernels.

GLM-5.3-Flash's MoE block adds one shared expert (the routed experts' SwiGLU shape) to the routed output,
and its first layers are dense SwiGLU MLPs; in an EXL3 checkpoint all of them, like the attention
projections, are 4-bpw trellis matrices with the weight convention W = diag(suh) . H . W' . H . diag(svh)
(harness/proto_fp8.py:61-76).  The reference's kernels stop at the routed experts ("then dense
projections", README.md:87); here they reuse the grouped pipeline's kernels unchanged:

* ``exl3_linear(x, trellis, suh, svh)`` — one projection y = x W: the input Hadamard (``row_had`` without
  a gather) and the trellis GEMM over all rows as a single expert (H128 + svh in its epilogue), fp32
  out (the PR77 ``fat_gemm_v2`` store) or fp16 out (the gate|up stage's row store);
* ``dense_mlp_prefill(x, mlp, limit)`` — a SwiGLU MLP held in the stacked expert layout with one expert
  (``w13_trellis [1, 2, d/16, f/16, 64]`` ...): the grouped pipeline with every token routed to expert 0
  with weight 1;
* ``moe_block_prefill(x, ids, weights, layer, shared, limit)`` — routed experts plus the shared expert,
  accumulated into one fp32 output (the shared expert's down GEMM adds onto the routed result with the
  same fp32 reductions the routed experts use).
"""
from __future__ import annotations

import torch

import b200_ext
import exl3_grouped_runtime as rt


def _single_expert_tables(rows: int, device: torch.device):
    counts = torch.tensor([rows], dtype=torch.int32, device=device)
    row0 = torch.zeros(1, dtype=torch.int32, device=device)
    expert_of_row = torch.zeros(rows, dtype=torch.int32, device=device)
    return counts, row0, expert_of_row


def exl3_linear(x2d: torch.Tensor, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor,
                out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """x2d [T, K] (any float dtype), trellis int16 [K/16, N/16, 64], suh fp16 [K], svh fp16 [N]
    -> x W as out_dtype (float32 or float16) [T, N]."""
    if out_dtype not in (torch.float32, torch.float16):
        raise RuntimeError("exl3_linear: out_dtype must be float32 or float16")
    if trellis.dim() != 3 or trellis.size(2) != 64:
        raise RuntimeError("exl3_linear: trellis must be [K/16, N/16, 64]")
    T, K = x2d.shape
    N = int(trellis.size(1)) * 16
    if int(trellis.size(0)) * 16 != K or suh.numel() != K or svh.numel() != N:
        raise RuntimeError("exl3_linear: K / N mismatch between x, trellis, suh and svh")
    dev = x2d.device
    out = torch.empty(T, N, dtype=out_dtype, device=dev)
    if T == 0:
        return out
    x16 = x2d.to(torch.float16).contiguous()
    counts, row0, expert_of_row = _single_expert_tables(T, dev)
    h = torch.empty(T, K, dtype=torch.float16, device=dev)
    b200_ext.row_had(x16, h, None, expert_of_row, suh.reshape(1, K), False)
    if out_dtype == torch.float32:
        b200_ext.fat_gemm_v2(h, trellis.contiguous(), out, svh.contiguous(), 4, True, False, 0)
    else:
        b200_ext.grouped_gemm(h, trellis.unsqueeze(0), None, svh.reshape(1, N), None, None, None, counts, row0,
                              None, None, out, 0)
    return out


def dense_mlp_prefill(x2d: torch.Tensor, mlp, limit: float, out: torch.Tensor | None = None,
                      stage_hook=None) -> torch.Tensor:
    """SwiGLU MLP in the stacked layout with one expert -> fp32 [T, d] (added into `out` if given)."""
    if int(mlp.w13_trellis.shape[0]) != 1:
        raise RuntimeError("dense_mlp_prefill: the MLP must be stored as one expert ([1, ...] tensors)")
    T = x2d.shape[0]
    ids = torch.zeros(T, 1, dtype=torch.int64, device=x2d.device)
    w = torch.ones(T, 1, dtype=torch.float16, device=x2d.device)
    return rt.grouped_prefill(x2d, ids, w, mlp, limit, stage_hook=stage_hook, out=out)


def moe_block_prefill(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, layer, shared, limit: float,
                      stage_hook=None) -> torch.Tensor:
    """Routed experts (grouped_prefill) + the shared expert (weight 1) -> one fp32 [T, d] output.
    `stage_hook` sees the routed stages by name and the shared expert's as "shared_<stage>"."""
    routed_hook = shared_hook = None
    if stage_hook is not None:
        routed_hook = lambda n: None if (n == "end" and shared is not None) else stage_hook(n)   # noqa: E731
        shared_hook = lambda n: stage_hook(n if n == "end" else "shared_" + n)                    # noqa: E731
    out = rt.grouped_prefill(x2d, ids, weights, layer, limit, stage_hook=routed_hook)
    if shared is not None:
        dense_mlp_prefill(x2d, shared, limit, out=out, stage_hook=shared_hook)
    return out
