"""Routing front-end of a GLM-5.3-Flash MoE layer on the GPU, feeding the grouped prefill directly.

The reference's runtime receives topk_ids / topk_weights from vLLM's router and sorts them
(kernel/exl3_grouped_runtime.py:59-67, 86-112).  GLM-5.3-Flash routes with the DeepSeek-V3 "noaux_tc"
sigmoid router (docs/research/02-glm-5.3-flash-architecture.md:33): sigmoid of an fp32 router GEMM, the
top-8 experts by score + e_score_correction_bias with one group (n_group = topk_group = 1), the unbiased
scores of those experts renormalised to sum 1 and multiplied by routed_scaling_factor = 2.5.

``NoauxTcRouter.route(x)`` runs that router as one sm_100a kernel (tcgen05 GEMM into TMEM, sigmoid, top-k
and weights in the epilogue); ``moe_prefill_from_hidden(x, router, layer, limit)`` runs the router, the
expert sort (whose histogram pass the router kernel already did) and stages 2-5, so the layer goes from
hidden states to its fp32 output without the routing ever leaving the GPU.
"""
from __future__ import annotations

import torch

import b200_ext
import exl3_grouped_runtime as rt


class NoauxTcRouter:
    """weight [E, d] (the checkpoint's router weight, any float dtype; kept as fp16, which holds every
    bf16 value in fp16's normal range exactly), bias [E] (e_score_correction_bias) or None."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, topk: int = 8, norm: bool = True,
                 scale: float = 2.5):
        self.weight = weight.to(torch.float16).contiguous()
        self.bias = None if bias is None else bias.to(device=weight.device, dtype=torch.float32).contiguous()
        self.topk, self.norm, self.scale = int(topk), bool(norm), float(scale)
        self.n_experts = int(weight.shape[0])

    def route(self, x2d: torch.Tensor):
        """x2d [T, d] -> (ids int64 [T, topk], weights fp32 [T, topk])."""
        x16 = x2d.to(torch.float16).contiguous()
        T = x16.shape[0]
        ids = torch.empty(T, self.topk, dtype=torch.int64, device=x16.device)
        w = torch.empty(T, self.topk, dtype=torch.float32, device=x16.device)
        if T:
            b200_ext.router_topk(x16, self.weight, self.bias, self.topk, self.norm, self.scale, ids, w)
        return ids, w


def moe_prefill_from_hidden(x2d: torch.Tensor, router: NoauxTcRouter, layer, limit: float, shared=None,
                            stage_hook=None, return_routing: bool = False, deterministic: bool | None = None):
    """Hidden states [T, d] -> routed-expert output fp32 [T, d] (+ the shared expert if given), with the
    router and the sort on the GPU.  With return_routing, also returns (ids, weights).  `deterministic`
    as for grouped_prefill."""
    if deterministic is None:
        deterministic = rt.deterministic_default()
    hook = stage_hook if stage_hook is not None else (lambda name: None)
    dev = x2d.device
    T, K = x2d.shape
    k, E = router.topk, router.n_experts
    if int(layer.w13_trellis.shape[0]) != E:
        raise RuntimeError("the router and the layer disagree on the number of experts")
    x16 = x2d.to(torch.float16).contiguous()
    # the combine writes every row; the atomic scatter adds onto zeros
    out = (torch.empty if T and deterministic else torch.zeros)(T, K, dtype=torch.float32, device=dev)
    ids = torch.empty(T, k, dtype=torch.int64, device=dev)
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    if T:
        b = rt.sort_buffers(T * k, E, dev)
        hook("route_front")
        b200_ext.route_front(x16, router.weight, router.bias, k, router.norm, router.scale, ids, w, b.token_sorted,
                             b.weight_sorted, b.expert_of_row, b.counts, b.expert_row0, b.block_expert, b.block_row0,
                             b.meta, slots=deterministic)
        rt.run_stages(x16, b, layer, limit, out, hook if shared is None else
                      (lambda n: None if n == "end" else hook(n)), ids, accumulate=False, slots=deterministic)
        if shared is not None:
            import exl3_dense
            exl3_dense.dense_mlp_prefill(x16, shared, limit, out=out,
                                         stage_hook=lambda n: hook(n if n == "end" else "shared_" + n))
    return (out, ids, w) if return_routing else out
