"""Small-batch (decode-sized) calls of the grouped pipeline, replayed from CUDA graphs.

The reference sends calls with tokens <= the fused kernel's row cap to exllamav3's fused per-expert MoE
kernel (kernel/exl3_grouped_runtime.py:95-98; its tuned variant kernel/tuned-fused-kernel-patch/.../
exl3_moe_kernel.cuh:24-256).  On B200 the grouped pipeline already decodes each expert's weights once
per 256-row tile, which is also what a fused small-batch kernel must do, so the work per call is the
same; what dominates at a few tokens is the host: six launches with their argument checks and tensor
allocations take longer than the kernels (one token: 0.24 ms per layer through the eager path).

``GraphedPrefill`` captures ``grouped_prefill`` once per token bucket (powers of two up to
``max_tokens``) into a CUDA graph with static input and output buffers and replays it: a call copies
its inputs into the bucket's buffers (padding tokens get expert id -1, which the sort leaves unrouted),
replays the graph and returns a view of the bucket's fp32 output.  Results equal ``grouped_prefill``'s
(bit for bit with deterministic=True; with the atomic down stage up to the order of the fp32 adds).
"""
from __future__ import annotations

import torch

import exl3_grouped_runtime as rt


class GraphedPrefill:
    """Per-layer small-batch prefill from CUDA graphs.  layer: the stacked layer; tokens <= max_tokens."""

    def __init__(self, layer, limit: float, topk: int, max_tokens: int = 64, device: torch.device | None = None,
                 deterministic: bool | None = None):
        if max_tokens < 1:
            raise RuntimeError("max_tokens must be positive")
        self.layer, self.limit, self.topk = layer, float(limit), int(topk)
        self.deterministic = rt.deterministic_default() if deterministic is None else bool(deterministic)
        self.device = device if device is not None else layer.w13_trellis.device
        self.d = int(layer.w13_trellis.shape[2]) * 16
        self.max_tokens = int(max_tokens)
        self._graphs = {}                  # bucket -> (graph, x, ids, w, out)

    @staticmethod
    def bucket(tokens: int) -> int:
        b = 1
        while b < tokens:
            b *= 2
        return b

    def _capture(self, b: int):
        dev = self.device
        x = torch.zeros(b, self.d, dtype=torch.float16, device=dev)
        ids = torch.full((b, self.topk), -1, dtype=torch.int64, device=dev)
        w = torch.zeros(b, self.topk, dtype=torch.float32, device=dev)
        # warm up on a side stream: loads the library and sets every kernel attribute before the capture
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                rt.grouped_prefill(x, ids, w, self.layer, self.limit, deterministic=self.deterministic)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = rt.grouped_prefill(x, ids, w, self.layer, self.limit, deterministic=self.deterministic)
        return graph, x, ids, w, out

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """x [T, d], ids [T, topk], weights [T, topk] -> fp32 [T, d] (a view of the bucket's output buffer,
        valid until the next call with the same bucket)."""
        T = int(x.shape[0])
        if T > self.max_tokens:
            raise RuntimeError(f"{T} tokens exceed max_tokens={self.max_tokens}")
        if tuple(ids.shape) != (T, self.topk) or tuple(weights.shape) != (T, self.topk):
            raise RuntimeError("ids / weights must be [T, topk]")
        if T == 0:
            return torch.zeros(0, self.d, dtype=torch.float32, device=self.device)
        b = self.bucket(T)
        if b not in self._graphs:
            self._graphs[b] = self._capture(b)
        graph, xs, ids_s, ws, out = self._graphs[b]
        xs[:T].copy_(x)
        ids_s[:T].copy_(ids)
        ws[:T].copy_(weights)
        if T < b:
            xs[T:].zero_()
            ids_s[T:].fill_(-1)
            ws[T:].zero_()
        graph.replay()
        return out[:T]
