"""Seeded synthetic MoE layers and routings for the EXL3 grouped prefill path.

No checkpoint is available, so every benchmark and parity case runs on inputs generated here:

* packed trellis words: uniform-random int16;
* per-expert sign/scale vectors su/sv: +-1 (Bernoulli 0.5) times fp16 U(0.5, 1.5), optionally times
  ``sv_scale``; gate and up share su (kernel/test_grouped.py:82-84 requires it);
* activations x ~ N(0, 1) fp16;
* routing: ``uniform`` = top-k of N(0,1) logits, ``zipf`` = top-k of log p + Gumbel noise with expert
  popularity p ~ rank^-s over a seeded permutation of the experts; route weights are the softmax of
  the selected scores.  ``skewed`` restates routing_skewed of kernel/test_grouped.py:95-106 and
  ``randperm`` restates routing of harness/test_exl3_moe_op.py:119-132.

The layer object carries the attributes grouped_prefill reads (kernel/exl3_grouped_runtime.py:57-82):
w13_trellis [E,2,d/16,f/16,64], w13_suh [E,2,d], w13_svh [E,2,f], w2_trellis [E,f/16,d/16,64],
w2_suh [E,f], w2_svh [E,d], _exl3_intermediate_local = f, expert_map = None.
"""
from __future__ import annotations

import torch


class SyntheticLayer(torch.nn.Module):
    """Stand-in for the vLLM MoE layer (FakeLayer of kernel/test_grouped.py:89-90)."""


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def _signed_scales(shape, g, device, scale: float) -> torch.Tensor:
    sign = torch.randint(0, 2, shape, generator=g, device=device, dtype=torch.int8).to(torch.float32) * 2 - 1
    mag = torch.rand(shape, generator=g, device=device, dtype=torch.float32) + 0.5
    return (sign * mag * scale).to(torch.float16)


def make_layer(n_experts: int, hidden: int, inter: int, seed: int = 0, device="cpu",
               sv_scale: float = 1.0) -> SyntheticLayer:
    """One synthetic EXL3 4-bpw MoE layer (BASELINE.json configs 0/1 shapes)."""
    assert hidden % 128 == 0 and inter % 128 == 0
    E, d, f = n_experts, hidden, inter
    g = _gen(seed, device)
    layer = SyntheticLayer()
    layer.w13_trellis = torch.randint(-32768, 32768, (E, 2, d // 16, f // 16, 64), generator=g,
                                      device=device, dtype=torch.int16)
    layer.w2_trellis = torch.randint(-32768, 32768, (E, f // 16, d // 16, 64), generator=g,
                                     device=device, dtype=torch.int16)
    suh = _signed_scales((E, d), g, device, 1.0)
    layer.w13_suh = torch.stack([suh, suh], dim=1).contiguous()
    layer.w13_svh = _signed_scales((E, 2, f), g, device, sv_scale)
    layer.w2_suh = _signed_scales((E, f), g, device, 1.0)
    layer.w2_svh = _signed_scales((E, d), g, device, sv_scale)
    layer._exl3_hidden_size = d
    layer._exl3_intermediate_local = f
    layer._exl3_bits = 4
    layer.expert_map = None
    return layer


def make_x(tokens: int, hidden: int, seed: int = 1, device="cpu", std: float = 1.0) -> torch.Tensor:
    g = _gen(seed, device)
    return (torch.randn(tokens, hidden, generator=g, device=device) * std).to(torch.float16)


def _select(scores: torch.Tensor, topk: int):
    vals, ids = torch.topk(scores, topk, dim=-1)
    w = torch.softmax(vals.float(), dim=-1)
    return ids.to(torch.int64), w


def routing(kind: str, tokens: int, n_experts: int, topk: int, seed: int = 2, device="cpu",
            zipf_s: float = 1.1, popularity_seed: int | None = None):
    """-> (ids int64 [T, k], weights fp32 [T, k]).  Zipf: expert popularity ranks are a random permutation;
    with `popularity_seed` the permutation comes from that seed and the samples from `seed` (two batches
    of one router), otherwise both come from `seed`."""
    if kind == "uniform":
        g = _gen(seed, device)
        logits = torch.randn(tokens, n_experts, generator=g, device=device)
        return _select(logits, topk)
    if kind == "zipf":
        g = _gen(seed, device)
        if popularity_seed is not None:
            perm = torch.randperm(n_experts, generator=_gen(popularity_seed, device), device=device)
        else:
            perm = torch.randperm(n_experts, generator=g, device=device)
        rank = torch.empty(n_experts, device=device, dtype=torch.float32)
        rank[perm] = torch.arange(1, n_experts + 1, device=device, dtype=torch.float32)
        logp = -zipf_s * torch.log(rank)
        logp = logp - torch.logsumexp(logp, 0)
        u = torch.rand(tokens, n_experts, generator=g, device=device).clamp_(1e-12, 1.0 - 1e-7)
        gumbel = -torch.log(-torch.log(u))
        return _select(logp[None, :] + gumbel, topk)
    if kind == "skewed":
        return routing_skewed(tokens, n_experts, topk, seed)
    if kind == "randperm":
        return routing_randperm(tokens, n_experts, topk, seed)
    raise ValueError(f"unknown routing kind {kind!r}")


def routing_skewed(tokens: int, n_experts: int, topk: int, seed: int, hot: int = 12, share: float = 0.55):
    """kernel/test_grouped.py:95-106 restated: `hot` experts take `share` of all slots."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.empty(tokens, topk, dtype=torch.long)
    for t in range(tokens):
        pool = []
        while len(pool) < topk:
            if torch.rand(1, generator=g).item() < share:
                e = int(torch.randint(0, hot, (1,), generator=g))
            else:
                e = int(torch.randint(0, n_experts, (1,), generator=g))
            if e not in pool:
                pool.append(e)
        ids[t] = torch.tensor(pool)
    w = torch.rand(tokens, topk, generator=g)
    w = w / w.sum(-1, keepdim=True)
    return ids, w


def routing_randperm(tokens: int, n_experts: int, topk: int, seed: int, fat_expert=None, fat_rows: int = 0):
    """harness/test_exl3_moe_op.py:119-132 restated: distinct top-k via randperm, rand weights normalised;
    optionally force `fat_expert` into slot 0 of the first `fat_rows` tokens (the fat-expert check)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.stack([torch.randperm(n_experts, generator=g)[:topk] for _ in range(tokens)])
    if fat_expert is not None:
        ids[:fat_rows, 0] = fat_expert
        for r in range(fat_rows):
            dup = (ids[r, 1:] == fat_expert).nonzero()
            for d in dup.view(-1).tolist():
                ids[r, 1 + d] = (fat_expert + 1 + d) % n_experts
    w = torch.rand(tokens, topk, generator=g)
    w = w / w.sum(-1, keepdim=True)
    return ids, w


def layer_to(layer: SyntheticLayer, device) -> SyntheticLayer:
    out = SyntheticLayer()
    for k, v in vars(layer).items():
        if k.startswith("_") and not k.startswith("_exl3"):
            continue
        setattr(out, k, v.to(device) if isinstance(v, torch.Tensor) else v)
    return out


def moe_flops(tokens: int, topk: int, hidden: int, inter: int) -> float:
    """Algorithmic FLOPs of one layer: 2*R*d*2f (gate|up) + 2*R*f*d (down) = 6*R*d*f."""
    return 6.0 * tokens * topk * hidden * inter


def packed_bytes(n_experts: int, hidden: int, inter: int) -> float:
    """4-bpw packed weight bytes: 3*d*f/2 per expert."""
    return n_experts * 3.0 * hidden * inter / 2.0


__all__ = ["SyntheticLayer", "make_layer", "make_x", "routing", "routing_skewed", "routing_randperm",
           "layer_to", "moe_flops", "packed_bytes"]
