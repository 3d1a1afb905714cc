"""CPU: the oracle's router restatement pinned against transformers' own GLM MoE router
(GlmMoeDsaTopkRouter + GlmMoeDsaMoE.route_tokens_to_experts: the noaux_tc sigmoid router GLM-5.3-Flash
uses, docs/research/02-glm-5.3-flash-architecture.md:33), and the router C-ABI argument checks."""
import ctypes
import types

import numpy as np
import pytest
import torch

import oracle


def _hf_route(x16, w16, bias, topk, scale):
    mod = pytest.importorskip("transformers.models.glm_moe_dsa.modeling_glm_moe_dsa")
    E, d = w16.shape
    gate = types.SimpleNamespace(config=types.SimpleNamespace(hidden_size=d), weight=torch.from_numpy(w16),
                                 e_score_correction_bias=torch.from_numpy(bias))
    logits = mod.GlmMoeDsaTopkRouter.forward(gate, torch.from_numpy(x16))
    moe = types.SimpleNamespace(gate=gate, n_group=1, n_routed_experts=E, topk_group=1, top_k=topk,
                                norm_topk_prob=True, routed_scaling_factor=scale)
    ids, w = mod.GlmMoeDsaMoE.route_tokens_to_experts(moe, logits)
    return ids.numpy(), w.numpy()


@pytest.mark.parametrize("T,d,E,k", [(64, 256, 288, 8), (33, 128, 16, 4), (20, 512, 64, 6)])
def test_oracle_router_matches_transformers(T, d, E, k):
    rng = np.random.default_rng(T + E)
    x16 = rng.standard_normal((T, d)).astype(np.float16)
    w16 = (rng.standard_normal((E, d)) * 0.05).astype(np.float16)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    ids, w, _ = oracle.router_topk(x16, w16, bias, k, norm=True, scale=2.5)
    hf_ids, hf_w = _hf_route(x16, w16, bias, k, 2.5)
    for t in range(T):
        got = dict(zip(ids[t].tolist(), w[t].tolist()))
        want = dict(zip(hf_ids[t].tolist(), hf_w[t].tolist()))
        assert set(got) == set(want), t
        for e in got:
            assert abs(got[e] - want[e]) <= 2e-6 * abs(want[e]), (t, e, got[e], want[e])


def test_oracle_router_orders_by_score_then_id():
    # equal selection scores: the lower expert id first; bias moves experts up the order
    x16 = np.zeros((1, 64), np.float16)
    w16 = np.zeros((8, 64), np.float16)
    bias = np.array([0, 0, 0.5, 0, 0, 0.25, 0, 0], np.float32)
    ids, w, _ = oracle.router_topk(x16, w16, bias, 4, norm=True, scale=1.0)
    assert ids[0].tolist() == [2, 5, 0, 1]
    assert np.allclose(w[0], 0.25)                      # unbiased scores are all sigmoid(0) = 0.5


def test_router_entry_points_validate_without_gpu():
    import b200_ext
    lib = b200_ext.load()
    P = ctypes.c_void_p
    rc = lib.exl3_router_topk(P(16), 10, 4096, P(16), 290, None, 8, 1, 2.5, P(16), P(16), None, None)
    assert rc != 0 and b"multiple of 16" in lib.exl3_last_error()
    rc = lib.exl3_router_topk(P(16), 10, 4096, P(16), 272, None, 8, 1, 2.5, P(16), P(16), None, None)
    assert rc != 0 and b"equal boxes" in lib.exl3_last_error()             # 2 x 136: not 16-multiples
    rc = lib.exl3_router_topk(P(16), 10, 4000, P(16), 288, None, 8, 1, 2.5, P(16), P(16), None, None)
    assert rc != 0 and b"multiple of 64" in lib.exl3_last_error()
    rc = lib.exl3_router_topk(P(16), 10, 4096, P(16), 288, None, 17, 1, 2.5, P(16), P(16), None, None)
    assert rc != 0 and b"topk must be 1..16" in lib.exl3_last_error()
    rc = lib.exl3_router_topk(P(18), 10, 4096, P(16), 288, None, 8, 1, 2.5, P(16), P(16), None, None)
    assert rc != 0 and b"16-byte aligned" in lib.exl3_last_error()
    assert lib.exl3_router_topk(None, 0, 4096, None, 288, None, 8, 1, 2.5, None, None, None, None) == 0
    assert lib.exl3_route_front_scratch_elems(8192, 8, 288) == 64 * 289
    assert lib.exl3_route_front_scratch_elems(8192, 6, 288) == max(64, (8192 * 6 + 2047) // 2048) * 289
    rc = lib.exl3_route_front(P(16), 8192, 4096, P(16), 288, None, 8, 1, 2.5, P(16), P(16), P(16), P(16), P(16),
                              P(16), P(16), P(16), P(16), 800, P(16), P(16), 100, None, None)
    assert rc != 0 and b"scratch must hold" in lib.exl3_last_error()
