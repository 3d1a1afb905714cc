"""GPU: the routing front-end (router_topk, route_front, moe_prefill_from_hidden) against the CPU oracle.

The router's logits are fp32 sums of exact fp16 products in a different order than the CPU's, so ids
are compared per token where the k-th and (k+1)-th selection scores are more than 1e-5 apart (near-ties
may legitimately swap); weights within 1e-5 relative.  The sort over the router's own output is integer
work and must equal the oracle's sort bit for bit, with the histogram pass fused (topk 8) or not (6)."""
import numpy as np
import pytest
import torch

import b200_ext
import exl3_grouped_runtime as rt
import exl3_router
import oracle
import synth

pytestmark = pytest.mark.gpu
LIMIT = 7.0


def _router_inputs(T, d, E, seed):
    rng = np.random.default_rng(seed)
    x16 = rng.standard_normal((T, d)).astype(np.float16)
    w16 = (rng.standard_normal((E, d)) / np.sqrt(d) * 2.0).astype(np.float16)
    bias = (rng.standard_normal(E) * 0.02).astype(np.float32)
    return x16, w16, bias


def _compare_routing(ids, w, x16, w16, bias, k, scale, min_frac=0.99):
    want_ids, want_w, sel = oracle.router_topk(x16, w16, bias, k, norm=True, scale=scale)
    srt = -np.sort(-sel, axis=1)
    margin = srt[:, k - 1] - srt[:, k] if sel.shape[1] > k else np.full(sel.shape[0], np.inf)
    clear = margin > 1e-5
    assert clear.mean() >= min_frac
    for t in np.nonzero(clear)[0]:
        assert set(ids[t].tolist()) == set(want_ids[t].tolist()), t
        got = dict(zip(ids[t].tolist(), w[t].tolist()))
        for e, we in zip(want_ids[t].tolist(), want_w[t].tolist()):
            assert abs(got[e] - we) <= 1e-5 * abs(we), (t, e, got[e], we)
    return clear


@pytest.mark.parametrize("T,d,E,k", [(1000, 4096, 288, 8), (300, 1024, 16, 4), (129, 512, 48, 6),
                                     (64, 256, 512, 16), (1, 64, 32, 1)])
def test_router_topk_matches_oracle(ext, cuda_device, T, d, E, k):
    dev = cuda_device
    x16, w16, bias = _router_inputs(T, d, E, seed=T + E)
    r = exl3_router.NoauxTcRouter(torch.from_numpy(w16).to(dev), torch.from_numpy(bias).to(dev), topk=k, scale=2.5)
    ids, w = r.route(torch.from_numpy(x16).to(dev))
    torch.cuda.synchronize()
    assert ext.read_status(dev) == 0
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    assert ((ids >= 0) & (ids < E)).all()
    assert all(len(set(row)) == k for row in ids.tolist())          # k distinct experts per token
    _compare_routing(ids, w, x16, w16, bias, k, 2.5)


@pytest.mark.parametrize("k", [8, 6])
def test_route_front_sort_is_the_sort_of_its_routing(ext, cuda_device, k):
    dev = cuda_device
    T, d, E = 1500, 2048, 288
    x16, w16, bias = _router_inputs(T, d, E, seed=k)
    x = torch.from_numpy(x16).to(dev)
    wr = torch.from_numpy(w16).to(dev)
    bs = torch.from_numpy(bias).to(dev)
    ids = torch.empty(T, k, dtype=torch.int64, device=dev)
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    b = rt.sort_buffers(T * k, E, dev)
    ext.route_front(x, wr, bs, k, True, 2.5, ids, w, b.token_sorted, b.weight_sorted, b.expert_of_row, b.counts,
                    b.expert_row0, b.block_expert, b.block_row0, b.meta)
    torch.cuda.synchronize()
    assert ext.read_status(dev) == 0
    ids_h, w_h = ids.cpu().numpy(), w.cpu().numpy()
    _compare_routing(ids_h, w_h, x16, w16, bias, k, 2.5)
    want = oracle.route_sort(ids_h, w_h, E)
    R = T * k
    assert np.array_equal(b.token_sorted.cpu().numpy(), want["token_sorted"][:R])
    assert np.array_equal(b.expert_of_row.cpu().numpy(), want["expert_of_row"][:R])
    assert np.array_equal(b.weight_sorted.cpu().numpy().view(np.uint16), want["weight_sorted"][:R].view(np.uint16))
    assert np.array_equal(b.counts.cpu().numpy(), want["counts"])
    assert np.array_equal(b.expert_row0.cpu().numpy(), want["expert_row0"])


def test_moe_prefill_from_hidden_equals_grouped_prefill_on_its_routing(ext, cuda_device):
    dev = cuda_device
    T, d, f, E, k = 700, 1024, 512, 32, 4
    layer = synth.layer_to(synth.make_layer(E, d, f, seed=31, sv_scale=0.05), dev)
    x16, w16, bias = _router_inputs(T, d, E, seed=32)
    r = exl3_router.NoauxTcRouter(torch.from_numpy(w16).to(dev), torch.from_numpy(bias).to(dev), topk=k, scale=2.5)
    x = torch.from_numpy(x16).to(dev)
    out, ids, w = exl3_router.moe_prefill_from_hidden(x, r, layer, LIMIT, return_routing=True, deterministic=True)
    ref = rt.grouped_prefill(x, ids, w, layer, LIMIT, deterministic=True)
    out_at = exl3_router.moe_prefill_from_hidden(x, r, layer, LIMIT, deterministic=False)
    torch.cuda.synchronize()
    assert ext.read_status(dev) == 0
    # same sorted routing into the same stages, every sum in a fixed order: the same bits
    assert torch.equal(out, ref)
    assert float((out_at - ref).norm() / ref.norm()) < 1e-6       # atomic down stage: only the add order differs
