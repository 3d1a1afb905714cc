"""GPU: the bounded-wait abort path of the tcgen05 kernels (trellis GEMM, router).

Every mbarrier wait in those kernels gives up after the limit set by exl3_set_wait_limit_ns (2 s by
default).  With the limit at 0 ns, any wait that is not already complete gives up at once, so these
tests drive the abort path without any fault: the kernel must record EXL3_ERR_WAIT_TIMEOUT in the
status word, stop every role, drain the copies and MMAs it issued, free its tensor memory and return.
The context must stay usable: the next call with the default limit must match the CPU oracle.  An
aborted router tile leaves its tokens unrouted (id -1), so the sort fused behind it stays in bounds."""
import numpy as np
import pytest
import torch

import exl3_grouped_runtime as rt
import oracle
import synth

pytestmark = pytest.mark.gpu
TIMEOUT = 1          # EXL3_ERR_WAIT_TIMEOUT


def _with_zero_limit(ext, fn):
    prev = ext.set_wait_limit_ns(0)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ext.set_wait_limit_ns(prev)


def test_fat_gemm_gives_up_then_recovers(ext, cuda_device):
    dev = cuda_device
    M, K, N = 300, 1024, 512
    rng = np.random.default_rng(5)
    a16 = rng.standard_normal((M, K)).astype(np.float16)
    packed = rng.integers(-32768, 32768, size=(K // 16, N // 16, 64), dtype=np.int64).astype(np.int16)
    svh = (rng.uniform(0.5, 1.5, N) * rng.choice([-1, 1], N)).astype(np.float16)
    a, pk, sv = (torch.from_numpy(v).to(dev) for v in (a16, packed, svh))
    out = torch.zeros(M, N, device=dev)
    ext.read_status(dev)                                    # start from a clear status word
    _with_zero_limit(ext, lambda: ext.fat_gemm_v2(a, pk, out, sv, 4, True, False, 0))
    assert ext.read_status(dev) == TIMEOUT
    out.zero_()
    ext.fat_gemm_v2(a, pk, out, sv, 4, True, False, 0)
    torch.cuda.synchronize()
    assert ext.read_status(dev) == 0
    want = oracle.fat_gemm_ref(a16, packed, svh)
    assert oracle.rel_l2(out.cpu().numpy(), want) < 1e-4


def test_grouped_layer_gives_up_then_recovers(ext, cuda_device):
    dev = cuda_device
    E, d, f, k, T = 16, 1024, 512, 4, 256
    layer = synth.make_layer(E, d, f, seed=61, sv_scale=0.05)
    x = synth.make_x(T, d, seed=62)
    ids, w = synth.routing("zipf", T, E, k, seed=63)
    Ld = synth.layer_to(layer, dev)
    xd, idd, wd = x.to(dev), ids.to(dev), w.to(dev)
    ext.read_status(dev)
    _with_zero_limit(ext, lambda: rt.grouped_prefill(xd, idd, wd, Ld, 7.0))
    assert ext.read_status(dev) == TIMEOUT
    for _ in range(2):                                      # the context is intact: two normal calls
        out = rt.grouped_prefill(xd, idd, wd, Ld, 7.0)
        torch.cuda.synchronize()
        assert ext.read_status(dev) == 0
    L = oracle.Layer(layer.w13_trellis.numpy(), layer.w13_suh.numpy(), layer.w13_svh.numpy(),
                     layer.w2_trellis.numpy(), layer.w2_suh.numpy(), layer.w2_svh.numpy())
    want = oracle.grouped_staged(x.numpy(), ids.numpy(), w.numpy(), L, 7.0)
    assert oracle.rel_l2(out.cpu().numpy(), want) < 1e-4


def test_route_front_gives_up_with_tokens_unrouted_then_recovers(ext, cuda_device):
    dev = cuda_device
    T, d, E, k = 1000, 1024, 288, 8
    rng = np.random.default_rng(7)
    x16 = rng.standard_normal((T, d)).astype(np.float16)
    w16 = (rng.standard_normal((E, d)) / np.sqrt(d) * 2.0).astype(np.float16)
    x, wr = torch.from_numpy(x16).to(dev), torch.from_numpy(w16).to(dev)
    ids = torch.empty(T, k, dtype=torch.int64, device=dev)
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    b = rt.sort_buffers(T * k, E, dev)

    def call():
        ext.route_front(x, wr, None, k, True, 1.0, ids, w, b.token_sorted, b.weight_sorted, b.expert_of_row,
                        b.counts, b.expert_row0, b.block_expert, b.block_row0, b.meta)

    ext.read_status(dev)
    _with_zero_limit(ext, call)
    assert ext.read_status(dev) == TIMEOUT
    ids_h = ids.cpu().numpy()
    gave_up = (ids_h == -1).all(axis=1)
    assert gave_up.any()
    # tiles that gave up are unrouted, and the sort agrees with the ids it was given
    want = oracle.route_sort(ids_h, w.cpu().numpy(), E)
    assert np.array_equal(b.counts.cpu().numpy(), want["counts"])
    n_valid = int(want["counts"].sum())
    assert np.array_equal(b.token_sorted.cpu().numpy()[:n_valid], want["token_sorted"][:n_valid])
    call()
    torch.cuda.synchronize()
    assert ext.read_status(dev) == 0
    want_ids, _, _ = oracle.router_topk(x16, w16, None, k, norm=True, scale=1.0)
    got = ids.cpu().numpy()
    assert ((got >= 0) & (got < E)).all()
    same = np.mean([set(a.tolist()) == set(b_.tolist()) for a, b_ in zip(got, want_ids)])
    assert same > 0.97
