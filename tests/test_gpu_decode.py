"""GPU: the small-batch path (exl3_decode.GraphedPrefill, grouped_prefill replayed from CUDA graphs) against
the eager grouped_prefill on the same inputs, at decode-sized token counts including padded buckets,
with the graphs reused across calls: bit-identical with the deterministic down stage, within the fp32
add order with the atomic one.  Also checked against the CPU oracle at one size."""
import numpy as np
import pytest
import torch

import exl3_decode
import exl3_grouped_runtime as rt
import oracle
import synth

pytestmark = pytest.mark.gpu
LIMIT = 7.0


def test_graphed_small_batches_match_eager(ext, cuda_device):
    dev = cuda_device
    E, d, f, k = 288, 4096, 1536, 8
    layer = synth.layer_to(synth.make_layer(E, d, f, seed=41, sv_scale=0.05), dev)
    gp = exl3_decode.GraphedPrefill(layer, LIMIT, k, max_tokens=32, deterministic=True)
    gp_at = exl3_decode.GraphedPrefill(layer, LIMIT, k, max_tokens=32, deterministic=False)
    for i, T in enumerate([1, 5, 8, 32, 5, 1, 3]):          # repeats reuse captured graphs
        x = synth.make_x(T, d, seed=100 + i).to(dev)
        ids, w = synth.routing("zipf", T, E, k, seed=200 + i, device=dev)
        got = gp(x, ids, w).clone()
        got_at = gp_at(x, ids, w).clone()
        want = rt.grouped_prefill(x, ids, w, layer, LIMIT, deterministic=True)
        torch.cuda.synchronize()
        assert torch.equal(got, want), T
        assert float((got_at - want).norm() / want.norm()) < 1e-6, T
    assert sorted(gp._graphs) == [1, 4, 8, 32]
    assert ext.read_status(dev) == 0


def test_graphed_small_batch_matches_oracle(ext, cuda_device):
    dev = cuda_device
    E, d, f, k, T = 16, 1024, 512, 4, 6
    layer = synth.make_layer(E, d, f, seed=43, sv_scale=0.05)
    L = oracle.Layer(*(getattr(layer, n).numpy() for n in
                       ("w13_trellis", "w13_suh", "w13_svh", "w2_trellis", "w2_suh", "w2_svh")))
    x = synth.make_x(T, d, seed=44)
    ids, w = synth.routing("uniform", T, E, k, seed=45)
    gp = exl3_decode.GraphedPrefill(synth.layer_to(layer, dev), LIMIT, k, max_tokens=8)
    got = gp(x.to(dev), ids.to(dev), w.to(dev)).cpu().numpy()
    want = oracle.grouped_staged(x.numpy(), ids.numpy(), w.numpy(), L, LIMIT)
    assert oracle.rel_l2(got, want) < 1e-4
    with pytest.raises(RuntimeError, match="exceed max_tokens"):
        gp(torch.zeros(9, d, dtype=torch.float16, device=dev), torch.zeros(9, k, dtype=torch.int64, device=dev),
           torch.zeros(9, k, device=dev))
