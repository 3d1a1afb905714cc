"""CPU: host logic of the small-batch path (token buckets, argument checks) and of the router front-end
module (no kernel runs)."""
import pytest
import torch

import exl3_decode
import exl3_router
import synth


def test_buckets_are_powers_of_two_covering_the_call():
    assert [exl3_decode.GraphedPrefill.bucket(t) for t in (1, 2, 3, 4, 5, 8, 9, 33, 64)] == \
        [1, 2, 4, 4, 8, 8, 16, 64, 64]


def test_graphed_prefill_checks_its_arguments_before_any_capture():
    layer = synth.make_layer(4, 128, 128, seed=1)
    gp = exl3_decode.GraphedPrefill(layer, 7.0, topk=2, max_tokens=8, device=torch.device("cpu"))
    with pytest.raises(RuntimeError, match="exceed max_tokens"):
        gp(torch.zeros(9, 128, dtype=torch.float16), torch.zeros(9, 2, dtype=torch.int64), torch.zeros(9, 2))
    with pytest.raises(RuntimeError, match=r"\[T, topk\]"):
        gp(torch.zeros(3, 128, dtype=torch.float16), torch.zeros(3, 1, dtype=torch.int64), torch.zeros(3, 1))
    out = gp(torch.zeros(0, 128, dtype=torch.float16), torch.zeros(0, 2, dtype=torch.int64), torch.zeros(0, 2))
    assert tuple(out.shape) == (0, 128) and not gp._graphs
    with pytest.raises(RuntimeError, match="max_tokens must be positive"):
        exl3_decode.GraphedPrefill(layer, 7.0, topk=2, max_tokens=0, device=torch.device("cpu"))


def test_router_module_checks():
    w = torch.zeros(16, 128)
    r = exl3_router.NoauxTcRouter(w, torch.zeros(16), topk=4)
    assert r.weight.dtype == torch.float16 and r.bias.dtype == torch.float32 and r.n_experts == 16
    with pytest.raises(RuntimeError, match="must be CUDA"):
        r.route(torch.zeros(4, 128))
    layer = synth.make_layer(8, 128, 128, seed=2)
    with pytest.raises(RuntimeError, match="disagree on the number of experts"):
        exl3_router.moe_prefill_from_hidden(torch.zeros(4, 128), r, layer, 7.0)
