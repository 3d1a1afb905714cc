"""CPU: argument checks of the dense / shared-expert entry points (no kernel runs)."""
import pytest
import torch

import exl3_dense
import exl3_grouped_runtime as rt
import synth


def test_exl3_linear_rejects_mismatched_shapes():
    x = torch.zeros(4, 256, dtype=torch.float16)
    tr = torch.zeros(16, 8, 64, dtype=torch.int16)
    with pytest.raises(RuntimeError, match="out_dtype"):
        exl3_dense.exl3_linear(x, tr, torch.ones(256).half(), torch.ones(128).half(), out_dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="K / N mismatch"):
        exl3_dense.exl3_linear(x, tr, torch.ones(128).half(), torch.ones(128).half())
    with pytest.raises(RuntimeError, match="K / N mismatch"):
        exl3_dense.exl3_linear(x, tr, torch.ones(256).half(), torch.ones(256).half())
    with pytest.raises(RuntimeError, match=r"\[K/16, N/16, 64\]"):
        exl3_dense.exl3_linear(x, tr.view(16, 8, 8, 8), torch.ones(256).half(), torch.ones(128).half())


def test_dense_mlp_needs_one_expert_and_out_is_checked():
    two = synth.make_layer(2, 128, 128, seed=1)
    with pytest.raises(RuntimeError, match="one expert"):
        exl3_dense.dense_mlp_prefill(torch.zeros(4, 128, dtype=torch.float16), two, 7.0)
    one = synth.make_layer(1, 128, 128, seed=1)
    with pytest.raises(RuntimeError, match="contiguous fp32"):
        rt.grouped_prefill(torch.zeros(4, 128, dtype=torch.float16), torch.zeros(4, 1, dtype=torch.int64),
                           torch.ones(4, 1), one, 7.0, out=torch.zeros(4, 64))
