"""CPU: the drop-in runtime module keeps the reference's dispatch behaviour (kernel/exl3_grouped_runtime.py:86-112)
and the reference's unchanged hook (kernel/patch_exl3_grouped.py) loads it."""
import logging
import os
import sys
import types

import pytest
import torch

import exl3_grouped_runtime as rt
from conftest import PKG

REF = os.environ.get("EXL3_REFERENCE_DIR", "")


class FakeOV(types.ModuleType):
    SWIGLU_LIMIT_DEFAULT = 7.0

    def __init__(self):
        super().__init__("fake_ov")
        self.calls = []

        def original(x, topk_ids, topk_weights, layer, *, limit=7.0, fused=None):
            self.calls.append(("original", x.shape, limit, fused))
            return torch.full_like(x, -1.0)

        self.apply_exl3_experts = original


class Layer:
    def __init__(self, cap=128, with_trellis=True, expert_map=None):
        self._exl3_fused_temps = [torch.zeros(1, cap)]
        if with_trellis:
            self.w13_trellis = torch.zeros(4, 2, 1, 1, 64, dtype=torch.int16)
        self.expert_map = expert_map


@pytest.fixture
def installed(monkeypatch):
    ov = FakeOV()
    seen = []

    def fake_grouped(x2d, ids, weights, layer, limit):
        seen.append((x2d.shape, ids.dtype, ids.shape, weights.shape, limit))
        return torch.ones(x2d.shape, dtype=torch.float32)

    monkeypatch.setattr(rt, "grouped_prefill", fake_grouped)
    monkeypatch.setattr(rt, "_load_ext", lambda: None)
    monkeypatch.setattr(rt, "_logged", False)
    rt.install(ov)
    return ov, seen


def test_prefill_calls_take_the_grouped_path(installed):
    ov, seen = installed
    layer = Layer(cap=128)
    x = torch.zeros(1, 300, 64, dtype=torch.bfloat16)
    ids = torch.zeros(1, 300, 8, dtype=torch.int32)
    w = torch.ones(1, 300, 8)
    out = ov.apply_exl3_experts(x, ids, w, layer, limit=5.0)
    assert seen == [(torch.Size([300, 64]), torch.int64, torch.Size([300, 8]), torch.Size([300, 8]), 5.0)]
    # the reference returns [tokens, hidden] in x's dtype (kernel/exl3_grouped_runtime.py:99-107)
    assert out.dtype == torch.bfloat16 and out.shape == (300, 64) and bool((out == 1).all())
    assert layer._exl3_last_apply == "grouped"
    assert ov.calls == []


@pytest.mark.parametrize("layer,tokens", [(Layer(cap=128), 128), (Layer(cap=128, expert_map=torch.zeros(4)), 300),
                                          (Layer(cap=128, with_trellis=False), 300)])
def test_other_calls_keep_the_original_path(installed, layer, tokens):
    ov, seen = installed
    x = torch.zeros(tokens, 64)
    out = ov.apply_exl3_experts(x, torch.zeros(tokens, 8, dtype=torch.long), torch.ones(tokens, 8), layer, fused=True)
    assert seen == [] and ov.calls and ov.calls[0][3] is True
    assert bool((out == -1).all())


def test_engaged_is_logged_once(installed, caplog):
    ov, _ = installed
    caplog.set_level(logging.INFO, logger="vllm.exl3.grouped")
    for _ in range(3):
        ov.apply_exl3_experts(torch.zeros(300, 64), torch.zeros(300, 8, dtype=torch.long), torch.ones(300, 8), Layer())
    assert sum("engaged" in r.message for r in caplog.records) == 1


def test_empty_routing_returns_zeros_without_launch(monkeypatch):
    monkeypatch.setattr(rt, "_load_ext", lambda: None)
    layer = types.SimpleNamespace(w13_trellis=torch.zeros(4, 2, 8, 8, 64, dtype=torch.int16),
                                  _exl3_intermediate_local=128)
    out = rt.grouped_prefill(torch.zeros(0, 128), torch.zeros(0, 8, dtype=torch.long), torch.zeros(0, 8), layer, 7.0)
    assert out.shape == (0, 128) and out.dtype == torch.float32


def test_small_batch_switch_sends_calls_at_or_below_the_cap_through_the_grouped_pipeline(monkeypatch):
    ov = FakeOV()
    seen = []

    def fake_small(x2d, ids, weights, layer, limit, max_tokens):
        seen.append((tuple(x2d.shape), ids.dtype, limit, max_tokens))
        return torch.full(x2d.shape, 2.0, dtype=torch.float32)

    monkeypatch.setenv("EXL3_GROUPED_SMALL_BATCH", "1")
    monkeypatch.setattr(rt, "small_batch_prefill", fake_small)
    monkeypatch.setattr(rt, "grouped_prefill", lambda *a, **k: pytest.fail("prefill path taken"))
    monkeypatch.setattr(rt, "_load_ext", lambda: None)
    rt.install(ov)
    layer = Layer(cap=128)
    x = torch.zeros(7, 64, dtype=torch.float16)
    # the switch only applies to CUDA tensors: make the CPU tensor look like one for the dispatch
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    out = ov.apply_exl3_experts(x, torch.zeros(7, 8, dtype=torch.int32), torch.ones(7, 8), layer, limit=6.0)
    assert seen == [((7, 64), torch.int64, 6.0, 128)]
    assert out.dtype == torch.float16 and bool((out == 2).all()) and layer._exl3_last_apply == "grouped-small-batch"
    # expert-parallel layers and layers without trellis tensors still keep the original path
    for other in (Layer(cap=128, expert_map=torch.zeros(4)), Layer(cap=128, with_trellis=False)):
        assert bool((ov.apply_exl3_experts(x, torch.zeros(7, 8, dtype=torch.long), torch.ones(7, 8), other) == -1).all())
    assert len(seen) == 1 and len(ov.calls) == 2


def test_small_batch_switch_is_off_by_default(monkeypatch):
    monkeypatch.delenv("EXL3_GROUPED_SMALL_BATCH", raising=False)
    assert not rt.small_batch_enabled()
    monkeypatch.setenv("EXL3_GROUPED_SMALL_BATCH", "0")
    assert not rt.small_batch_enabled()
    monkeypatch.setenv("EXL3_GROUPED_SMALL_BATCH", "1")
    assert rt.small_batch_enabled()


def test_hook_contract_installs_this_runtime(monkeypatch):
    """The contract of the reference's hook block (kernel/patch_exl3_grouped.py:12-21), restated: with
    EXL3_GROUPED_PREFILL != "0", put dirname(EXL3_GROUPED_SRC) on sys.path, import exl3_grouped_runtime and
    call install(module).  Pointing EXL3_GROUPED_SRC into this package must install THIS runtime."""
    monkeypatch.setenv("EXL3_GROUPED_PREFILL", "1")
    monkeypatch.setenv("EXL3_GROUPED_SRC", os.path.join(PKG, "exl3_grouped_runtime.py"))
    monkeypatch.setattr(rt, "_load_ext", lambda: None)
    ov = FakeOV()
    original = ov.apply_exl3_experts
    monkeypatch.setattr(sys, "path", list(sys.path))
    if os.environ.get("EXL3_GROUPED_PREFILL", "0") != "0":
        src_dir = os.path.dirname(os.environ["EXL3_GROUPED_SRC"])
        if src_dir not in sys.path:
            sys.path.insert(0, src_dir)
        import exl3_grouped_runtime as gp_rt
        gp_rt.install(ov)
    assert ov.apply_exl3_experts is not original
    assert ov.apply_exl3_experts.__name__ == "apply_exl3_experts_grouped"
    assert sys.modules["exl3_grouped_runtime"].__file__.startswith(PKG)


@pytest.mark.skipif(not REF or not os.path.isdir(REF), reason="EXL3_REFERENCE_DIR (a reference checkout) not set")
def test_reference_hook_installs_this_runtime(monkeypatch):
    """Execute the hook block that kernel/patch_exl3_grouped.py appends, against a fake overlay module,
    with EXL3_GROUPED_SRC pointing into this package: it must import and install THIS runtime."""
    src = open(os.path.join(REF, "kernel", "patch_exl3_grouped.py")).read()
    block = src.split("block = f'''", 1)[1].split("'''", 1)[0].replace("{marker}", "# hook")
    monkeypatch.setenv("EXL3_GROUPED_PREFILL", "1")
    monkeypatch.setenv("EXL3_GROUPED_SRC", os.path.join(PKG, "exl3_grouped_runtime.py"))
    ov = FakeOV()
    ov.__dict__["__name__"] = "fake_ov_for_hook"
    monkeypatch.setitem(sys.modules, "fake_ov_for_hook", ov)
    monkeypatch.setattr(rt, "_load_ext", lambda: None)
    original = ov.apply_exl3_experts
    exec(compile(block, "patch_exl3_grouped.py:block", "exec"), ov.__dict__)
    assert ov.apply_exl3_experts is not original
    assert ov.apply_exl3_experts.__name__ == "apply_exl3_experts_grouped"
    assert sys.modules["exl3_grouped_runtime"].__file__.startswith(PKG)
