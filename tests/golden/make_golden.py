#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own Python code on the CPU.

Run where a checkout of the reference is available (its directory from --ref or EXL3_REFERENCE_DIR):

    python tests/golden/make_golden.py --ref /path/to/reference

What is executed from the reference, unmodified (loaded from its files; nothing is copied into this
repository):

* kernel/exl3_grouped_runtime.py — the whole module is imported and ``grouped_prefill`` runs on CPU
  tensors.  Its extension handle ``_ext`` is replaced by a recorder whose stage functions are the CPU
  oracle, so the reference's own host code computes the expert sort (argsort stable, token/weight/
  expert arrays, counts, expert_row0, max_blocks) and wires every stage call; the recorder captures
  those tensors and arguments.
* harness/proto_fp8.py:61-64 (the Sylvester H128 builder), :66-76 ``full_weight`` (the exllamav3
  weight convention) and :123-134 ``ref_fp16`` (the per-expert reference loop) — extracted with ``ast``
  and executed with ``ext.reconstruct`` bound to the oracle's trellis decode (exllamav3 is absent, so
  the decode itself is this library's documented codebook: parity with EXL3 checkpoints is unpinned).
* kernel/test_grouped.py:95-106 ``routing_skewed`` and harness/test_exl3_moe_op.py:119-150
  ``routing`` / ``routing_skewed`` — executed to produce reference routings.

The fixtures are small .npz files; the tests read only them (never the reference checkout).
"""
from __future__ import annotations

import argparse
import ast
import importlib.util
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "glm53-exl3-prefill_b200"))
import oracle  # noqa: E402
import synth  # noqa: E402

LIMIT = 7.0


# ------------------------------------------------------------------------------------ reference code loaders
def _module_statements(path: str, pred) -> str:
    src = open(path).read()
    tree = ast.parse(src)
    return "\n".join(ast.get_source_segment(src, n) for n in tree.body if pred(n))


def load_functions(path: str, names, ns: dict) -> dict:
    code = _module_statements(path, lambda n: isinstance(n, ast.FunctionDef) and n.name in names)
    exec(compile(code, path, "exec"), ns)
    return ns


def reference_h128(ref: str) -> torch.Tensor:
    """harness/proto_fp8.py:61-64 executed as written."""
    path = os.path.join(ref, "harness", "proto_fp8.py")
    src = open(path).read()
    tree = ast.parse(src)
    stmts = [n for n in tree.body if 61 <= n.lineno <= 64]
    code = "\n".join(ast.get_source_segment(src, n) for n in stmts)
    assert "H128" in code and "while" in code, "proto_fp8.py H128 builder not found at :61-64"
    ns = dict(torch=torch, math=math, dev=torch.device("cpu"))
    exec(compile(code, path, "exec"), ns)
    return ns["H128"]


class _OracleReconstructExt:
    """Stands in for exllamav3_ext: reconstruct(w, trellis, K, mcg, mul1) with the oracle's decode."""

    @staticmethod
    def reconstruct(w, trellis, K, mcg, mul1):
        assert K == 4 and mcg and not mul1
        w.copy_(torch.from_numpy(oracle.reconstruct(trellis.numpy()).copy()))


def reference_loop_fns(ref: str):
    ns = dict(torch=torch, math=math, dev=torch.device("cpu"), ext=_OracleReconstructExt())
    ns["H128"] = reference_h128(ref)
    load_functions(os.path.join(ref, "harness", "proto_fp8.py"), {"full_weight", "ref_fp16"}, ns)
    return ns


def reference_runtime(ref: str):
    path = os.path.join(ref, "kernel", "exl3_grouped_runtime.py")
    spec = importlib.util.spec_from_file_location("reference_exl3_grouped_runtime", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# ------------------------------------------------------------------------------------ oracle-backed recorder
class Recorder:
    """The extension object handed to the reference's grouped_prefill: records every call and computes
    each stage with the CPU oracle so the reference's host code runs end to end."""

    def __init__(self):
        self.calls = []

    def build_blocks(self, counts, block_expert, block_row0, meta):
        self.calls.append(("build_blocks", dict(counts=counts.clone(), max_blocks=block_expert.numel())))
        be, br, m = oracle.build_blocks(counts.numpy(), block_expert.numel(), block_row0.numpy())
        block_expert.copy_(torch.from_numpy(be))
        block_row0.copy_(torch.from_numpy(br))
        meta.copy_(torch.from_numpy(m))

    def row_had(self, src, dst, token_sorted, expert_of_row, suh, gather):
        self.calls.append(("row_had", dict(token_sorted=token_sorted.clone(), expert_of_row=expert_of_row.clone(),
                                           suh_stride=suh.stride(0), gather=bool(gather))))
        out = oracle.row_had(src.numpy(), token_sorted.numpy(), expert_of_row.numpy(), suh.numpy(), gather=gather)
        dst.copy_(torch.from_numpy(out.copy()))

    def act_had(self, gu, act, expert_of_row, suh_down, limit):
        self.calls.append(("act_had", dict(limit=float(limit))))
        act.copy_(torch.from_numpy(oracle.act_had(gu.numpy(), expert_of_row.numpy(), suh_down.numpy(), limit).copy()))

    def grouped_gemm(self, a, packed_gate, packed_up, svh_gate, svh_up, block_expert, block_row0, counts, expert_row0,
                     token_sorted, route_weight, out, mode):
        self.calls.append(("grouped_gemm", dict(mode=int(mode), weight_sorted=route_weight.clone(),
                                                two=packed_up is not None)))
        a_np = a.numpy()
        E = packed_gate.shape[0]
        N = packed_gate.shape[2] * 16
        for e in range(E):
            c = int(counts[e])
            if c == 0:
                continue
            r0 = int(expert_row0[e])
            rows = a_np[r0:r0 + c]
            if mode == 0:
                mats = [(packed_gate, svh_gate, 0)] + ([(packed_up, svh_up, N)] if packed_up is not None else [])
                for pk, sv, col in mats:
                    y = oracle.fat_gemm_ref(rows, pk[e].numpy(), sv[e].numpy())
                    out[r0:r0 + c, col:col + N] = torch.from_numpy(oracle.f2h(y).copy())
            else:
                y = oracle.fat_gemm_ref(rows, packed_gate[e].numpy(), svh_gate[e].numpy())
                o = out.numpy()
                np.add.at(o, token_sorted[r0:r0 + c].numpy(),
                          y * route_weight[r0:r0 + c].numpy().astype(np.float32)[:, None])


def _layer_np(layer):
    return oracle.Layer(layer.w13_trellis.numpy(), layer.w13_suh.numpy(), layer.w13_svh.numpy(),
                        layer.w2_trellis.numpy(), layer.w2_suh.numpy(), layer.w2_svh.numpy())


# ------------------------------------------------------------------------------------ fixtures
def sort_cases(ref: str):
    """Routing cases -> the reference runtime's sort outputs."""
    tg = load_functions(os.path.join(ref, "kernel", "test_grouped.py"), {"routing_skewed"},
                        dict(torch=torch, dev=torch.device("cpu")))
    hm = load_functions(os.path.join(ref, "harness", "test_exl3_moe_op.py"), {"routing", "routing_skewed"},
                        dict(torch=torch, dev=torch.device("cpu")))
    cases = []

    def add(name, ids, w, E):
        cases.append((name, ids.to(torch.int64), w, E))

    ids, w = synth.routing("uniform", 256, 16, 4, seed=2)
    add("cfg0_uniform", ids, w, 16)
    ids, w = synth.routing("zipf", 512, 288, 8, seed=3)
    add("zipf_t512_e288", ids, w, 288)
    tg.update(topk=8, E=32)
    ids, w = tg["routing_skewed"](64, 7)
    add("ref_skewed_t64_e32", ids, w, 32)
    hm.update(topk=8, n_load=64)
    ids, w = hm["routing"](512, 5, fat_expert=7, fat_rows=400)
    add("ref_fat_expert7_t512_e64", ids, w, 64)
    ids, w = hm["routing_skewed"](96, 11)
    add("ref_opskewed_t96_e64", ids, w, 64)
    add("single_expert", torch.zeros(5, 1, dtype=torch.int64), torch.ones(5, 1), 1)
    g = torch.Generator().manual_seed(9)
    add("mostly_empty_e300", torch.randint(0, 300, (3, 2), generator=g), torch.rand(3, 2, generator=g), 300)
    ids, w = synth.routing("uniform", 200, 1024, 8, seed=4)
    add("e1024_t200", ids, w, 1024)
    ids, w = synth.routing("zipf", 1, 288, 8, seed=5)
    add("one_token", ids, w, 288)
    add("hot_dup_400rows", torch.full((100, 4), 3, dtype=torch.int64), torch.rand(100, 4, generator=g), 8)
    ids, w = synth.routing("uniform", 300, 64, 6, seed=6)
    add("fp16_weights", ids, w.to(torch.float16), 64)
    ids, w = synth.routing("uniform", 300, 64, 6, seed=7)
    add("bf16_weights", ids, w.to(torch.bfloat16), 64)
    ids, w = synth.routing("zipf", 4096, 288, 8, seed=8)
    add("zipf_t4096_e288", ids, w, 288)

    mod = reference_runtime(ref)
    out = {}
    for name, ids, w, E in cases:
        T, k = ids.shape
        rec = Recorder()
        mod._ext = rec
        d, f = 128, 128
        layer = types.SimpleNamespace(
            w13_trellis=torch.zeros(E, 2, d // 16, f // 16, 64, dtype=torch.int16),
            w13_suh=torch.ones(E, 2, d, dtype=torch.float16), w13_svh=torch.ones(E, 2, f, dtype=torch.float16),
            w2_trellis=torch.zeros(E, f // 16, d // 16, 64, dtype=torch.int16),
            w2_suh=torch.ones(E, f, dtype=torch.float16), w2_svh=torch.ones(E, d, dtype=torch.float16),
            _exl3_intermediate_local=f)
        x = torch.zeros(T, d, dtype=torch.float16)
        mod.grouped_prefill(x, ids, w, layer, LIMIT)
        bb = [c for c in rec.calls if c[0] == "build_blocks"][0][1]
        rh = [c for c in rec.calls if c[0] == "row_had"][0][1]
        gg = [c for c in rec.calls if c[0] == "grouped_gemm"][0][1]
        counts = bb["counts"].numpy()
        max_blocks = bb["max_blocks"]
        sentinel = np.full(max_blocks, -7, dtype=np.int32)
        be, br, meta = oracle.build_blocks(counts, max_blocks, sentinel)
        wdt = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[w.dtype]
        wbits = w.float().numpy() if wdt == "f32" else w.view(torch.int16).numpy().view(np.uint16)
        out[name] = dict(ids=ids.numpy(), weights=wbits, weight_dtype=np.array(wdt), n_experts=np.int32(E),
                         token_sorted=rh["token_sorted"].numpy(), expert_of_row=rh["expert_of_row"].numpy(),
                         weight_sorted=gg["weight_sorted"].numpy().view(np.uint16), counts=counts,
                         expert_row0=None, max_blocks=np.int32(max_blocks), block_expert=be, block_row0=br,
                         meta=meta)
        er0 = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
        out[name]["expert_row0"] = er0
    return out


def layer_case(ref: str, E, d, f, k, T, routing_kind, seed, sv_scale):
    """One layer: inputs (seeded), the reference runtime's output with oracle stages, the reference
    per-expert loop (proto_fp8 ref_fp16) and the reference full_weight of expert 0's gate."""
    layer = synth.make_layer(E, d, f, seed=seed, sv_scale=sv_scale)
    x = synth.make_x(T, d, seed=seed + 1)
    ids, w = synth.routing(routing_kind, T, E, k, seed=seed + 2)
    mod = reference_runtime(ref)
    rec = Recorder()
    mod._ext = rec
    out_grouped = mod.grouped_prefill(x, ids, w, layer, LIMIT).numpy()

    ns = reference_loop_fns(ref)

    def lin(e, which):
        if which == "down":
            pk, suh, svh = layer.w2_trellis[e], layer.w2_suh[e], layer.w2_svh[e]
            K, N = f, d
        else:
            j = 0 if which == "gate" else 1
            pk, suh, svh = layer.w13_trellis[e, j], layer.w13_suh[e, j], layer.w13_svh[e, j]
            K, N = d, f
        return types.SimpleNamespace(in_features=K, out_features=N, trellis=pk, K=4, mcg=True, mul1=False,
                                     suh=suh, svh=svh)

    wfull = []
    for e in range(E):
        g = ns["full_weight"](lin(e, "gate"))
        u = ns["full_weight"](lin(e, "up"))
        dn = ns["full_weight"](lin(e, "down"))
        wfull.append((g.half(), u.half(), dn.half()))
        if e == 0:
            w0_gate = g.numpy().copy()
    ns.update(Wfull=wfull, E=E, hidden=d, LIMIT=LIMIT)
    out_loop = ns["ref_fp16"](x, ids, w).numpy()
    return dict(E=np.int32(E), d=np.int32(d), f=np.int32(f), k=np.int32(k), T=np.int32(T), seed=np.int32(seed),
                sv_scale=np.float32(sv_scale), routing=np.array(routing_kind), limit=np.float32(LIMIT),
                x=x.numpy(), ids=ids.numpy(), weights=w.numpy(),
                w13_checksum=np.int64(layer.w13_trellis.to(torch.int64).sum().item()),
                w2_checksum=np.int64(layer.w2_trellis.to(torch.int64).sum().item()),
                out_grouped_ref_runtime=out_grouped, out_ref_loop=out_loop, full_weight_e0_gate=w0_gate)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("EXL3_REFERENCE_DIR"),
                    help="checkout of the reference (default: $EXL3_REFERENCE_DIR)")
    a = ap.parse_args()
    ref = a.ref
    if not ref or not os.path.isdir(ref):
        ap.error(f"reference checkout not found (--ref or EXL3_REFERENCE_DIR): {ref!r}")
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    np.save(os.path.join(HERE, "h128_reference.npy"), reference_h128(ref).numpy())

    cases = sort_cases(ref)
    flat = {}
    for name, dct in cases.items():
        for key, val in dct.items():
            flat[f"{name}__{key}"] = val
    flat["case_names"] = np.array(sorted(cases))
    np.savez_compressed(os.path.join(HERE, "sort_cases.npz"), **flat)

    small = layer_case(ref, E=8, d=256, f=128, k=4, T=64, routing_kind="uniform", seed=10, sv_scale=1.0)
    np.savez_compressed(os.path.join(HERE, "layer_small.npz"), **small)
    small_real = layer_case(ref, E=8, d=256, f=256, k=4, T=96, routing_kind="zipf", seed=20, sv_scale=0.05)
    np.savez_compressed(os.path.join(HERE, "layer_small_unsaturated.npz"), **small_real)
    cfg0 = layer_case(ref, E=16, d=1024, f=512, k=4, T=256, routing_kind="uniform", seed=30, sv_scale=1.0)
    cfg0.pop("full_weight_e0_gate")
    cfg0.pop("out_grouped_ref_runtime")      # reproducible from the small cases' pinned wiring; keeps the file small
    np.savez_compressed(os.path.join(HERE, "layer_cfg0.npz"), **cfg0)
    for fn in sorted(os.listdir(HERE)):
        if fn.endswith((".npz", ".npy")):
            print(f"{fn}: {os.path.getsize(os.path.join(HERE, fn)) / 1024:.0f} KB")


if __name__ == "__main__":
    main()
