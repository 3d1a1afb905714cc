"""CPU oracle for the routed-expert EXL3 MoE prefill path (numpy + the C restatement in exl3_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module; the product (the package's C-ABI library and its Python shim) never
does.  It is the checker, never the thing measured or shipped.

Two restatements of the reference live here:

* ``grouped_staged`` — the five-stage grouped pipeline with the reference's rounding points
  (kernel/exl3_grouped_runtime.py:50-83, kernel/exl3_grouped_prefill.cu:63-279): stable expert sort,
  block table, row_had (fp16), gate|up trellis GEMM with the H128*svh epilogue (fp16), act_had
  (fp16), down GEMM with the route-weighted fp32 scatter.
* ``moe_loop`` — the reference per-expert loop (harness/proto_fp8.py:123-134, the in-tree
  restatement of the overlay's apply_exl3_python_loop) on real-domain weights built with the
  exllamav3 convention W = diag(suh) H W' H diag(svh) (harness/proto_fp8.py:61-76).

``fat_gemm_ref`` is the GEMM-stage reference of kernel/test_fat_v2.py:87-95 (reconstruct -> fp32
matmul -> H128 * svh) and its scatter form kernel/test_fat_v2.py:135.

Parity of the trellis codebook with real EXL3 checkpoints is UNPINNED (exllamav3's decode source is
absent); see the header of exl3_oracle.c.  Everything downstream of the decode is pinned by
tests/golden (generated from the reference's own Python code).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "libexl3_oracle.so")
SRC = os.path.join(HERE, "exl3_oracle.c")
HAD_SCALE = np.float32(0.088388347648)

_lib = None


def build(force: bool = False) -> str:
    """Compile exl3_oracle.c into oracle/_build/libexl3_oracle.so (gcc, OpenMP, no fast-math)."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(SRC):
        tmp = LIB_PATH + ".tmp%d" % os.getpid()
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-fno-fast-math", "-ffp-contract=off",
                               "-o", tmp, SRC, "-lm"])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I32 = ctypes.c_int
        F = ctypes.c_float
        sig = {
            "orc_f2h": ([F], ctypes.c_uint16),
            "orc_h2f": ([ctypes.c_uint16], F),
            "orc_f2h_array": ([P, P, I64], None),
            "orc_h2f_array": ([P, P, I64], None),
            "orc_trellis_state_bitwise": ([P, I32], ctypes.c_uint32),
            "orc_trellis_state": ([P, I32], ctypes.c_uint32),
            "orc_codebook": ([ctypes.c_uint32], ctypes.c_uint16),
            "orc_decode_tile": ([P, P], None),
            "orc_reconstruct": ([P, I32, I32, P], None),
            "orc_reconstruct_f32": ([P, I32, I32, P], None),
            "orc_had128": ([P], None),
            "orc_had_epilogue": ([P, I64, I32, I64, P], None),
            "orc_row_had": ([P, P, I64, I32, P, P, P, I64, I32], None),
            "orc_swiglu": ([F, F, F], F),
            "orc_act_had": ([P, P, I64, I32, P, P, I64, F], None),
            "orc_build_blocks": ([P, I32, I32, P, P, P], None),
            "orc_route_sort": ([P, P, I32, I64, I32, I32, P, P, P, P, P], I64),
        }
        for name, (args, res) in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = res
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _u16(a: np.ndarray) -> np.ndarray:
    """View an fp16/int16 array as uint16 bits (C-contiguous)."""
    return np.ascontiguousarray(a).view(np.uint16)


# ------------------------------------------------------------------------------------ primitives
def f2h(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f2h_array(_p(x), _p(out), x.size)
    return out.view(np.float16)


def decode_tile(words: np.ndarray) -> np.ndarray:
    """64 int16 words -> 256 fp16 weights in tile order j (k = j % 16, n = j // 16)."""
    w = _u16(words.reshape(64))
    out = np.empty(256, dtype=np.uint16)
    lib().orc_decode_tile(_p(w), _p(out))
    return out.view(np.float16)


def reconstruct(packed: np.ndarray, dtype=np.float16) -> np.ndarray:
    """packed [tiles_k, tiles_n, 64] int16 -> W' [16*tiles_k, 16*tiles_n] (fp16, or fp32 if asked)."""
    tk, tn, w = packed.shape
    assert w == 64
    src = _u16(packed)
    if dtype == np.float32:
        out = np.empty((16 * tk, 16 * tn), dtype=np.float32)
        lib().orc_reconstruct_f32(_p(src), tk, tn, _p(out))
        return out
    out = np.empty((16 * tk, 16 * tn), dtype=np.uint16)
    lib().orc_reconstruct(_p(src), tk, tn, _p(out))
    return out.view(np.float16)


def had128_matrix() -> np.ndarray:
    """Sylvester H128 / sqrt(128) (harness/proto_fp8.py:61-64)."""
    h = np.ones((1, 1), dtype=np.float64)
    while h.shape[0] < 128:
        h = np.block([[h, h], [h, -h]])
    return (h / np.sqrt(128.0)).astype(np.float32)


def had_epilogue(y: np.ndarray, svh: np.ndarray) -> np.ndarray:
    """In place on fp32 [M, N]: per 128 columns H128 * 0.088388347648 * svh."""
    assert y.dtype == np.float32 and y.flags["C_CONTIGUOUS"]
    M, N = y.shape
    lib().orc_had_epilogue(_p(y), M, N, N, _p(_u16(svh.astype(np.float16))))
    return y


def row_had(src: np.ndarray, token_sorted: np.ndarray, expert_of_row: np.ndarray, suh: np.ndarray,
            gather: bool = True) -> np.ndarray:
    """src fp16 [T, K]; suh fp16 [E, K] (any row stride) -> fp16 [R, K]."""
    R = token_sorted.shape[0] if gather else src.shape[0]
    K = src.shape[1]
    suh_c = np.ascontiguousarray(suh.astype(np.float16))
    dst = np.empty((R, K), dtype=np.uint16)
    ts = np.ascontiguousarray(token_sorted if gather else np.zeros(1), dtype=np.int64)
    eor = np.ascontiguousarray(expert_of_row, dtype=np.int32)
    lib().orc_row_had(_p(_u16(src)), _p(dst), R, K, _p(ts), _p(eor), _p(_u16(suh_c)), suh_c.shape[1],
                      1 if gather else 0)
    return dst.view(np.float16)


def act_had(gu: np.ndarray, expert_of_row: np.ndarray, suh_down: np.ndarray, limit: float) -> np.ndarray:
    """gu fp16 [R, 2I] -> act fp16 [R, I]."""
    R, I2 = gu.shape
    I = I2 // 2
    suh_c = np.ascontiguousarray(suh_down.astype(np.float16))
    act = np.empty((R, I), dtype=np.uint16)
    eor = np.ascontiguousarray(expert_of_row, dtype=np.int32)
    lib().orc_act_had(_p(_u16(gu)), _p(act), R, I, _p(eor), _p(_u16(suh_c)), suh_c.shape[1], float(limit))
    return act.view(np.float16)


def build_blocks(counts: np.ndarray, max_blocks: int, block_row0_init: np.ndarray | None = None):
    """-> (block_expert, block_row0, meta) int32, as build_blocks_kernel leaves them."""
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    be = np.zeros(max_blocks, dtype=np.int32)
    br = np.zeros(max_blocks, dtype=np.int32) if block_row0_init is None else block_row0_init.astype(np.int32).copy()
    meta = np.zeros(2, dtype=np.int32)
    lib().orc_build_blocks(_p(counts), counts.shape[0], max_blocks, _p(be), _p(br), _p(meta))
    return be, br, meta


def route_sort(ids: np.ndarray, weights: np.ndarray, n_experts: int):
    """ids int64 [T, k], weights [T, k] (fp32/fp16/bf16-as-uint16 not supported here: fp32/fp16) ->
    dict(token_sorted int64 [R], weight_sorted fp16 [R], expert_of_row int32 [R], counts int32 [E],
    expert_row0 int32 [E], invalid int)."""
    T, k = ids.shape
    ids_c = np.ascontiguousarray(ids, dtype=np.int64)
    if weights.dtype == np.float32:
        w, wd = np.ascontiguousarray(weights), 0
    elif weights.dtype == np.float16:
        w, wd = np.ascontiguousarray(weights).view(np.uint16), 1
    else:
        raise TypeError("weights must be float32 or float16")
    R = T * k
    ts = np.zeros(R, dtype=np.int64)
    ws = np.zeros(R, dtype=np.uint16)
    eor = np.zeros(R, dtype=np.int32)
    counts = np.zeros(max(n_experts, 1), dtype=np.int32)
    row0 = np.zeros(max(n_experts, 1), dtype=np.int32)
    invalid = lib().orc_route_sort(_p(ids_c), _p(w), wd, T, k, n_experts, _p(ts), _p(ws), _p(eor),
                                   _p(counts), _p(row0))
    return dict(token_sorted=ts, weight_sorted=ws.view(np.float16), expert_of_row=eor,
                counts=counts[:n_experts], expert_row0=row0[:n_experts], invalid=int(invalid))


# ------------------------------------------------------------------------------------ GEMM stage
def fat_gemm_ref(a: np.ndarray, packed: np.ndarray, svh: np.ndarray, w: np.ndarray | None = None) -> np.ndarray:
    """kernel/test_fat_v2.py:87-95: reconstruct -> fp32 matmul -> H128 * svh.  a fp16 [M, K]."""
    if w is None:
        w = reconstruct(packed)
    y = np.ascontiguousarray(a.astype(np.float32) @ w.astype(np.float32))
    return had_epilogue(y, svh)


def fat_gemm_scatter_ref(a, packed, svh, token_idx, route_weight, out_rows):
    """kernel/test_fat_v2.py:135: zeros.index_add_(0, tok, ref * rw)."""
    y = fat_gemm_ref(a, packed, svh)
    out = np.zeros((out_rows, y.shape[1]), dtype=np.float32)
    np.add.at(out, token_idx, y * route_weight.astype(np.float32)[:, None])
    return out


# ------------------------------------------------------------------------------------ layer
class Layer:
    """Numpy view of the stacked layer tensors (kernel/test_grouped.py:76-81):
    w13_trellis [E,2,d/16,f/16,64] int16, w13_suh [E,2,d] fp16, w13_svh [E,2,f] fp16,
    w2_trellis [E,f/16,d/16,64] int16, w2_suh [E,f] fp16, w2_svh [E,d] fp16."""

    def __init__(self, w13_trellis, w13_suh, w13_svh, w2_trellis, w2_suh, w2_svh):
        self.w13_trellis = np.asarray(w13_trellis)
        self.w13_suh = np.asarray(w13_suh)
        self.w13_svh = np.asarray(w13_svh)
        self.w2_trellis = np.asarray(w2_trellis)
        self.w2_suh = np.asarray(w2_suh)
        self.w2_svh = np.asarray(w2_svh)
        self.E = self.w13_trellis.shape[0]
        self.d = self.w13_trellis.shape[2] * 16
        self.f = self.w13_trellis.shape[3] * 16
        self._dec = {}

    def decoded(self, e: int):
        """(W'_gate, W'_up, W'_down) fp16 for expert e (cached)."""
        if e not in self._dec:
            self._dec[e] = (reconstruct(self.w13_trellis[e, 0]), reconstruct(self.w13_trellis[e, 1]),
                            reconstruct(self.w2_trellis[e]))
        return self._dec[e]

    def full_weights(self, e: int):
        """Real-domain fp32 (gate [d,f], up [d,f], down [f,d]): diag(suh) H W' H diag(svh)."""
        g, u, dn = self.decoded(e)
        return (full_weight(g, self.w13_suh[e, 0], self.w13_svh[e, 0]),
                full_weight(u, self.w13_suh[e, 1], self.w13_svh[e, 1]),
                full_weight(dn, self.w2_suh[e], self.w2_svh[e]))


def full_weight(wq: np.ndarray, suh: np.ndarray, svh: np.ndarray) -> np.ndarray:
    """harness/proto_fp8.py:66-76 restated: [K, N] fp32 = diag(suh) . H . W' . H . diag(svh)."""
    K, N = wq.shape
    H = had128_matrix()
    w = wq.astype(np.float32)
    w = np.matmul(H, w.reshape(-1, 128, N)).reshape(K, N)
    w = w * suh.astype(np.float32)[:, None]
    w = np.matmul(w.reshape(K, -1, 128), H).reshape(K, N)
    w = w * svh.astype(np.float32)[None, :]
    return w


def _mm_f16(a16: np.ndarray, b16: np.ndarray) -> np.ndarray:
    """fp16 @ fp16 with fp32 accumulation, result rounded to fp16 (what a torch half matmul returns)."""
    return f2h(a16.astype(np.float32) @ b16.astype(np.float32))


def moe_loop(x16: np.ndarray, ids: np.ndarray, wts: np.ndarray, layer: Layer, limit: float,
             experts=None) -> np.ndarray:
    """Reference per-expert loop (harness/proto_fp8.py:123-134) -> fp32 [T, d]."""
    T = x16.shape[0]
    out = np.zeros((T, layer.d), dtype=np.float32)
    experts = range(layer.E) if experts is None else experts
    for e in experts:
        tok, kpos = np.nonzero(ids == e)
        if tok.size == 0:
            continue
        h = x16[tok]
        g, u, d = (w.astype(np.float16) for w in layer.full_weights(e))
        gate = _mm_f16(h, g).astype(np.float32)
        up = _mm_f16(h, u).astype(np.float32)
        gc = np.minimum(gate, np.float32(limit))
        act = gc / (np.float32(1.0) + np.exp(-gc)) * np.clip(up, -limit, limit).astype(np.float32)
        down = _mm_f16(f2h(act), d).astype(np.float32)
        np.add.at(out, tok, down * wts[tok, kpos].astype(np.float32)[:, None])
    return out


def grouped_staged(x16: np.ndarray, ids: np.ndarray, wts: np.ndarray, layer: Layer, limit: float,
                   return_stages: bool = False):
    """The five-stage grouped pipeline restated on the CPU -> fp32 [T, d] (and the stage tensors)."""
    T, k = ids.shape
    E, d, f = layer.E, layer.d, layer.f
    s = route_sort(ids, wts.astype(np.float32) if wts.dtype != np.float16 else wts, E)
    ts, eor, counts, row0 = s["token_sorted"], s["expert_of_row"], s["counts"], s["expert_row0"]
    R = int(counts.sum())
    h13 = row_had(x16, ts[:R], eor[:R], layer.w13_suh[:, 0], gather=True)
    gu = np.empty((R, 2 * f), dtype=np.float16)
    for e in range(E):
        c = int(counts[e])
        if c == 0:
            continue
        r0 = int(row0[e])
        wg, wu, _ = layer.decoded(e)
        gu[r0:r0 + c, :f] = f2h(fat_gemm_ref(h13[r0:r0 + c], None, layer.w13_svh[e, 0], w=wg))
        gu[r0:r0 + c, f:] = f2h(fat_gemm_ref(h13[r0:r0 + c], None, layer.w13_svh[e, 1], w=wu))
    act = act_had(gu, eor[:R], layer.w2_suh, limit)
    out = np.zeros((T, d), dtype=np.float32)
    wsorted = s["weight_sorted"].astype(np.float32)
    for e in range(E):
        c = int(counts[e])
        if c == 0:
            continue
        r0 = int(row0[e])
        _, _, wd = layer.decoded(e)
        y = fat_gemm_ref(act[r0:r0 + c], None, layer.w2_svh[e], w=wd)
        np.add.at(out, ts[r0:r0 + c], y * wsorted[r0:r0 + c, None])
    if return_stages:
        return out, dict(sort=s, h13=h13, gu=gu, act=act)
    return out


def token_rows(x16: np.ndarray, ids: np.ndarray, wts: np.ndarray, layer: Layer, limit: float, tokens,
               with_loop: bool = True):
    """Layer outputs for a subset of tokens only, at any layer size -> (grouped fp32 [n, d], loop fp32 [n, d]
    or None), n = len(tokens).

    Every stage of both restatements is row-wise, so a token's output depends only on its own routes:
    ``grouped`` equals ``grouped_staged(...)[tokens]`` (row_had -> fat-GEMM gate|up rounded to fp16 ->
    act_had -> fat-GEMM down, weighted by the fp16-rounded route weight and added in ascending expert
    order, the order of the sorted scatter), and ``loop`` equals ``moe_loop(...)[tokens]``.  Experts are
    decoded one at a time and not cached, so a 288-expert layer fits in memory."""
    tokens = np.asarray(tokens, dtype=np.int64)
    sub_ids = np.asarray(ids)[tokens]
    sub_w = np.asarray(wts)[tokens].astype(np.float32)
    n, d = tokens.shape[0], layer.d
    w16 = f2h(sub_w).astype(np.float32)                   # the sort's fp16 route weights
    out_g = np.zeros((n, d), dtype=np.float32)
    out_l = np.zeros((n, d), dtype=np.float32) if with_loop else None
    for e in np.unique(sub_ids[(sub_ids >= 0) & (sub_ids < layer.E)]):
        e = int(e)
        rows, kpos = np.nonzero(sub_ids == e)
        wg, wu, wd = (reconstruct(layer.w13_trellis[e, 0]), reconstruct(layer.w13_trellis[e, 1]),
                      reconstruct(layer.w2_trellis[e]))
        eor = np.full(rows.shape[0], e, dtype=np.int32)
        h13 = row_had(x16, tokens[rows], eor, layer.w13_suh[:, 0], gather=True)
        gu = np.concatenate([f2h(fat_gemm_ref(h13, None, layer.w13_svh[e, 0], w=wg)),
                             f2h(fat_gemm_ref(h13, None, layer.w13_svh[e, 1], w=wu))], axis=1)
        act = act_had(gu, eor, layer.w2_suh, limit)
        y = fat_gemm_ref(act, None, layer.w2_svh[e], w=wd)
        np.add.at(out_g, rows, y * w16[rows, kpos][:, None])
        if with_loop:
            g, u, dn = (full_weight(wq, su, sv).astype(np.float16) for wq, su, sv in
                        ((wg, layer.w13_suh[e, 0], layer.w13_svh[e, 0]), (wu, layer.w13_suh[e, 1], layer.w13_svh[e, 1]),
                         (wd, layer.w2_suh[e], layer.w2_svh[e])))
            h = x16[tokens[rows]]
            gate = _mm_f16(h, g).astype(np.float32)
            up = _mm_f16(h, u).astype(np.float32)
            gc = np.minimum(gate, np.float32(limit))
            a = gc / (np.float32(1.0) + np.exp(-gc)) * np.clip(up, -limit, limit).astype(np.float32)
            down = _mm_f16(f2h(a), dn).astype(np.float32)
            np.add.at(out_l, rows, down * sub_w[rows, kpos][:, None])
    return out_g, out_l


# ------------------------------------------------------------------------------------ router
def router_topk(x16: np.ndarray, w16: np.ndarray, bias: np.ndarray | None, topk: int, norm: bool = True,
                scale: float = 1.0):
    """GLM-5.3-Flash noaux_tc router (docs/research/02-glm-5.3-flash-architecture.md:33; the DeepSeek-V3
    sigmoid router with n_group = topk_group = 1) restated -> (ids int64 [T, k], weights fp32 [T, k]).
    logits = x . w^T in fp32; s = sigmoid; the k experts with the largest s + bias, ordered by
    (s + bias descending, expert id ascending); weights = s / (sequential sum of the k scores + 1e-20)
    if norm, times scale."""
    logits = x16.astype(np.float32) @ w16.astype(np.float32).T
    s = (np.float32(1.0) / (np.float32(1.0) + np.exp(-logits))).astype(np.float32)
    sel = s + (bias.astype(np.float32)[None, :] if bias is not None else np.float32(0.0))
    T, E = s.shape
    eidx = np.broadcast_to(np.arange(E), (T, E))
    order = np.lexsort((eidx, -sel), axis=-1)[:, :topk]
    ids = order.astype(np.int64)
    w = np.take_along_axis(s, order, axis=1).astype(np.float32)
    if norm:
        acc = np.zeros(T, np.float32)
        for j in range(topk):
            acc = (acc + w[:, j]).astype(np.float32)
        w = (w / (acc + np.float32(1e-20))[:, None]).astype(np.float32)
    return ids, (w * np.float32(scale)).astype(np.float32), sel


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
