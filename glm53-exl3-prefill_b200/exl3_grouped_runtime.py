"""Serving integration of the B200 grouped EXL3 prefill MoE — drop-in for kernel/exl3_grouped_runtime.py.

Installed into vLLM's exl3 overlay module by the reference's unchanged hook (kernel/patch_exl3_grouped.py)
when EXL3_GROUPED_PREFILL=1: the hook puts dirname(EXL3_GROUPED_SRC) on sys.path and calls
``exl3_grouped_runtime.install(module)``, so pointing EXL3_GROUPED_SRC at any file in this directory
selects this implementation.  Prefill calls (tokens > the fused kernel's row cap) go through one launch
per stage over all experts on sm_100a; decode calls keep the original path untouched (unless
EXL3_GROUPED_SMALL_BATCH=1, below).

Env (same names as the reference, kernel/exl3_grouped_runtime.py:7-10):
  EXL3_GROUPED_PREFILL=1   enable (read by the hook)
  EXL3_GROUPED_SRC         any file in this directory (the hook adds its directory to sys.path)
  EXL3_GROUPED_BUILD       optional directory holding a prebuilt libexl3_b200.so (default: ./lib);
                           the library is built ahead of time by build_ext.py, never at import
and one of this implementation's own:
  EXL3_GROUPED_SMALL_BATCH=1  calls with tokens <= the fused kernel's row cap also take the grouped
                           pipeline instead of the original path: replayed from per-layer CUDA graphs
                           (exl3_decode.GraphedPrefill), or run eagerly when the caller is itself
                           capturing a CUDA graph (the caller's graph then holds the launches)
"""
import logging
import os
import sys
import time
import types

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

logger = logging.getLogger("vllm.exl3.grouped")
_ext = None
_logged = False


def _load_ext():
    """Load the prebuilt C-ABI library; returns the binding module (build_blocks, row_had, act_had,
    grouped_gemm, route_sort with the reference's signatures).  Raises if the library is missing."""
    global _ext
    if _ext is not None:
        return _ext
    import b200_ext
    t0 = time.time()
    b200_ext.load()
    _ext = b200_ext
    logger.info("EXL3 grouped prefill extension loaded in %.0fs from %s", time.time() - t0, b200_ext.lib_path())
    return _ext


def deterministic_default() -> bool:
    """EXL3_GROUPED_DETERMINISTIC: "1" sums each token's routes in a fixed order (bit-repeatable layer
    output), "0" (the default) with fp32 atomics in the down GEMM's epilogue, as the reference does."""
    return os.environ.get("EXL3_GROUPED_DETERMINISTIC", "0") not in ("", "0")


def grouped_prefill(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, layer, limit: float,
                    stage_hook=None, out: torch.Tensor | None = None,
                    deterministic: bool | None = None) -> torch.Tensor:
    """x2d [T, K] (any float dtype), ids [T, topk] long, weights [T, topk] -> out [T, K] fp32.

    Same contract as kernel/exl3_grouped_runtime.py:50-83.  The host sort block (:59-72) is one GPU sort
    here (route_sort); then row_had -> grouped_gemm(mode 0) -> act_had -> the down stage, either
      * as the reference (deterministic=False): grouped_gemm mode 1 adds each route's weighted row into
        out[token] with fp32 atomics (:274-275), the order of the adds left to the hardware; or
      * deterministic=True: the sort runs over the flattened routing so that each sorted row keeps its
        routing slot t*topk + j, the down GEMM stores each route's weighted row at its slot (mode 2) and
        combine_slots sums every token's rows in slot order: the same sum, a fixed order, the same bits
        call after call, for one more pass over the R weighted rows (0.2 ms at config 1).
    deterministic=None takes EXL3_GROUPED_DETERMINISTIC.  Everything runs on the current stream with no
    host synchronisation.  `stage_hook`, if given, is called with a stage name before each stage launch
    and with "end" after the last one (used to record CUDA events between kernels).  `out` (fp32 [T, K],
    contiguous), if given, is added into; otherwise a new tensor is returned."""
    hook = stage_hook if stage_hook is not None else (lambda name: None)
    if deterministic is None:
        deterministic = deterministic_default()
    gp = _load_ext()
    dev = x2d.device
    T, K = x2d.shape
    topk = ids.shape[1]
    R = T * topk
    E = int(layer.w13_trellis.shape[0])
    accumulate = out is not None
    if out is None:
        # the combine writes every row; the atomic scatter adds onto zeros
        out = (torch.empty if deterministic and R else torch.zeros)(T, K, dtype=torch.float32, device=dev)
    elif out.dtype != torch.float32 or tuple(out.shape) != (T, K) or not out.is_contiguous() or out.device != dev:
        raise RuntimeError("out must be a contiguous fp32 [T, K] tensor on the input's device")
    if R == 0:
        return out
    x16 = x2d.to(torch.float16).contiguous()
    ids_c = ids.contiguous()
    w_c = weights.contiguous()
    if w_c.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        w_c = w_c.to(torch.float16)       # the reference's own cast (kernel/exl3_grouped_runtime.py:63)
    b = sort_buffers(R, E, dev)
    hook("route_sort")
    if deterministic:
        # the flattened routing sorted by expert: the same stable order as the reference's argsort, with the
        # routing slot t*topk + j (not the token t) kept per sorted row
        gp.route_sort(ids_c.view(-1, 1), w_c.view(-1, 1), E, b.token_sorted, b.weight_sorted, b.expert_of_row,
                      b.counts, b.expert_row0, b.block_expert, b.block_row0, b.meta)
    else:
        gp.route_sort(ids_c, w_c, E, b.token_sorted, b.weight_sorted, b.expert_of_row, b.counts, b.expert_row0,
                      b.block_expert, b.block_row0, b.meta)
    return run_stages(x16, b, layer, limit, out, hook, ids_c, accumulate, slots=deterministic)


def sort_buffers(R: int, E: int, dev):
    """Outputs of the expert sort for R routed rows over E experts (the reference's own buffers,
    kernel/exl3_grouped_runtime.py:69-80)."""
    b = types.SimpleNamespace()
    max_blocks = R // 128 + E
    b.token_sorted = torch.empty(R, dtype=torch.int64, device=dev)
    b.weight_sorted = torch.empty(R, dtype=torch.float16, device=dev)
    b.expert_of_row = torch.empty(R, dtype=torch.int32, device=dev)
    b.counts = torch.empty(E, dtype=torch.int32, device=dev)
    b.expert_row0 = torch.empty(E, dtype=torch.int32, device=dev)
    b.block_expert = torch.empty(max_blocks, dtype=torch.int32, device=dev)
    b.block_row0 = torch.empty_like(b.block_expert)
    b.meta = torch.zeros(2, dtype=torch.int32, device=dev)
    return b


def run_stages(x16: torch.Tensor, b, layer, limit: float, out: torch.Tensor, hook, ids: torch.Tensor,
               accumulate: bool, slots: bool) -> torch.Tensor:
    """Stages 2-5 over the sorted routing `b` (from route_sort, or the router front-end).

    slots=True: b.token_sorted holds each sorted row's routing slot s = t*topk + j: row_had (token
    s // topk) -> grouped_gemm(mode 0) -> act_had -> grouped_gemm(mode 2: w * y stored at row s) ->
    combine_slots into the fp32 `out` (added to it if `accumulate`).
    slots=False: b.token_sorted holds tokens: row_had -> grouped_gemm(mode 0) -> act_had ->
    grouped_gemm(mode 1: w * y added into out[token] with fp32 atomics; `out` holds zeros or the values
    to add onto)."""
    gp = _load_ext()
    R, K = b.token_sorted.numel(), x16.shape[1]
    T, topk = int(ids.shape[0]), int(ids.shape[1])
    I = int(layer._exl3_intermediate_local)
    E = int(layer.w13_trellis.shape[0])
    dev = x16.device
    h13 = torch.empty(R, K, dtype=torch.float16, device=dev)
    gu = torch.empty(R, 2 * I, dtype=torch.float16, device=dev)
    act = torch.empty(R, I, dtype=torch.float16, device=dev)
    hook("row_had")
    if slots:
        gp.ep_row_had([x16.data_ptr()], T, topk, h13, b.token_sorted, b.expert_of_row, 0, layer.w13_suh[:, 0])
    else:
        gp.row_had(x16, h13, b.token_sorted, b.expert_of_row, layer.w13_suh[:, 0], True)
    hook("gemm_gate_up")
    gp.grouped_gemm(h13, layer.w13_trellis[:, 0], layer.w13_trellis[:, 1], layer.w13_svh[:, 0], layer.w13_svh[:, 1],
                    b.block_expert, b.block_row0, b.counts, b.expert_row0, b.token_sorted, b.weight_sorted, gu, 0)
    hook("act_had")
    gp.act_had(gu, act, b.expert_of_row, layer.w2_suh, float(limit))
    hook("gemm_down")
    if slots:
        y = torch.empty(R, K, dtype=torch.float32, device=dev)
        gp.grouped_gemm(act, layer.w2_trellis, None, layer.w2_svh, None,
                        b.block_expert, b.block_row0, b.counts, b.expert_row0, b.token_sorted, b.weight_sorted, y, 2)
        hook("combine")
        gp.combine_slots(y, ids, E, out, accumulate)
    else:
        gp.grouped_gemm(act, layer.w2_trellis, None, layer.w2_svh, None,
                        b.block_expert, b.block_row0, b.counts, b.expert_row0, b.token_sorted, b.weight_sorted, out, 1)
    hook("end")
    return out


def small_batch_enabled() -> bool:
    """EXL3_GROUPED_SMALL_BATCH set to anything but "" / "0"."""
    return os.environ.get("EXL3_GROUPED_SMALL_BATCH", "0") not in ("", "0")


def small_batch_prefill(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, layer, limit: float,
                        max_tokens: int) -> torch.Tensor:
    """A decode-sized call (tokens <= max_tokens) through the grouped pipeline -> fp32 [T, K] (a fresh tensor).

    Outside a stream capture it replays the layer's exl3_decode.GraphedPrefill (created on first use and
    kept on the layer as ``_exl3_b200_graphed``); while the caller captures a CUDA graph of its own (an
    engine's decode graphs) it runs grouped_prefill eagerly, so the caller's graph records the launches."""
    if torch.cuda.is_current_stream_capturing():
        return grouped_prefill(x2d, ids, weights, layer, limit)
    import exl3_decode
    topk = int(ids.shape[1])
    gp = getattr(layer, "_exl3_b200_graphed", None)
    if gp is None or gp.topk != topk or gp.limit != float(limit) or gp.max_tokens < max_tokens:
        gp = exl3_decode.GraphedPrefill(layer, limit, topk, max_tokens=exl3_decode.GraphedPrefill.bucket(max_tokens),
                                        device=x2d.device)
        layer._exl3_b200_graphed = gp
    return gp(x2d, ids, weights).clone()


def install(ov):
    """Wrap ov.apply_exl3_experts: prefill-sized calls use the grouped path; everything else is untouched
    (kernel/exl3_grouped_runtime.py:86-112), unless EXL3_GROUPED_SMALL_BATCH=1 also sends the calls at or
    below the row cap through the grouped pipeline (small_batch_prefill)."""
    global _logged
    original = ov.apply_exl3_experts
    small_batch = small_batch_enabled()

    def apply_exl3_experts_grouped(x, topk_ids, topk_weights, layer, *, limit=ov.SWIGLU_LIMIT_DEFAULT, fused=None):
        global _logged
        tokens = x.shape[-2]
        temps = getattr(layer, "_exl3_fused_temps", None)
        cap = int(temps[0].shape[1]) if temps else 0
        expert_map = getattr(layer, "expert_map", None)
        small = tokens <= cap
        if (small and not (small_batch and tokens > 0 and x.is_cuda)) or expert_map is not None or \
                not hasattr(layer, "w13_trellis"):
            return original(x, topk_ids, topk_weights, layer, limit=limit, fused=fused)
        x2d = x.reshape(tokens, x.shape[-1])
        ids = topk_ids.reshape(tokens, -1).to(torch.long)
        weights = topk_weights.reshape(tokens, -1)
        if small:
            out = small_batch_prefill(x2d, ids, weights, layer, float(limit), cap)
            layer._exl3_last_apply = "grouped-small-batch"
            return out.to(dtype=x.dtype)
        out = grouped_prefill(x2d, ids, weights, layer, float(limit))
        layer._exl3_last_apply = "grouped"
        if not _logged:
            logger.info("EXL3 grouped prefill engaged (tokens=%d > cap=%d, experts=%d)", tokens, cap,
                        int(layer.w13_trellis.shape[0]))
            _logged = True
        return out.to(dtype=x.dtype)

    # The overlay's MoE method resolves apply_exl3_experts through the module namespace on every call, so
    # replacing the module attribute is enough; no caller holds a reference to the original.
    ov.apply_exl3_experts = apply_exl3_experts_grouped
    _load_ext()  # load at boot rather than on the first prefill
    logger.info("EXL3 grouped prefill installed (EXL3_GROUPED_PREFILL=1%s)",
                ", EXL3_GROUPED_SMALL_BATCH=1" if small_batch else "")
