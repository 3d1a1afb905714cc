"""Torch-facing binding of libexl3_b200.so (the sm_100a C-ABI library), loaded with ctypes.

The functions keep the names, argument order and error behaviour of the reference's pybind modules:

* ``build_blocks``, ``row_had``, ``act_had``, ``grouped_gemm``  — kernel/exl3_grouped_prefill.cu:380-386
* ``fat_gemm_v2``, ``fat_gemm_v2_scatter``, ``smem_bytes``       — kernel/exl3_fat_gemm_v2.cu:328-333
* ``exl3_fat_gemm``, ``exl3_fat_gemm_scatter`` (PR77 names)       — kernel/test_fat_v2.py:122,134

plus ``route_sort`` (the fused sort + block table that replaces kernel/exl3_grouped_runtime.py:59-72) and
the expert-parallel entry points ``ep_*`` (new: the reference has no expert parallelism).
Argument checks raise ``RuntimeError`` with the reference's TORCH_CHECK messages.  Every call runs on
the current torch stream of the tensors' device and never synchronises.  There is no fallback: if the
library is missing the import of this module's loader fails loudly.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libexl3_b200.so"

_lib = None
_lock = threading.Lock()
_status = {}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_F64 = ctypes.c_double

_SIGNATURES = {
    "exl3_last_error": ([], ctypes.c_char_p),
    "exl3_abi_version": ([], _I32),
    "exl3_set_wait_limit_ns": ([_I64], _I64),
    "exl3_build_blocks": ([_P, _I64, _P, _P, _I64, _P, _P], _I32),
    "exl3_route_sort": ([_P, _I32, _P, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64,
                         _P], _I32),
    "exl3_route_sort_scratch_elems": ([_I64, _I64], _I64),
    "exl3_router_topk": ([_P, _I64, _I64, _P, _I64, _P, _I64, _I64, _F64, _P, _P, _P, _P], _I32),
    "exl3_route_front_scratch_elems": ([_I64, _I64, _I64], _I64),
    "exl3_route_front_slots": ([_P, _I64, _I64, _P, _I64, _P, _I64, _I64, _F64, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                _I64, _P, _P, _I64, _P, _P], _I32),
    "exl3_combine_slots": ([_P, _P, _I32, _I64, _I64, _I64, _P, _I64, _I32, _P], _I32),
    "exl3_route_front": ([_P, _I64, _I64, _P, _I64, _P, _I64, _I64, _F64, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                          _I64, _P, _P, _I64, _P, _P], _I32),
    "exl3_row_had": ([_P, _I64, _P, _I64, _I64, _P, _P, _P, _I64, _I32, _P], _I32),
    "exl3_act_had": ([_P, _P, _I64, _I64, _P, _P, _I64, _F64, _P], _I32),
    "exl3_grouped_gemm": ([_P, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _I64, _P, _P, _I64, _P, _P,
                           _P, _P, _P, _I64, _I64, _I64, _P, _P], _I32),
    "exl3_fat_gemm_v2": ([_P, _I64, _I64, _P, _I64, _P, _P, _I64, _I32, _I32, _I64, _P, _P], _I32),
    "exl3_fat_gemm_v2_scatter": ([_P, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I64, _I32, _I32, _I64, _P, _P],
                                 _I32),
    "exl3_smem_bytes": ([_I64], _I64),
    "exl3_fat_gemm": ([_P, _I64, _I64, _P, _I64, _P, _P, _I64, _I32, _I32, _P, _P], _I32),
    "exl3_fat_gemm_scatter": ([_P, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I64, _I32, _I32, _P, _P], _I32),
    "exl3_ep_alloc": ([_I64, ctypes.POINTER(_P)], _I32),
    "exl3_ep_free": ([_P], _I32),
    "exl3_ep_ipc_handle": ([_P, _P], _I32),
    "exl3_ep_ipc_open": ([_P, ctypes.POINTER(_P)], _I32),
    "exl3_ep_ipc_close": ([_P], _I32),
    "exl3_ep_pull_rows": ([_P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P, _P], _I32),
    "exl3_ep_row_had": ([_P, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _P, _P], _I32),
    "exl3_ep_act_had": ([_P, _P, _I64, _I64, _P, _I64, _P, _I64, _F64, _P, _P], _I32),
    "exl3_ep_gemm_store": ([_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _P, _P, _P, _P, _P], _I32),
    "exl3_ep_combine_push": ([_P, _I64, _P, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _P], _I32),
    "exl3_ep_combine_reduce": ([_P, _I64, _P, _I64, _I64, _I64, _I64, _P, _I64, _P], _I32),
}


def lib_path() -> str:
    """EXL3_B200_LIB, else EXL3_GROUPED_BUILD/libexl3_b200.so if present, else the in-tree lib/."""
    p = os.environ.get("EXL3_B200_LIB")
    if p:
        return p
    build = os.environ.get("EXL3_GROUPED_BUILD")
    if build and os.path.exists(os.path.join(build, LIB_NAME)):
        return os.path.join(build, LIB_NAME)
    return os.path.join(HERE, "lib", LIB_NAME)


def load():
    """Load the C-ABI library (once).  Raises RuntimeError when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(f"EXL3 B200 extension not built: {path} is missing "
                                   f"(run python {os.path.join(HERE, 'build_ext.py')})")
            lib = ctypes.CDLL(path)
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def _check(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


def _call(fn, *args):
    rc = fn(*args)
    if rc != 0:
        raise RuntimeError(load().exl3_last_error().decode(errors="replace"))


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def status_tensor(dev: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels set to a non-zero code when they give up (bounded waits)."""
    key = (dev.type, dev.index if dev.index is not None else torch.cuda.current_device())
    t = _status.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _status[key] = t
    return t


def set_wait_limit_ns(ns: int) -> int:
    """Time limit of the tcgen05 kernels' bounded waits for later launches (ns < 0: the 2 s default).
    Returns the previous limit."""
    return int(load().exl3_set_wait_limit_ns(int(ns)))


def read_status(dev: torch.device, reset: bool = True) -> int:
    """Synchronising read of the device status word (0 = no kernel gave up)."""
    t = status_tensor(dev)
    v = int(t.item())
    if reset and v:
        t.zero_()
    return v


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tensors must be CUDA")


# ------------------------------------------------------------------------------------ stage 1
def build_blocks(counts, block_expert, block_row0, meta):
    """kernel/exl3_grouped_prefill.cu:285-294."""
    _check(all(t.dtype == torch.int32 for t in (counts, block_expert, block_row0, meta)), "int32 tensors")
    _check(counts.numel() <= 1024, "too many experts")
    _cuda(counts, block_expert, block_row0, meta)
    lib = load()
    with torch.cuda.device(counts.device):
        _call(lib.exl3_build_blocks, _ptr(counts), counts.numel(), _ptr(block_expert), _ptr(block_row0),
              block_expert.numel(), _ptr(meta), _stream(counts.device))


_WDTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def route_sort_scratch_elems(rows, n_experts):
    """int32 elements of scratch route_sort needs for `rows` routed rows."""
    return int(load().exl3_route_sort_scratch_elems(int(rows), int(n_experts)))


def route_sort(ids, weights, n_experts, token_sorted, weight_sorted, expert_of_row, counts, expert_row0,
               block_expert, block_row0, meta, invalid_count=None, scratch=None):
    """Stable expert sort + block table in one launch (replaces kernel/exl3_grouped_runtime.py:59-72).

    ids [T, topk] int64/int32, weights [T, topk] fp32/fp16/bf16 -> token_sorted int64 [R],
    weight_sorted fp16 [R], expert_of_row int32 [R], counts/expert_row0 int32 [E], block tables."""
    _check(ids.dtype in (torch.int64, torch.int32), "ids must be int64 or int32")
    _check(weights.dtype in _WDTYPE, "weights must be float32, float16 or bfloat16")
    _check(ids.is_contiguous() and weights.is_contiguous() and ids.numel() == weights.numel(),
           "ids / weights must be contiguous [T, topk]")
    _check(token_sorted.dtype == torch.int64 and weight_sorted.dtype == torch.float16 and
           expert_of_row.dtype == torch.int32, "routing dtypes")
    _check(all(t.dtype == torch.int32 for t in (counts, expert_row0, block_expert, block_row0, meta)), "int32 tensors")
    _check(1 <= n_experts <= 1024, "too many experts")
    _cuda(ids, weights, token_sorted, weight_sorted, expert_of_row, counts, expert_row0, block_expert, block_row0, meta)
    T = ids.shape[0] if ids.dim() == 2 else ids.numel()
    topk = ids.shape[1] if ids.dim() == 2 else 1
    lib = load()
    need = route_sort_scratch_elems(T * topk, n_experts)
    if scratch is None:
        scratch = torch.empty(need, dtype=torch.int32, device=ids.device)
    _check(scratch.dtype == torch.int32 and scratch.is_cuda and scratch.numel() >= need, "route_sort: scratch too small")
    with torch.cuda.device(ids.device):
        _call(lib.exl3_route_sort, _ptr(ids), 1 if ids.dtype == torch.int64 else 0, _ptr(weights),
              _WDTYPE[weights.dtype], T, topk, n_experts, block_expert.numel(), _ptr(token_sorted),
              _ptr(weight_sorted), _ptr(expert_of_row), _ptr(counts), _ptr(expert_row0), _ptr(block_expert),
              _ptr(block_row0), _ptr(meta), _ptr(invalid_count), _ptr(scratch), scratch.numel(), _stream(ids.device))


# ------------------------------------------------------------------------------------ routing front-end
def _check_router(x, w_router, bias, topk, ids, weights):
    _check(x.dtype == torch.float16 and x.is_contiguous() and x.dim() == 2, "router: x fp16 [T, d] contiguous")
    _check(w_router.dtype == torch.float16 and w_router.is_contiguous() and w_router.dim() == 2
           and w_router.size(1) == x.size(1), "router: weight fp16 [E, d] contiguous")
    _check(bias is None or (bias.dtype == torch.float32 and bias.is_contiguous() and bias.numel() == w_router.size(0)),
           "router: bias fp32 [E]")
    T = x.size(0)
    _check(ids.dtype == torch.int64 and ids.is_contiguous() and tuple(ids.shape) == (T, topk), "router: ids int64 [T, topk]")
    _check(weights.dtype == torch.float32 and weights.is_contiguous() and tuple(weights.shape) == (T, topk),
           "router: weights fp32 [T, topk]")
    _cuda(x, w_router, bias, ids, weights)


def router_topk(x, w_router, bias, topk, norm, scale, ids, weights):
    """GLM-5.3-Flash noaux_tc router on the GPU: ids int64 / weights fp32 [T, topk] from x fp16 [T, d]."""
    _check_router(x, w_router, bias, topk, ids, weights)
    lib = load()
    dev = x.device
    with torch.cuda.device(dev):
        _call(lib.exl3_router_topk, _ptr(x), x.size(0), x.size(1), _ptr(w_router), w_router.size(0), _ptr(bias),
              int(topk), 1 if norm else 0, float(scale), _ptr(ids), _ptr(weights), _ptr(status_tensor(dev)),
              _stream(dev))


def route_front_scratch_elems(T: int, topk: int, n_experts: int) -> int:
    n = int(load().exl3_route_front_scratch_elems(int(T), int(topk), int(n_experts)))
    _check(n >= 0, "route_front: invalid arguments")
    return n


def route_front(x, w_router, bias, topk, norm, scale, ids, weights, token_sorted, weight_sorted, expert_of_row,
                counts, expert_row0, block_expert, block_row0, meta, scratch=None, slots=False):
    """router_topk + the expert sort of route_sort over its output (two launches for topk 1, 2, 4, 8, 16).
    With slots, token_sorted receives each sorted row's routing slot t*topk + j instead of its token."""
    _check_router(x, w_router, bias, topk, ids, weights)
    E = w_router.size(0)
    _check(token_sorted.dtype == torch.int64 and weight_sorted.dtype == torch.float16 and
           expert_of_row.dtype == torch.int32, "routing dtypes")
    _check(all(t.dtype == torch.int32 for t in (counts, expert_row0, block_expert, block_row0, meta)), "int32 tensors")
    _check(counts.numel() == E and expert_row0.numel() == E, "counts / expert_row0 must have one entry per expert")
    _check(token_sorted.numel() >= x.size(0) * topk, "sorted arrays must hold T * topk rows")
    _cuda(token_sorted, weight_sorted, expert_of_row, counts, expert_row0, block_expert, block_row0, meta)
    need = route_front_scratch_elems(x.size(0), topk, E)
    if scratch is None:
        scratch = torch.empty(need, dtype=torch.int32, device=x.device)
    _check(scratch.dtype == torch.int32 and scratch.is_cuda and scratch.numel() >= need, "route_front: scratch too small")
    lib = load()
    dev = x.device
    with torch.cuda.device(dev):
        _call(lib.exl3_route_front_slots if slots else lib.exl3_route_front, _ptr(x), x.size(0), x.size(1),
              _ptr(w_router), E, _ptr(bias), int(topk),
              1 if norm else 0, float(scale), _ptr(ids), _ptr(weights), _ptr(token_sorted), _ptr(weight_sorted),
              _ptr(expert_of_row), _ptr(counts), _ptr(expert_row0), _ptr(block_expert), _ptr(block_row0),
              block_expert.numel(), _ptr(meta), _ptr(scratch), scratch.numel(), _ptr(status_tensor(dev)),
              _stream(dev))


# ------------------------------------------------------------------------------------ stages 2, 4
def row_had(src, dst, token_sorted, expert_of_row, suh, gather):
    """kernel/exl3_grouped_prefill.cu:297-311."""
    rows, K = int(dst.size(0)), int(dst.size(1))
    _check(K % 128 == 0 and suh.size(-1) == K, "K must be a multiple of 128 and match suh")
    _check(src.dtype == torch.float16 and dst.dtype == torch.float16 and suh.dtype == torch.float16,
           "row_had: fp16 tensors")
    _check(src.is_contiguous() and dst.is_contiguous() and suh.stride(-1) == 1 and src.size(1) == K,
           "row_had: contiguous rows")
    _check(expert_of_row.dtype == torch.int32 and (not gather or token_sorted.dtype == torch.int64), "routing dtypes")
    _cuda(src, dst, suh, expert_of_row, token_sorted if gather else None)
    lib = load()
    with torch.cuda.device(src.device):
        _call(lib.exl3_row_had, _ptr(src), src.size(0), _ptr(dst), rows, K, _ptr(token_sorted) if gather else None,
              _ptr(expert_of_row), _ptr(suh), suh.stride(0), 1 if gather else 0, _stream(src.device))


def act_had(gu, act, expert_of_row, suh_down, limit):
    """kernel/exl3_grouped_prefill.cu:313-322."""
    rows, I = int(act.size(0)), int(act.size(1))
    _check(gu.size(1) == 2 * I and I % 128 == 0, "gate|up width must be 2I, I multiple of 128")
    _check(gu.dtype == torch.float16 and act.dtype == torch.float16 and suh_down.dtype == torch.float16,
           "act_had: fp16 tensors")
    _check(gu.is_contiguous() and act.is_contiguous() and suh_down.stride(-1) == 1 and gu.size(0) >= rows,
           "act_had: contiguous rows")
    _check(expert_of_row.dtype == torch.int32, "routing dtypes")
    _cuda(gu, act, suh_down, expert_of_row)
    lib = load()
    with torch.cuda.device(gu.device):
        _call(lib.exl3_act_had, _ptr(gu), _ptr(act), rows, I, _ptr(expert_of_row), _ptr(suh_down),
              suh_down.stride(0), float(limit), _stream(gu.device))


# ------------------------------------------------------------------------------------ stages 3, 5
def grouped_gemm(a, packed_gate, packed_up, svh_gate, svh_up, block_expert, block_row0, counts, expert_row0,
                 token_sorted, route_weight, out, mode):
    """kernel/exl3_grouped_prefill.cu:326-378 (mode 0: gate|up fp16 rows; mode 1: down, fp32 scatter), plus
    mode 2 (down, fp32 row store of w[r] * y[r] at row token_sorted[r]: the slot-ordered down stage)."""
    _check(a.dtype == torch.float16 and a.is_contiguous(), "a fp16 contiguous")
    _check(packed_gate.dim() == 4 and packed_gate.size(3) == 64 and packed_gate.stride(3) == 1
           and packed_gate.stride(2) == 64 and packed_gate.stride(1) == packed_gate.size(2) * 64,
           "packed [E, tiles_k, tiles_n, 64] with contiguous inner dims (expert stride may be larger: [E,2,...] views)")
    _check(packed_gate.dtype == torch.int16, "packed must be int16")
    size_k, tiles_k, tiles_n = int(a.size(1)), int(packed_gate.size(1)), int(packed_gate.size(2))
    _check(size_k == tiles_k * 16 and size_k % 64 == 0, "K mismatch")
    size_n_each = tiles_n * 16
    _check(size_n_each % 128 == 0, "N must be a multiple of 128")
    n_tensors = 2 if packed_up is not None else 1
    expert_stride = packed_gate.stride(0)
    svh_stride = svh_gate.stride(0)
    _check(svh_gate.size(-1) == size_n_each and svh_gate.stride(-1) == 1, "svh N mismatch")
    _check(svh_gate.dtype == torch.float16, "svh must be float16")
    if packed_up is not None:
        _check(packed_up.stride(0) == expert_stride and svh_up is not None and svh_up.stride(0) == svh_stride
               and tuple(packed_up.shape) == tuple(packed_gate.shape) and packed_up.stride() == packed_gate.stride(),
               "gate/up strides must match")
    _check(counts.dtype == torch.int32 and expert_row0.dtype == torch.int32, "int32 tensors")
    E = int(packed_gate.size(0))
    _check(counts.numel() == E and expert_row0.numel() == E, "counts / expert_row0 must have one entry per expert")
    if mode == 0:
        _check(out.dtype == torch.float16 and out.size(1) == n_tensors * size_n_each and out.is_contiguous(),
               "mode 0: out fp16 [rows, n_tensors*N]")
    else:
        _check(mode in (1, 2), "mode must be 0 (gate|up), 1 (down scatter) or 2 (down row store)")
        _check(out.dtype == torch.float32 and out.size(1) == size_n_each and n_tensors == 1 and out.is_contiguous(),
               f"mode {mode}: out fp32 [T, N], single tensor")
        _check(token_sorted.dtype == torch.int64 and route_weight.dtype == torch.float16, "routing dtypes")
    _cuda(a, packed_gate, packed_up, svh_gate, svh_up, counts, expert_row0, out)
    lib = load()
    dev = a.device
    with torch.cuda.device(dev):
        _call(lib.exl3_grouped_gemm, _ptr(a), a.size(0), size_k, _ptr(packed_gate), _ptr(packed_up), E, tiles_k,
              tiles_n, expert_stride, _ptr(svh_gate), _ptr(svh_up), svh_stride, _ptr(block_expert),
              _ptr(block_row0), 0 if block_expert is None else block_expert.numel(), _ptr(counts),
              _ptr(expert_row0), _ptr(token_sorted) if mode != 0 else None,
              _ptr(route_weight) if mode != 0 else None, _ptr(out), out.size(0), out.size(1), int(mode),
              _ptr(status_tensor(dev)), _stream(dev))


def combine_slots(y, ids, n_experts, out, accumulate=False):
    """out[t] = (accumulate ? out[t] : 0) + sum over j ascending (ids[t, j] in [0, E)) of y[t*topk + j]
    (fp32, deterministic): the per-token combine of the slot-ordered down stage (grouped_gemm mode 2)."""
    _check(ids.dim() == 2 and ids.dtype in (torch.int64, torch.int32) and ids.is_contiguous(),
           "ids must be contiguous int64 or int32 [T, topk]")
    T, topk = int(ids.size(0)), int(ids.size(1))
    _check(y.dtype == torch.float32 and y.is_contiguous() and y.dim() == 2 and y.size(0) >= T * topk,
           "combine_slots: y fp32 [T*topk, K]")
    _check(out.dtype == torch.float32 and out.is_contiguous() and tuple(out.shape) == (T, y.size(1)),
           "combine_slots: out fp32 [T, K]")
    _cuda(y, ids, out)
    lib = load()
    with torch.cuda.device(out.device):
        _call(lib.exl3_combine_slots, _ptr(y), _ptr(ids), 1 if ids.dtype == torch.int64 else 0, T, topk,
              int(n_experts), _ptr(out), out.size(1), 1 if accumulate else 0, _stream(out.device))


# ------------------------------------------------------------------------------------ expert parallelism
# No reference counterpart (the reference refuses expert-parallel layers, kernel/exl3_grouped_runtime.py:96-98).
IPC_HANDLE_BYTES = 64
MAX_RANKS = 8


def ep_alloc(nbytes: int, device: torch.device) -> int:
    """cudaMalloc of a buffer whose IPC handle other ranks can map; returns the device address."""
    lib = load()
    out = _P()
    with torch.cuda.device(device):
        _call(lib.exl3_ep_alloc, int(nbytes), ctypes.byref(out))
    return int(out.value)


def ep_free(addr: int, device: torch.device):
    lib = load()
    with torch.cuda.device(device):
        _call(lib.exl3_ep_free, _P(addr))


def ep_ipc_handle(addr: int, device: torch.device) -> bytes:
    lib = load()
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        _call(lib.exl3_ep_ipc_handle, _P(addr), ctypes.cast(buf, _P))
    return buf.raw


def ep_ipc_open(handle: bytes, device: torch.device) -> int:
    _check(len(handle) == IPC_HANDLE_BYTES, "ep_ipc_open: 64-byte handle")
    lib = load()
    buf = ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
    out = _P()
    with torch.cuda.device(device):
        _call(lib.exl3_ep_ipc_open, ctypes.cast(buf, _P), ctypes.byref(out))
    return int(out.value)


def ep_ipc_close(addr: int, device: torch.device):
    lib = load()
    with torch.cuda.device(device):
        _call(lib.exl3_ep_ipc_close, _P(addr))


def _ptr_array(addrs):
    _check(1 <= len(addrs) <= MAX_RANKS, f"ep: 1..{MAX_RANKS} ranks")
    return (_P * len(addrs))(*[_P(int(a)) for a in addrs])


def ep_pull_rows(x_ranks, rank, tokens_per_rank, ids_pos, e0, e1, x_pulled):
    """Dispatch: copy every other rank's token row with a route to expert positions [e0, e1) into its
    global row of x_pulled (fp16 [n_ranks * tokens_per_rank, K]); each such row crosses NVLink once."""
    _check(ids_pos.dtype == torch.int64 and ids_pos.is_contiguous() and ids_pos.dim() == 2, "ids_pos int64 [T, topk]")
    _check(x_pulled.dtype == torch.float16 and x_pulled.is_contiguous()
           and x_pulled.size(0) == len(x_ranks) * tokens_per_rank and ids_pos.size(0) == x_pulled.size(0),
           "x_pulled fp16 [n_ranks * tokens_per_rank, K]")
    _cuda(ids_pos, x_pulled)
    lib = load()
    with torch.cuda.device(x_pulled.device):
        _call(lib.exl3_ep_pull_rows, _ptr_array(x_ranks), len(x_ranks), int(rank), int(tokens_per_rank),
              x_pulled.size(1), _ptr(ids_pos), ids_pos.size(1), int(e0), int(e1), _ptr(x_pulled),
              _stream(x_pulled.device))


def ep_row_had(x_ranks, tokens_per_rank, topk, dst, slot_sorted, expert_of_row, expert_base, suh, slot_row=None,
               rows_dev=None):
    """Stage 2 over routing slots: the row of slot s is token t = s // topk, read from x_ranks[t // tpr]
    (device addresses of n_ranks fp16 [tokens_per_rank, K] buffers); slot_row[s] = r if given.  With
    rows_dev (a device int32 count, e.g. the sort's meta[1:]) only min(dst rows, count) rows are done."""
    rows, K = int(dst.size(0)), int(dst.size(1))
    _check(K % 128 == 0 and suh.size(-1) == K, "K must be a multiple of 128 and match suh")
    _check(dst.dtype == torch.float16 and suh.dtype == torch.float16 and dst.is_contiguous() and suh.stride(-1) == 1,
           "row_had: fp16 tensors")
    _check(slot_sorted.dtype == torch.int64 and expert_of_row.dtype == torch.int32, "routing dtypes")
    _check(slot_row is None or (slot_row.dtype == torch.int32 and slot_row.is_contiguous()
                                and slot_row.numel() >= len(x_ranks) * tokens_per_rank * topk),
           "slot_row int32 [n_ranks * tokens_per_rank * topk]")
    _cuda(dst, suh, slot_sorted, expert_of_row, *([slot_row] if slot_row is not None else []))
    lib = load()
    with torch.cuda.device(dst.device):
        _call(lib.exl3_ep_row_had, _ptr_array(x_ranks), len(x_ranks), int(tokens_per_rank), int(topk), _ptr(dst),
              rows, K, _ptr(slot_sorted), _ptr(expert_of_row), int(expert_base), _ptr(suh), suh.stride(0),
              _ptr(slot_row) if slot_row is not None else None, _ptr(rows_dev), _stream(dst.device))


def ep_act_had(gu, act, expert_of_row, expert_base, suh_down, limit, rows_dev=None):
    """act_had with suh_down row expert_of_row[r] - expert_base; with rows_dev (a device int32 count) only
    min(act rows, count) rows are done."""
    rows, I = int(act.size(0)), int(act.size(1))
    _check(gu.size(1) == 2 * I and I % 128 == 0, "gate|up width must be 2I, I multiple of 128")
    _check(gu.dtype == torch.float16 and act.dtype == torch.float16 and suh_down.dtype == torch.float16,
           "act_had: fp16 tensors")
    _check(gu.is_contiguous() and act.is_contiguous() and suh_down.stride(-1) == 1 and gu.size(0) >= rows,
           "act_had: contiguous rows")
    _check(expert_of_row.dtype == torch.int32, "routing dtypes")
    _cuda(gu, act, suh_down, expert_of_row)
    lib = load()
    with torch.cuda.device(gu.device):
        _call(lib.exl3_ep_act_had, _ptr(gu), _ptr(act), rows, I, _ptr(expert_of_row), int(expert_base),
              _ptr(suh_down), suh_down.stride(0), float(limit), _ptr(rows_dev), _stream(gu.device))


def ep_gemm_store(a, packed, svh, counts, expert_row0, route_weight, y_local):
    """Stage 5 over this rank's experts: y_local[r] = w[r] * y[r] (fp32 [rows, N], weighted rows)."""
    _check(a.dtype == torch.float16 and a.is_contiguous(), "a fp16 contiguous")
    _check(packed.dim() == 4 and packed.size(3) == 64 and packed.stride(3) == 1 and packed.stride(2) == 64
           and packed.stride(1) == packed.size(2) * 64 and packed.dtype == torch.int16,
           "packed [E, tiles_k, tiles_n, 64] with contiguous inner dims")
    size_k, tiles_k, tiles_n = int(a.size(1)), int(packed.size(1)), int(packed.size(2))
    _check(size_k == tiles_k * 16 and size_k % 64 == 0, "K mismatch")
    _check(svh.size(-1) == tiles_n * 16 and svh.stride(-1) == 1 and svh.dtype == torch.float16, "svh N mismatch")
    E = int(packed.size(0))
    _check(counts.dtype == torch.int32 and expert_row0.dtype == torch.int32 and counts.numel() == E
           and expert_row0.numel() == E, "counts / expert_row0 must have one entry per expert")
    _check(route_weight.dtype == torch.float16 and route_weight.numel() >= a.size(0), "routing dtypes")
    _check(y_local.dtype == torch.float32 and y_local.is_contiguous() and y_local.size(0) >= a.size(0)
           and y_local.size(1) == tiles_n * 16, "y_local fp32 [rows, N]")
    _cuda(a, packed, svh, counts, expert_row0, route_weight, y_local)
    lib = load()
    dev = a.device
    with torch.cuda.device(dev):
        _call(lib.exl3_ep_gemm_store, _ptr(a), a.size(0), size_k, _ptr(packed), E, tiles_k, tiles_n,
              packed.stride(0), _ptr(svh), svh.stride(0), _ptr(counts), _ptr(expert_row0), _ptr(route_weight),
              _ptr(y_local), _ptr(status_tensor(dev)), _stream(dev))


def ep_combine_push(y_local, ids_pos, e0, e1, slot_row, staging_ranks, rank, tokens_per_rank, staging_f16):
    """Combine, expert side: one summed row per (token, this rank) into the token owner's staging buffer
    (row (t % tpr) * n_ranks + rank; fp16 if staging_f16 else fp32)."""
    _check(y_local.dtype == torch.float32 and y_local.is_contiguous() and y_local.size(1) % 128 == 0,
           "y_local fp32 [rows, K]")
    _check(ids_pos.dtype == torch.int64 and ids_pos.is_contiguous() and ids_pos.dim() == 2
           and ids_pos.size(0) == len(staging_ranks) * tokens_per_rank, "ids_pos int64 [n_ranks * tpr, topk]")
    _check(slot_row.dtype == torch.int32 and slot_row.numel() >= ids_pos.numel(), "slot_row int32")
    _cuda(y_local, ids_pos, slot_row)
    lib = load()
    with torch.cuda.device(y_local.device):
        _call(lib.exl3_ep_combine_push, _ptr(y_local), y_local.size(1), _ptr(ids_pos), ids_pos.size(1), int(e0),
              int(e1), _ptr(slot_row), _ptr_array(staging_ranks), len(staging_ranks), int(rank), int(tokens_per_rank),
              1 if staging_f16 else 0, _stream(y_local.device))


def ep_combine_reduce(staging, ids_pos, n_experts, n_ranks, out):
    """out[t] = sum over the ranks r (ascending) owning any of t's routed experts of staging[t * n_ranks + r]."""
    T, topk = int(ids_pos.size(0)), int(ids_pos.size(1))
    _check(ids_pos.dtype == torch.int64 and ids_pos.is_contiguous(), "ids_pos int64 [T, topk]")
    _check(staging.dtype in (torch.float16, torch.float32) and staging.is_contiguous()
           and staging.size(0) >= T * n_ranks and staging.size(1) == out.size(1), "staging [T * n_ranks, K]")
    _check(out.dtype == torch.float32 and out.is_contiguous() and out.size(0) >= T, "out fp32 [T, K]")
    _cuda(staging, ids_pos, out)
    lib = load()
    with torch.cuda.device(out.device):
        _call(lib.exl3_ep_combine_reduce, _ptr(staging), 1 if staging.dtype == torch.float16 else 0, _ptr(ids_pos),
              T, topk, int(n_experts), int(n_ranks), _ptr(out), out.size(1), _stream(out.device))


# ------------------------------------------------------------------------------------ PR77 drop-in
def _check_fat(a, packed, out, svh, K, mcg, mul1):
    """kernel/exl3_fat_gemm_v2.cu:236-252."""
    _check(a.is_cuda and packed.is_cuda and out.is_cuda and svh.is_cuda, "tensors must be CUDA")
    _check(a.is_contiguous() and packed.is_contiguous() and out.is_contiguous() and svh.is_contiguous(),
           "tensors must be contiguous")
    _check(a.dtype == torch.float16, "a must be float16")
    _check(packed.dtype == torch.int16, "packed must be int16")
    _check(out.dtype == torch.float32, "out must be float32")
    _check(svh.dtype == torch.float16, "svh must be float16")
    _check(a.dim() == 2 and packed.dim() == 3 and out.dim() == 2 and svh.dim() == 1, "rank mismatch")
    _check(K == 4 and mcg and not mul1, "only K4 MCG tensors")
    _check(a.size(1) == packed.size(0) * 16, "a K dimension does not match packed tensor")
    _check(svh.numel() == packed.size(1) * 16, "svh N dimension does not match packed tensor")
    _check(svh.numel() % 128 == 0, "N must be divisible by 128")
    _check(packed.size(2) == 64, "packed K4 block width must be 64 int16 words")
    _check(a.size(1) % 64 == 0, "K must be divisible by 64")


def fat_gemm_v2(a, packed, out, svh, K, mcg, mul1, variant):
    """kernel/exl3_fat_gemm_v2.cu:298-303."""
    _check_fat(a, packed, out, svh, K, mcg, mul1)
    _check(out.size(0) == a.size(0) and out.size(1) == svh.numel(), "out shape must be [M, N]")
    _check(0 <= int(variant) <= 3, "unknown variant")
    lib = load()
    with torch.cuda.device(a.device):
        _call(lib.exl3_fat_gemm_v2, _ptr(a), a.size(0), a.size(1), _ptr(packed), svh.numel(), _ptr(out), _ptr(svh),
              int(K), int(bool(mcg)), int(bool(mul1)), int(variant), _ptr(status_tensor(a.device)), _stream(a.device))


def fat_gemm_v2_scatter(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1, variant):
    """kernel/exl3_fat_gemm_v2.cu:305-314."""
    _check_fat(a, packed, out, svh, K, mcg, mul1)
    _check(out.size(1) == svh.numel(), "out N dimension mismatch")
    _check(token_idx.is_cuda and route_weight.is_cuda and token_idx.is_contiguous() and route_weight.is_contiguous(),
           "routing tensors")
    _check(token_idx.dtype == torch.int64 and route_weight.dtype == torch.float16, "routing dtypes")
    _check(token_idx.numel() == a.size(0) and route_weight.numel() == a.size(0), "routing tensors must have M elements")
    _check(0 <= int(variant) <= 3, "unknown variant")
    lib = load()
    with torch.cuda.device(a.device):
        _call(lib.exl3_fat_gemm_v2_scatter, _ptr(a), a.size(0), a.size(1), _ptr(packed), svh.numel(), _ptr(out),
              out.size(0), _ptr(svh), _ptr(token_idx), _ptr(route_weight), int(K), int(bool(mcg)), int(bool(mul1)),
              int(variant), _ptr(status_tensor(a.device)), _stream(a.device))


def smem_bytes(variant):
    """kernel/exl3_fat_gemm_v2.cu:316-326: dynamic shared memory per variant (-1: unknown variant)."""
    return int(load().exl3_smem_bytes(int(variant)))


def exl3_fat_gemm(a, packed, out, svh, K, mcg, mul1):
    """PR77 name (kernel/test_fat_v2.py:122)."""
    fat_gemm_v2(a, packed, out, svh, K, mcg, mul1, 0)


def exl3_fat_gemm_scatter(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1):
    """PR77 name (kernel/test_fat_v2.py:134)."""
    fat_gemm_v2_scatter(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1, 0)
