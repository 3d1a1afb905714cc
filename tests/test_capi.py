"""CPU: the C-ABI library builds, loads without a GPU, exports every symbol include/exl3_b200.h declares,
and rejects bad arguments with the reference's messages before any launch."""
import ctypes
import os
import re

import pytest
import torch

import b200_ext
import build_ext
from conftest import REPO

HEADER = os.path.join(REPO, "include", "exl3_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(exl3_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build_ext.build()
    return b200_ext.load()


def test_header_declares_the_reference_entry_points():
    names = _declared()
    for n in ("exl3_build_blocks", "exl3_row_had", "exl3_act_had", "exl3_grouped_gemm", "exl3_fat_gemm_v2",
              "exl3_fat_gemm_v2_scatter", "exl3_smem_bytes", "exl3_fat_gemm", "exl3_fat_gemm_scatter",
              "exl3_route_sort", "exl3_route_sort_noalloc", "exl3_set_wait_limit_ns", "exl3_combine_slots",
              "exl3_route_front_slots", "exl3_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(b200_ext.lib_path())
    missing = [n for n in _declared() if not hasattr(raw, n)]
    assert not missing, missing


def test_abi_version_and_smem(lib):
    assert lib.exl3_abi_version() == 2
    for v in range(4):
        assert 0 < lib.exl3_smem_bytes(v) <= 232448
    assert lib.exl3_smem_bytes(4) == -1
    assert b200_ext.smem_bytes(-1) == -1


def test_validation_errors_without_gpu(lib):
    rc = lib.exl3_build_blocks(None, 2000, None, None, 0, None, None)
    assert rc != 0 and b"too many experts" in lib.exl3_last_error()
    rc = lib.exl3_row_had(None, 0, None, 4, 100, None, None, None, 0, 1, None)
    assert rc != 0 and b"K must be a multiple of 128" in lib.exl3_last_error()
    rc = lib.exl3_fat_gemm_v2(None, 4, 128, None, 128, None, None, 3, 1, 0, 0, None, None)
    assert rc != 0
    rc = lib.exl3_grouped_gemm(None, 4, 100, None, None, 8, 6, 8, 0, None, None, 128, None, None, 0, None, None,
                               None, None, None, 0, 128, 0, None, None)
    assert rc != 0 and b"K mismatch" in lib.exl3_last_error()


def test_expert_parallel_entry_points_validate_without_gpu(lib):
    P = ctypes.c_void_p
    zero = (P * 1)(P(16))
    rc = lib.exl3_ep_row_had(zero, 0, 64, 8, None, 10, 4096, None, None, 0, None, 4096, None, None, None)
    assert rc != 0 and b"1..8 ranks" in lib.exl3_last_error()
    nine = (P * 9)(*[P(16)] * 9)
    rc = lib.exl3_ep_row_had(nine, 9, 64, 8, None, 10, 4096, None, None, 0, None, 4096, None, None, None)
    assert rc != 0 and b"1..8 ranks" in lib.exl3_last_error()
    rc = lib.exl3_ep_row_had(zero, 1, 0, 8, None, 10, 4096, None, None, 0, None, 4096, None, None, None)
    assert rc != 0 and b"rows per rank" in lib.exl3_last_error()
    rc = lib.exl3_ep_row_had(zero, 1, 64, 64, None, 10, 4096, None, None, 0, None, 4096, None, None, None)
    assert rc != 0 and b"topk must be 1..32" in lib.exl3_last_error()
    unaligned = (P * 1)(P(18))
    rc = lib.exl3_ep_row_had(unaligned, 1, 64, 8, None, 10, 4096, None, None, 0, None, 4096, None, None, None)
    assert rc != 0 and b"16-byte aligned" in lib.exl3_last_error()
    two = (P * 2)(P(16), P(32))
    rc = lib.exl3_ep_pull_rows(two, 2, 2, 64, 4096, None, 8, 0, 4, None, None)
    assert rc != 0 and b"rank outside" in lib.exl3_last_error()
    rc = lib.exl3_ep_pull_rows(two, 2, 0, 64, 4096, None, 8, 4, 4, None, None)
    assert rc != 0 and b"invalid expert range" in lib.exl3_last_error()
    rc = lib.exl3_ep_pull_rows(two, 2, 0, 64, 4000, None, 8, 0, 4, None, None)
    assert rc != 0 and b"multiple of 128" in lib.exl3_last_error()
    assert lib.exl3_ep_pull_rows(zero, 1, 0, 64, 4096, None, 8, 0, 4, None, None) == 0   # one rank: no-op
    rc = lib.exl3_ep_gemm_store(None, 10, 100, None, 4, 6, 8, 0, None, 128, None, None, None, None, None, None)
    assert rc != 0 and b"K mismatch" in lib.exl3_last_error()
    rc = lib.exl3_ep_combine_push(None, 4096, None, 8, 0, 4, None, two, 2, 0, 64, 2, None)
    assert rc != 0 and b"staging_f16" in lib.exl3_last_error()
    rc = lib.exl3_ep_combine_push(None, 4096, None, 8, 0, 4, None, two, 2, 0, 64, 1, None)
    assert rc != 0 and b"must be CUDA" in lib.exl3_last_error()
    rc = lib.exl3_ep_combine_reduce(None, 1, None, 10, 0, 8, 2, None, 4096, None)
    assert rc != 0 and b"topk must be 1..32" in lib.exl3_last_error()
    rc = lib.exl3_ep_combine_reduce(None, 1, None, 10, 8, 8, 2, None, 4094, None)
    assert rc != 0 and b"multiple of 128" in lib.exl3_last_error()
    rc = lib.exl3_ep_combine_reduce(None, 1, None, 10, 8, 8, 9, None, 4096, None)
    assert rc != 0 and b"1..8 ranks" in lib.exl3_last_error()
    assert lib.exl3_ep_combine_reduce(None, 1, None, 0, 8, 8, 2, None, 4096, None) == 0     # nothing to do
    rc = lib.exl3_ep_alloc(0, ctypes.byref(P()))
    assert rc != 0 and b"invalid arguments" in lib.exl3_last_error()


def test_noalloc_route_sort_refusals_without_gpu(lib):
    """exl3_route_sort_noalloc checks its arguments, and the size of its built-in array, before it touches
    a device: every refusal below returns a code and a message on a host without a GPU."""
    P, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    fn = lib.exl3_route_sort_noalloc
    fn.argtypes = [P, I32, P, I32, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P]
    fn.restype = I32
    fake = P(256)                                         # never dereferenced: every case fails before a launch

    def call(ids=fake, wdt=0, T=64, topk=8, E=288, max_blocks=None, null=None):
        mb = (T * topk) // 128 + E if max_blocks is None else max_blocks
        ptrs = [fake] * 9
        if null is not None:
            ptrs[null] = None
        return fn(ids, 1, fake, wdt, T, topk, E, mb, *ptrs, None)

    for E in (0, -3, 1025):
        assert call(E=E) != 0 and b"too many experts" in lib.exl3_last_error()
    for T, topk in ((64, 0), (-1, 8), (1 << 30, 8)):
        assert call(T=T, topk=topk) != 0 and b"invalid routing shape" in lib.exl3_last_error()
    for wdt in (-1, 3):
        assert call(wdt=wdt) != 0 and b"unknown weight dtype" in lib.exl3_last_error()
    for mb in (-1, 1 << 31):
        assert call(max_blocks=mb) != 0 and b"invalid max_blocks" in lib.exl3_last_error()
    for i in (0, 1, 2, 3, 4, 5, 7):                      # token_sorted .. block_row0, meta
        assert call(null=i) != 0 and b"routing tensors must be CUDA" in lib.exl3_last_error(), i
    assert call(ids=None) != 0 and b"routing tensors must be CUDA" in lib.exl3_last_error()
    # 1024 experts x 70 chunks of 2048 routed rows: more scratch than the 65536-entry array holds
    assert b200_ext.route_sort_scratch_elems(140000, 1024) > 65536
    assert call(T=17500, topk=8, E=1024) != 0
    assert b"built-in array holds 65536" in lib.exl3_last_error()


def test_slot_down_stage_entry_points_validate_without_gpu(lib):
    P = ctypes.c_void_p
    fn = lib.exl3_combine_slots
    fn.argtypes = [P, P, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int64,
                   ctypes.c_int, P]
    fn.restype = ctypes.c_int
    fake = P(256)
    assert fn(fake, fake, 1, 10, 0, 288, fake, 4096, 0, None) != 0 and b"topk must be 1..32" in lib.exl3_last_error()
    assert fn(fake, fake, 1, 10, 33, 288, fake, 4096, 0, None) != 0
    assert fn(fake, fake, 1, 10, 8, 0, fake, 4096, 0, None) != 0 and b"too many experts" in lib.exl3_last_error()
    assert fn(fake, fake, 1, 10, 8, 288, fake, 4000, 0, None) != 0 and b"multiple of 128" in lib.exl3_last_error()
    assert fn(None, fake, 1, 10, 8, 288, fake, 4096, 0, None) != 0 and b"must be CUDA" in lib.exl3_last_error()
    assert fn(P(258), fake, 1, 10, 8, 288, fake, 4096, 0, None) != 0 and b"16-byte aligned" in lib.exl3_last_error()
    assert fn(None, None, 1, 0, 8, 288, None, 4096, 0, None) == 0                  # nothing to do
    rc = lib.exl3_grouped_gemm(None, 4, 128, None, None, 8, 8, 8, 8 * 8 * 64, None, None, 128, None, None, 0, fake,
                               fake, None, None, fake, 0, 128, 2, None, None)
    assert rc != 0 and b"routing dtypes" in lib.exl3_last_error()
    rc = lib.exl3_grouped_gemm(None, 4, 128, None, None, 8, 8, 8, 8 * 8 * 64, None, None, 128, None, None, 0, fake,
                               fake, None, None, fake, 0, 128, 3, None, None)
    assert rc != 0 and b"mode must be 0" in lib.exl3_last_error()


def test_wait_limit_setter_returns_previous_value(lib):
    prev = b200_ext.set_wait_limit_ns(-1)                 # the default
    try:
        assert b200_ext.set_wait_limit_ns(1234) == 2_000_000_000
        assert b200_ext.set_wait_limit_ns(0) == 1234
        assert b200_ext.set_wait_limit_ns(-5) == 0
        assert b200_ext.set_wait_limit_ns(-1) == 2_000_000_000
    finally:
        b200_ext.set_wait_limit_ns(prev)


def test_shim_checks_mirror_reference_messages(lib):
    i32 = torch.zeros(4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="int32 tensors"):
        b200_ext.build_blocks(i32.float(), i32, i32, i32)
    with pytest.raises(RuntimeError, match="too many experts"):
        b200_ext.build_blocks(torch.zeros(1025, dtype=torch.int32), i32, i32, i32)
    a = torch.zeros(4, 128, dtype=torch.float16)
    pk = torch.zeros(8, 8, 64, dtype=torch.int16)
    out = torch.zeros(4, 128)
    svh = torch.zeros(128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="tensors must be CUDA"):
        b200_ext.fat_gemm_v2(a, pk, out, svh, 4, True, False, 0)
    with pytest.raises(RuntimeError, match="a fp16 contiguous"):
        b200_ext.grouped_gemm(a.float(), pk[None], None, svh[None], None, None, None, i32, i32, None, None, out, 0)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(b200_ext, "_lib", None)
    monkeypatch.setenv("EXL3_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="not built"):
        b200_ext.load()
