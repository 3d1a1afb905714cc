"""GPU: exl3_route_sort_noalloc, the routing entry point for callers that cannot allocate device memory
while the prefill runs (an engine whose KV cache already holds nearly all of the GPU, or a host program
that drives the C ABI without a device allocator).  It keeps its chunk histograms in a fixed array
inside the library instead of a caller buffer; its results must be those of exl3_route_sort, call
after call, and routings too large for the array must be refused with a clear message.

Collected last on purpose (test_zz_*), and written so that it passes alone in a fresh process too."""
import ctypes

import pytest
import torch

import synth

pytestmark = pytest.mark.gpu

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int


def _bind(lib):
    fn = lib.exl3_route_sort_noalloc
    fn.argtypes = [_P, _I32, _P, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]
    fn.restype = _I32
    return fn


def _buffers(dev, R, E):
    mb = R // 128 + E
    return [torch.full((R,), -5, dtype=torch.int64, device=dev), torch.full((R,), 7.0, dtype=torch.float16, device=dev),
            torch.full((R,), -5, dtype=torch.int32, device=dev), torch.full((E,), -5, dtype=torch.int32, device=dev),
            torch.full((E,), -5, dtype=torch.int32, device=dev), torch.full((mb,), -5, dtype=torch.int32, device=dev),
            torch.full((mb,), -7, dtype=torch.int32, device=dev), torch.full((2,), -5, dtype=torch.int32, device=dev),
            torch.full((1,), -5, dtype=torch.int32, device=dev)]


def _noalloc(fn, ids, w, E, outs):
    stream = torch.cuda.current_stream(ids.device).cuda_stream
    wdt = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[w.dtype]
    return fn(ids.data_ptr(), 1 if ids.dtype == torch.int64 else 0, w.data_ptr(), wdt, ids.shape[0], ids.shape[1], E,
              outs[5].numel(), *[o.data_ptr() for o in outs], stream)


def test_noalloc_route_sort_matches_the_scratch_entry_point(ext, cuda_device):
    lib = ext.load()
    fn = _bind(lib)
    dev = cuda_device
    cases = [("zipf", 4096, 288, 8, 11), ("uniform", 1000, 64, 6, 12)]
    for kind, T, E, k, seed in cases:                    # two calls in a row, different shapes
        ids, w = synth.routing(kind, T, E, k, seed=seed, device=dev)
        want = _buffers(dev, T * k, E)
        ext.route_sort(ids, w, E, *want)
        got = _buffers(dev, T * k, E)
        rc = _noalloc(fn, ids, w, E, got)
        assert rc == 0, lib.exl3_last_error()
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            assert torch.equal(a.view(torch.int16) if a.dtype == torch.float16 else a,
                               b.view(torch.int16) if b.dtype == torch.float16 else b), kind


def test_noalloc_route_sort_refuses_routings_beyond_its_array(ext, cuda_device):
    lib = ext.load()
    fn = _bind(lib)
    dev = cuda_device
    E, k = 1024, 8
    T = 140000 // k + 1024                                # needs more than 65536 int32 of scratch
    assert ext.route_sort_scratch_elems(T * k, E) > 65536
    ids = torch.zeros(T, k, dtype=torch.int64, device=dev)
    w = torch.ones(T, k, device=dev)
    outs = _buffers(dev, T * k, E)
    rc = _noalloc(fn, ids, w, E, outs)
    assert rc != 0
    assert b"built-in array holds 65536" in lib.exl3_last_error()
