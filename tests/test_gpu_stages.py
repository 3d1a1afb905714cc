"""GPU parity of each stage against the CPU oracle / reference goldens, through the C-ABI library.

Bars: sort and block tables bit-exact (reference runtime goldens); row_had bit-exact (same fp32
butterfly order as the oracle); act_had within 1 fp16 ulp (exp differs between CUDA and libm);
GEMM stage rel-L2 <= 1e-4 against the fat-GEMM reference restatement (kernel/test_fat_v2.py:87-95)."""
import os

import numpy as np
import pytest
import torch

import oracle
import synth
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
GEMM_TOL = 1e-4


def _case(z, name):
    return {k.split("__", 1)[1]: z[k] for k in z.files if k.startswith(name + "__")}


def _weights(c):
    wd = str(c["weight_dtype"])
    if wd == "f32":
        return torch.from_numpy(c["weights"])
    return torch.from_numpy(c["weights"].view(np.int16)).view(torch.float16 if wd == "f16" else torch.bfloat16)


def _route(ext, dev, ids, w, E, sentinel=-7):
    T, k = ids.shape
    R = T * k
    mb = R // 128 + E
    outs = dict(token_sorted=torch.full((R,), -5, dtype=torch.int64, device=dev),
                weight_sorted=torch.full((R,), 9.0, dtype=torch.float16, device=dev),
                expert_of_row=torch.full((R,), -5, dtype=torch.int32, device=dev),
                counts=torch.full((E,), -5, dtype=torch.int32, device=dev),
                expert_row0=torch.full((E,), -5, dtype=torch.int32, device=dev),
                block_expert=torch.full((mb,), -5, dtype=torch.int32, device=dev),
                block_row0=torch.full((mb,), sentinel, dtype=torch.int32, device=dev),
                meta=torch.full((2,), -5, dtype=torch.int32, device=dev),
                invalid=torch.full((1,), -5, dtype=torch.int32, device=dev))
    ext.route_sort(ids.to(dev).contiguous(), w.to(dev).contiguous(), E, outs["token_sorted"], outs["weight_sorted"],
                   outs["expert_of_row"], outs["counts"], outs["expert_row0"], outs["block_expert"],
                   outs["block_row0"], outs["meta"], outs["invalid"])
    torch.cuda.synchronize()
    return {k: v.cpu() for k, v in outs.items()}


# ------------------------------------------------------------------------------------ stage 1
def test_route_sort_bit_exact_vs_reference_runtime(ext, cuda_device):
    z = np.load(os.path.join(GOLDEN, "sort_cases.npz"))
    for name in [str(n) for n in z["case_names"]]:
        c = _case(z, name)
        E = int(c["n_experts"])
        for ids_dtype in (torch.int64, torch.int32):
            got = _route(ext, cuda_device, torch.from_numpy(c["ids"]).to(ids_dtype), _weights(c), E)
            assert np.array_equal(got["token_sorted"].numpy(), c["token_sorted"]), name
            assert np.array_equal(got["expert_of_row"].numpy(), c["expert_of_row"]), name
            assert np.array_equal(got["weight_sorted"].view(torch.int16).numpy().view(np.uint16), c["weight_sorted"]), name
            assert np.array_equal(got["counts"].numpy(), c["counts"]), name
            assert np.array_equal(got["expert_row0"].numpy(), c["expert_row0"]), name
            assert np.array_equal(got["block_expert"].numpy(), c["block_expert"]), name
            assert np.array_equal(got["block_row0"].numpy(), c["block_row0"]), name     # tail keeps the sentinel
            assert np.array_equal(got["meta"].numpy(), c["meta"]), name
            assert int(got["invalid"][0]) == 0


def test_build_blocks_bit_exact(ext, cuda_device):
    z = np.load(os.path.join(GOLDEN, "sort_cases.npz"))
    for name in [str(n) for n in z["case_names"]]:
        c = _case(z, name)
        mb = int(c["max_blocks"])
        counts = torch.from_numpy(c["counts"]).to(cuda_device)
        be = torch.full((mb,), 123, dtype=torch.int32, device=cuda_device)
        br = torch.full((mb,), -7, dtype=torch.int32, device=cuda_device)
        meta = torch.zeros(2, dtype=torch.int32, device=cuda_device)
        ext.build_blocks(counts, be, br, meta)
        assert np.array_equal(be.cpu().numpy(), c["block_expert"]), name
        assert np.array_equal(br.cpu().numpy(), c["block_row0"]), name
        assert np.array_equal(meta.cpu().numpy(), c["meta"]), name


def test_route_sort_invalid_ids_are_counted_and_tail_is_safe(ext, cuda_device):
    ids = torch.tensor([[0, 5], [3, -1], [9, 1], [2, 2]], dtype=torch.int64)
    w = torch.rand(4, 2)
    got = _route(ext, cuda_device, ids, w, 4)
    s = oracle.route_sort(ids.numpy(), w.numpy(), 4)
    assert int(got["invalid"][0]) == 3 == s["invalid"]
    n = int(s["counts"].sum())
    assert np.array_equal(got["token_sorted"][:n].numpy(), s["token_sorted"][:n])
    assert np.array_equal(got["counts"].numpy(), s["counts"])
    assert bool((got["token_sorted"][n:] == 0).all()) and bool((got["expert_of_row"][n:] == 0).all())


# ------------------------------------------------------------------------------------ stages 2 and 4
@pytest.mark.parametrize("K,T,E,k", [(4096, 64, 16, 4), (384, 33, 5, 3), (128, 7, 3, 2), (1024, 256, 16, 4)])
def test_row_had_bit_exact(ext, cuda_device, K, T, E, k):
    g = torch.Generator().manual_seed(K + T)
    x = synth.make_x(T, K, seed=K)
    suh2 = (torch.rand(E, 2, K, generator=g) + 0.5).half() * torch.where(torch.rand(E, 2, K, generator=g) < 0.5, -1, 1).half()
    ids, w = synth.routing("uniform", T, E, k, seed=T)
    s = oracle.route_sort(ids.numpy(), w.numpy(), E)
    R = T * k
    want = oracle.row_had(x.numpy(), s["token_sorted"], s["expert_of_row"], suh2[:, 0].numpy(), gather=True)
    dst = torch.empty(R, K, dtype=torch.float16, device=cuda_device)
    suh_dev = suh2.to(cuda_device)
    ext.row_had(x.to(cuda_device), dst, torch.from_numpy(s["token_sorted"]).to(cuda_device),
                torch.from_numpy(s["expert_of_row"]).to(cuda_device), suh_dev[:, 0], True)
    assert np.array_equal(dst.cpu().numpy().view(np.uint16), want.view(np.uint16))
    # non-gather form: src row r
    want2 = oracle.row_had(want, None, s["expert_of_row"], suh2[:, 1].numpy(), gather=False)
    dst2 = torch.empty_like(dst)
    ext.row_had(dst, dst2, None, torch.from_numpy(s["expert_of_row"]).to(cuda_device), suh_dev[:, 1], False)
    assert np.array_equal(dst2.cpu().numpy().view(np.uint16), want2.view(np.uint16))


@pytest.mark.parametrize("I,R,E,scale", [(1536, 300, 8, 30.0), (512, 1000, 16, 3.0), (128, 5, 2, 1.0), (384, 77, 4, 0.2)])
def test_act_had_within_one_ulp(ext, cuda_device, I, R, E, scale):
    g = torch.Generator().manual_seed(I + R)
    gu = (torch.randn(R, 2 * I, generator=g) * scale).half()
    eor = torch.randint(0, E, (R,), generator=g, dtype=torch.int32)
    suh = (torch.rand(E, I, generator=g) + 0.5).half()
    want = oracle.act_had(gu.numpy(), eor.numpy(), suh.numpy(), 7.0)
    act = torch.empty(R, I, dtype=torch.float16, device=cuda_device)
    ext.act_had(gu.to(cuda_device), act, eor.to(cuda_device), suh.to(cuda_device), 7.0)
    got = act.cpu().numpy()
    # The only non-exact step is exp (CUDA expf vs libm): a rare 1-ulp change of a pre-Hadamard fp16
    # value spreads over its 128-column block, so compare per row and bound how often anything differs.
    diff = got.astype(np.float64) - want.astype(np.float64)
    rows = np.linalg.norm(diff, axis=1) / np.maximum(np.linalg.norm(want.astype(np.float64), axis=1), 1e-30)
    assert oracle.rel_l2(got, want) < 1e-4
    assert float(rows.max()) < 2e-3
    assert float((diff != 0).mean()) < 5e-3


# ------------------------------------------------------------------------------------ stages 3 and 5
def _grouped_problem(E, d, f, counts, seed, sv_scale=1.0):
    layer = synth.make_layer(E, d, f, seed=seed, sv_scale=sv_scale)
    counts = np.asarray(counts, np.int32)
    R = int(counts.sum())
    g = torch.Generator().manual_seed(seed)
    row0 = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
    return layer, counts, row0, R, g


@pytest.mark.parametrize("counts", [[300, 0, 1, 128, 129, 256, 257, 5], [2000, 7, 0, 0, 64, 511, 512, 513]])
def test_grouped_gemm_gate_up_vs_fat_gemm_reference(ext, cuda_device, counts):
    E, d, f = len(counts), 1024, 512
    layer, counts, row0, R, g = _grouped_problem(E, d, f, counts, seed=sum(counts))
    a = (torch.randn(R, d, generator=g) * 0.5).half()
    dev = cuda_device
    L = synth.layer_to(layer, dev)
    gu = torch.full((R, 2 * f), float("nan"), dtype=torch.float16, device=dev)
    ext.grouped_gemm(a.to(dev), L.w13_trellis[:, 0], L.w13_trellis[:, 1], L.w13_svh[:, 0], L.w13_svh[:, 1],
                     None, None, torch.from_numpy(counts).to(dev), torch.from_numpy(row0).to(dev), None, None, gu, 0)
    got = gu.float().cpu().numpy()
    an = a.numpy()
    for e in range(E):
        c, r0 = int(counts[e]), int(row0[e])
        if c == 0:
            continue
        for j in range(2):
            want = oracle.fat_gemm_ref(an[r0:r0 + c], layer.w13_trellis[e, j].numpy(), layer.w13_svh[e, j].numpy())
            want16 = oracle.f2h(want).astype(np.float32)
            sl = got[r0:r0 + c, j * f:(j + 1) * f]
            assert np.isfinite(sl).all(), (e, j)
            assert oracle.rel_l2(sl, want) < GEMM_TOL + 4e-4, (e, j)      # fp16 output rounding vs fp32 ref
            assert oracle.rel_l2(sl, want16) < GEMM_TOL, (e, j)          # same rounding point as the reference
    assert int(ext.read_status(dev)) == 0


@pytest.mark.parametrize("counts,T", [([300, 0, 1, 128, 129, 256, 257, 5], 1200), ([700, 3, 0, 255], 800)])
def test_grouped_gemm_down_scatter_vs_reference(ext, cuda_device, counts, T):
    E, d, f = len(counts), 1024, 512
    layer, counts, row0, R, g = _grouped_problem(E, d, f, counts, seed=sum(counts) + 1)
    act = (torch.randn(R, f, generator=g) * 2.0).half()
    tok = torch.cat([torch.randperm(T, generator=g)[:c] for c in counts]).to(torch.int64)
    rw = (torch.rand(R, generator=g) * 0.5 + 0.25).half()
    dev = cuda_device
    L = synth.layer_to(layer, dev)
    out = torch.zeros(T, d, dtype=torch.float32, device=dev)
    ext.grouped_gemm(act.to(dev), L.w2_trellis, None, L.w2_svh, None, None, None, torch.from_numpy(counts).to(dev),
                     torch.from_numpy(row0).to(dev), tok.to(dev), rw.to(dev), out, 1)
    want = np.zeros((T, d), np.float32)
    an = act.numpy()
    for e in range(E):
        c, r0 = int(counts[e]), int(row0[e])
        if c == 0:
            continue
        y = oracle.fat_gemm_ref(an[r0:r0 + c], layer.w2_trellis[e].numpy(), layer.w2_svh[e].numpy())
        np.add.at(want, tok[r0:r0 + c].numpy(), y * rw[r0:r0 + c].numpy().astype(np.float32)[:, None])
    assert oracle.rel_l2(out.cpu().numpy(), want) < GEMM_TOL


@pytest.mark.parametrize("counts,T,k", [([300, 0, 1, 128, 129, 256, 257, 5], 300, 4), ([700, 3, 0, 255], 400, 3)])
def test_grouped_gemm_down_row_store_and_combine(ext, cuda_device, counts, T, k):
    """Mode 2 stores w[r] * y[r] at row slot[r]; combine_slots sums each token's slot rows (ids in range,
    j ascending).  Together: the reference's scatter (kernel/exl3_grouped_prefill.cu:274-275) without
    atomics.  Slots of invalid ids are never written and must not be read."""
    E, d, f = len(counts), 1024, 512
    layer, counts, row0, R, g = _grouped_problem(E, d, f, counts, seed=sum(counts) + 2)
    assert R <= T * k
    act = (torch.randn(R, f, generator=g) * 2.0).half()
    slots = torch.randperm(T * k, generator=g)[:R].to(torch.int64)              # every routed row its own slot
    ids = torch.full((T * k,), -1, dtype=torch.int64)
    eor = np.repeat(np.arange(E), counts)
    ids[slots] = torch.from_numpy(eor).to(torch.int64)
    ids = ids.view(T, k)
    rw = (torch.rand(R, generator=g) * 0.5 + 0.25).half()
    dev = cuda_device
    L = synth.layer_to(layer, dev)
    y = torch.full((T * k, d), float("nan"), dtype=torch.float32, device=dev)   # unwritten rows stay NaN
    ext.grouped_gemm(act.to(dev), L.w2_trellis, None, L.w2_svh, None, None, None, torch.from_numpy(counts).to(dev),
                     torch.from_numpy(row0).to(dev), slots.to(dev), rw.to(dev), y, 2)
    out = torch.full((T, d), float("nan"), dtype=torch.float32, device=dev)
    ext.combine_slots(y, ids.to(dev), E, out)
    base = torch.ones(T, d, dtype=torch.float32, device=dev)
    ext.combine_slots(y, ids.to(torch.int32).to(dev), E, base, accumulate=True)
    torch.cuda.synchronize()
    an = act.numpy()
    want_y = np.zeros((T * k, d), np.float32)
    for e in range(E):
        c, r0 = int(counts[e]), int(row0[e])
        if c == 0:
            continue
        yv = oracle.fat_gemm_ref(an[r0:r0 + c], layer.w2_trellis[e].numpy(), layer.w2_svh[e].numpy())
        want_y[slots[r0:r0 + c].numpy()] = yv * rw[r0:r0 + c].numpy().astype(np.float32)[:, None]
    got_y = y.cpu().numpy()
    assert oracle.rel_l2(got_y[slots.numpy()], want_y[slots.numpy()]) < GEMM_TOL
    want = np.zeros((T, d), np.float32)
    idn = ids.numpy()
    for t in range(T):
        for j in range(k):
            if 0 <= idn[t, j] < E:
                want[t] += got_y[t * k + j]
    assert np.array_equal(out.cpu().numpy(), want)                                # same order, same bits
    assert oracle.rel_l2(base.cpu().numpy(), 1.0 + want) < 1e-6                   # added onto the existing out
    assert int(ext.read_status(dev)) == 0


@pytest.mark.parametrize("counts", [[300, 0, 1, 128, 129, 256, 257, 5, 16, 17, 100, 33],
                                    [64, 3, 1, 2, 120, 127, 128, 96, 8, 9, 31, 32],
                                    [96, 97, 352, 353, 65, 63, 0, 1]])
def test_thin_kernel_matches_the_256_row_kernel(ext, cuda_device, counts, monkeypatch):
    """With EXL3_B200_THIN_MAX_ROWS=128 tiles of 1..128 rows run on the thin kernel (decoded weights in TMEM
    as the A operand, D^T); EXL3_B200_THIN_KERNEL=0 sends them to the 256-row kernel, and
    EXL3_B200_THIN_MAX_ROWS=64 / 96 (the default) split them (1..64 or 1..96 rows thin, the rest of the
    one-block tiles on the 256-row kernel; 96/97 and 352/353 rows sit on the default's boundary): all must
    give the same rows (up to the tensor cores' accumulation order), for gate|up (mode 0) and the down row
    store (mode 2)."""
    E, d, f = len(counts), 1024, 512
    layer, counts, row0, R, g = _grouped_problem(E, d, f, counts, seed=sum(counts) + 3)
    a = (torch.randn(R, d, generator=g) * 0.5).half()
    act = (torch.randn(R, f, generator=g) * 2.0).half()
    rw = (torch.rand(R, generator=g) * 0.5 + 0.25).half()
    dev = cuda_device
    L = synth.layer_to(layer, dev)
    c_d, r_d = torch.from_numpy(counts).to(dev), torch.from_numpy(row0).to(dev)
    slots = torch.arange(R, dtype=torch.int64, device=dev)
    outs = {}
    for flag, max_rows in (("1", "128"), ("0", "128"), ("1", "64"), ("1", "96")):    # all thin / none / splits
        monkeypatch.setenv("EXL3_B200_THIN_KERNEL", flag)
        monkeypatch.setenv("EXL3_B200_THIN_MAX_ROWS", max_rows)
        gu = torch.full((R, 2 * f), float("nan"), dtype=torch.float16, device=dev)
        ext.grouped_gemm(a.to(dev), L.w13_trellis[:, 0], L.w13_trellis[:, 1], L.w13_svh[:, 0], L.w13_svh[:, 1],
                         None, None, c_d, r_d, None, None, gu, 0)
        y = torch.full((R, d), float("nan"), dtype=torch.float32, device=dev)
        ext.grouped_gemm(act.to(dev), L.w2_trellis, None, L.w2_svh, None, None, None, c_d, r_d, slots, rw.to(dev), y, 2)
        torch.cuda.synchronize()
        outs[flag + max_rows] = (gu.float().cpu().numpy(), y.cpu().numpy())
    outs["1"] = outs["1128"]
    for j in range(2):
        for key in ("1128", "0128", "164", "196"):
            assert np.isfinite(outs[key][j]).all()
        assert oracle.rel_l2(outs["1128"][j], outs["0128"][j]) < 2e-6, j
        assert oracle.rel_l2(outs["164"][j], outs["0128"][j]) < 2e-6, j
        assert oracle.rel_l2(outs["196"][j], outs["0128"][j]) < 2e-6, j
    an = a.numpy()
    for e in range(E):                                            # and the thin rows against the reference
        c, r0 = int(counts[e]), int(row0[e])
        if c == 0:
            continue
        want = oracle.fat_gemm_ref(an[r0:r0 + c], layer.w13_trellis[e, 0].numpy(), layer.w13_svh[e, 0].numpy())
        assert oracle.rel_l2(outs["1"][0][r0:r0 + c, :f], oracle.f2h(want).astype(np.float32)) < GEMM_TOL, e
    assert int(ext.read_status(dev)) == 0


@pytest.mark.parametrize("M", [300, 1, 128, 513])
def test_fat_gemm_v2_all_variants(ext, cuda_device, M):
    """kernel/test_fat_v2.py:116-140: gate|up (K=d, N=2f) direct and down (K=f, N=d) scatter, M=300 has a
    partial last block."""
    import exl3_fat_gemm_v2 as ext2
    d, f = 1024, 512
    g = torch.Generator().manual_seed(M)
    packed13 = torch.randint(-32768, 32768, (d // 16, 2 * f // 16, 64), generator=g, dtype=torch.int16)
    svh13 = (torch.rand(2 * f, generator=g) + 0.5).half()
    h13 = (torch.randn(M, d, generator=g) * 0.5).half()
    want = oracle.fat_gemm_ref(h13.numpy(), packed13.numpy(), svh13.numpy())
    dev = cuda_device
    for v in range(4):
        out = torch.empty(M, 2 * f, dtype=torch.float32, device=dev)
        ext2.fat_gemm_v2(h13.to(dev), packed13.to(dev), out, svh13.to(dev), 4, True, False, v)
        assert oracle.rel_l2(out.cpu().numpy(), want) < GEMM_TOL, v
    out = torch.empty(M, 2 * f, dtype=torch.float32, device=dev)
    ext2.exl3_fat_gemm(h13.to(dev), packed13.to(dev), out, svh13.to(dev), 4, True, False)
    assert oracle.rel_l2(out.cpu().numpy(), want) < GEMM_TOL
    packed2 = torch.randint(-32768, 32768, (f // 16, d // 16, 64), generator=g, dtype=torch.int16)
    svh2 = (torch.rand(d, generator=g) + 0.5).half()
    h2 = (torch.randn(M, f, generator=g) * 0.5).half()
    tok = torch.randperm(4096, generator=g)[:M].contiguous()
    rw = (torch.rand(M, generator=g) * 0.5 + 0.25).half()
    want_s = oracle.fat_gemm_scatter_ref(h2.numpy(), packed2.numpy(), svh2.numpy(), tok.numpy(), rw.numpy(), 4096)
    base = torch.randn(4096, d, generator=g)
    for v in range(4):
        out_s = base.clone().to(dev)
        ext2.fat_gemm_v2_scatter(h2.to(dev), packed2.to(dev), out_s, svh2.to(dev), tok.to(dev), rw.to(dev), 4, True,
                                 False, v)
        assert oracle.rel_l2(out_s.cpu().numpy() - base.numpy(), want_s) < GEMM_TOL, v
    with pytest.raises(RuntimeError, match="only K4 MCG tensors"):
        ext2.fat_gemm_v2(h13.to(dev), packed13.to(dev), out, svh13.to(dev), 3, True, False, 0)
    with pytest.raises(RuntimeError, match="unknown variant"):
        ext2.fat_gemm_v2(h13.to(dev), packed13.to(dev), out, svh13.to(dev), 4, True, False, 4)


@pytest.mark.parametrize("N,K,M", [(384, 256, 300), (640, 512, 700), (128, 64, 5)])
def test_fat_gemm_odd_column_groups_use_single_cta_kernel(ext, cuda_device, N, K, M):
    """N/128 odd: the column tiles cannot all be paired, so the single-CTA kernel runs; same bar."""
    import exl3_fat_gemm_v2 as ext2
    g = torch.Generator().manual_seed(N + K)
    packed = torch.randint(-32768, 32768, (K // 16, N // 16, 64), generator=g, dtype=torch.int16)
    svh = (torch.rand(N, generator=g) + 0.5).half()
    a = (torch.randn(M, K, generator=g) * 0.5).half()
    want = oracle.fat_gemm_ref(a.numpy(), packed.numpy(), svh.numpy())
    out = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
    ext2.fat_gemm_v2(a.to(cuda_device), packed.to(cuda_device), out, svh.to(cuda_device), 4, True, False, 1)
    assert oracle.rel_l2(out.cpu().numpy(), want) < GEMM_TOL
    tok = torch.randperm(2 * M, generator=g)[:M].contiguous()
    rw = (torch.rand(M, generator=g) * 0.5 + 0.25).half()
    want_s = oracle.fat_gemm_scatter_ref(a.numpy(), packed.numpy(), svh.numpy(), tok.numpy(), rw.numpy(), 2 * M)
    out_s = torch.zeros(2 * M, N, dtype=torch.float32, device=cuda_device)
    ext2.fat_gemm_v2_scatter(a.to(cuda_device), packed.to(cuda_device), out_s, svh.to(cuda_device),
                             tok.to(cuda_device), rw.to(cuda_device), 4, True, False, 2)
    assert oracle.rel_l2(out_s.cpu().numpy(), want_s) < GEMM_TOL
    assert ext.read_status(cuda_device) == 0
