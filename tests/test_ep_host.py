"""CPU, world_size 2 (gloo): the expert-parallel host logic of ep.ExpertParallel.

The orchestration under test is the product's (padding to tokens_per_rank, the routing all-gather, the
pull arguments, the global sort over routing slots, slicing this rank's experts out of it, local expert
offsets, the push, the barrier and the per-token reduce).  The device stages are replaced by a backend
built on the CPU oracle: the pull becomes a copy out of an all-gather of the token buffers (rows that the
pull did not request stay NaN, so a missing row poisons the result), and the pushes into the owners'
staging buffers a sum of per-rank staging arrays (every (token, source rank) row is written by one
rank), which is what the NVLink reads and stores compute.  The result must equal the oracle's
single-process grouped pipeline on all tokens with all experts."""
import os
import tempfile
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
PATHS = [os.path.join(REPO, "glm53-exl3-prefill_b200"), os.path.join(REPO, "oracle")]


class OracleBackend:
    """ep.ExpertParallel backend on the CPU oracle (test infrastructure)."""

    def __init__(self, group, rank, world, tpr, d, topk, combine_f16):
        self.group, self.rank, self.world, self.tpr, self.d, self.topk = group, rank, world, tpr, d, topk
        self.f16 = combine_f16
        self.x = torch.zeros(tpr, d, dtype=torch.float16)
        self.out = torch.zeros(tpr, d, dtype=torch.float32)
        self.slot_row = np.full(world * tpr * topk, -1, np.int64)
        self.x_all = self.x_view = self.acc = None
        self._layers = {}

    def all_gather(self, dst, src):
        dist.all_gather_into_tensor(dst, src, group=self.group)

    def publish(self):
        xa = torch.empty(self.world * self.tpr, self.d, dtype=torch.float16)
        dist.all_gather_into_tensor(xa, self.x.contiguous(), group=self.group)
        self.x_all = xa.numpy()
        self.acc = np.zeros((self.world * self.tpr * self.world, self.d), np.float32)

    def pull(self, ids_pos, e0, e1):
        ids = ids_pos.numpy()
        view = np.full_like(self.x_all, np.nan)
        own = slice(self.rank * self.tpr, (self.rank + 1) * self.tpr)
        view[own] = self.x_all[own]                       # this rank's tokens are read in place
        for t in range(self.world * self.tpr):
            if t // self.tpr != self.rank and any(e0 <= e < e1 for e in ids[t]):
                view[t] = self.x_all[t]
        self.x_view = view

    def barrier(self):
        t = torch.from_numpy(self.acc)
        dist.all_reduce(t, group=self.group)
        n = self.tpr * self.world
        self.staging = t[self.rank * n:(self.rank + 1) * n].numpy()

    def reduce(self, ids_pos, n_experts, T):
        import ep
        ids = ids_pos.numpy()
        for t in range(T):
            ranks = sorted({ep.owner_rank(int(e), n_experts, self.world) for e in ids[t] if 0 <= e < n_experts})
            acc = np.zeros(self.d, np.float32)
            for r in ranks:
                acc += self.staging[t * self.world + r]
            self.out[t] = torch.from_numpy(acc)

    def local_ids(self, ids_pos, e0, e1, out):
        ids = ids_pos.numpy()
        out.copy_(torch.from_numpy(np.where((ids >= e0) & (ids < e1), ids - e0, -1)))

    def route_sort(self, ids, w, n_experts, bufs):
        import oracle
        s = oracle.route_sort(ids.numpy(), w.numpy(), n_experts)
        bufs.token_sorted.copy_(torch.from_numpy(s["token_sorted"]))
        bufs.weight_sorted.copy_(torch.from_numpy(s["weight_sorted"]))
        bufs.expert_of_row.copy_(torch.from_numpy(s["expert_of_row"]))
        bufs.counts.copy_(torch.from_numpy(s["counts"]))
        bufs.expert_row0.copy_(torch.from_numpy(s["expert_row0"]))
        bufs.meta[1] = int(s["counts"].sum())              # this rank's rows, first in the sorted arrays

    def _layer(self, layer):
        import oracle
        key = id(layer)
        if key not in self._layers:
            self._layers[key] = oracle.Layer(*(getattr(layer, n).numpy() for n in
                                              ("w13_trellis", "w13_suh", "w13_svh", "w2_trellis", "w2_suh", "w2_svh")))
        return self._layers[key]

    def row_had(self, h13, slot_sorted, expert_of_row, rows_dev, suh):
        import oracle
        n = int(rows_dev[0])
        ss = slot_sorted.numpy()[:n]
        h = oracle.row_had(self.x_view, ss // self.topk, expert_of_row.numpy()[:n], suh.numpy())
        assert not np.isnan(h).any(), "stage 2 read a token row that was neither local nor pulled"
        h13[:n].copy_(torch.from_numpy(h))
        self.slot_row[:] = -1
        self.slot_row[ss] = np.arange(n)

    def gemm_gate_up(self, h13, layer, counts, row0, gu):
        import oracle
        L = self._layer(layer)
        f = L.f
        a = h13.numpy()
        for e in range(L.E):
            c, r0 = int(counts[e]), int(row0[e])
            if c == 0:
                continue
            wg, wu, _ = L.decoded(e)
            gu[r0:r0 + c, :f] = torch.from_numpy(oracle.f2h(oracle.fat_gemm_ref(a[r0:r0 + c], None, L.w13_svh[e, 0], w=wg)))
            gu[r0:r0 + c, f:] = torch.from_numpy(oracle.f2h(oracle.fat_gemm_ref(a[r0:r0 + c], None, L.w13_svh[e, 1], w=wu)))

    def act_had(self, gu, act, expert_of_row, rows_dev, suh, limit):
        import oracle
        n = int(rows_dev[0])
        act[:n].copy_(torch.from_numpy(oracle.act_had(gu.numpy()[:n], expert_of_row.numpy()[:n], suh.numpy(), limit)))

    def gemm_down(self, act, layer, counts, row0, weight_sorted, y):
        import oracle
        L = self._layer(layer)
        a, ws = act.numpy(), weight_sorted.numpy().astype(np.float32)
        for e in range(L.E):
            c, r0 = int(counts[e]), int(row0[e])
            if c == 0:
                continue
            _, _, wd = L.decoded(e)
            y[r0:r0 + c] = torch.from_numpy(oracle.fat_gemm_ref(a[r0:r0 + c], None, L.w2_svh[e], w=wd)
                                            * ws[r0:r0 + c, None])

    def push(self, y, ids_pos, e0, e1):
        ids, yl = ids_pos.numpy(), y.numpy()
        for t in range(self.world * self.tpr):
            js = [j for j in range(self.topk) if e0 <= ids[t, j] < e1]
            if not js:
                continue
            acc = np.zeros(self.d, np.float32)
            for j in js:
                r = self.slot_row[t * self.topk + j]
                assert r >= 0, "a routed slot has no row"
                acc += yl[r]
            if self.f16:
                acc = acc.astype(np.float16).astype(np.float32)
            dst = (t % self.tpr) * self.world + self.rank + (t // self.tpr) * self.tpr * self.world
            assert not self.acc[dst].any(), "a (token, rank) row was written twice"
            self.acc[dst] = acc

    def close(self):
        pass


def _rendezvous_file():
    """A fresh file for a file:// rendezvous (no TCP port that a previous run may still hold)."""
    fd, path = tempfile.mkstemp(prefix="exl3_ep_rdzv_")
    os.close(fd)
    os.unlink(path)
    return path


def _worker(rank, world, rdzv, case):
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import ep
    import oracle
    import synth
    dist.init_process_group("gloo", init_method="file://" + rdzv, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        E, d, f, k, tpr = 8, 256, 256, 2, 48
        tokens = case["tokens"]
        T_all = sum(tokens)
        layer = synth.make_layer(E, d, f, seed=5, sv_scale=0.05)
        x_all = synth.make_x(T_all, d, seed=6)
        ids_all, w_all = synth.routing("zipf", max(T_all, 1), E, k, seed=7)
        ids_all, w_all = ids_all[:T_all], w_all[:T_all]
        if case.get("experts_lt") is not None:
            ids_all = ids_all % case["experts_lt"]            # leave the last rank's experts unrouted
        off = sum(tokens[:rank])
        mine = slice(off, off + tokens[rank])
        e0, e1 = ep.expert_range(rank, world, E)
        placement = None
        if case.get("placement") == "random":
            placement = torch.randperm(E, generator=torch.Generator().manual_seed(3)).tolist()
        elif case.get("placement") == "balanced":
            placement = ep.balanced_placement(torch.bincount(ids_all.flatten(), minlength=E).tolist(), world)
        lay = ep.layer_slice(layer, e0, e1) if placement is None else ep.layer_take(layer, placement[e0:e1])
        f16 = case.get("combine") == "fp16"
        eng = ep.ExpertParallel(tpr, d, E, k, f, device=torch.device("cpu"),
                                backend=OracleBackend(None, rank, world, tpr, d, k, f16), placement=placement,
                                combine_dtype=torch.float16 if f16 else torch.float32)
        for _ in range(case.get("calls", 1)):                # the buffers are reused call after call
            got = eng.prefill(x_all[mine], ids_all[mine], w_all[mine], lay, 7.0, copy=True)
        L = oracle.Layer(*(getattr(layer, n).numpy() for n in
                           ("w13_trellis", "w13_suh", "w13_svh", "w2_trellis", "w2_suh", "w2_svh")))
        want = oracle.grouped_staged(x_all.numpy(), ids_all.numpy(), w_all.numpy(), L, 7.0)[mine]
        assert got.shape == (tokens[rank], d)
        if tokens[rank]:
            # fp32 partial sums: only the summation order differs; fp16: one rounding per (token, rank) sum
            tol = 1e-3 if f16 else 1e-6
            assert oracle.rel_l2(got.numpy(), want) < tol, (rank, oracle.rel_l2(got.numpy(), want))
        with pytest.raises(RuntimeError, match="exceed tokens_per_rank"):
            eng.prefill(torch.zeros(tpr + 1, d, dtype=torch.float16), torch.zeros(tpr + 1, k, dtype=torch.int64),
                        torch.ones(tpr + 1, k), lay, 7.0)
        with pytest.raises(RuntimeError, match="this rank's experts"):
            eng.prefill(x_all[mine], ids_all[mine], w_all[mine], ep.layer_slice(layer, 0, E), 7.0)
        eng.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [
    dict(tokens=[40, 33]),                      # unequal token counts, padding to tokens_per_rank
    dict(tokens=[48, 48], calls=2),             # full buffers, two calls in a row
    dict(tokens=[30, 0]),                       # a rank without tokens
    dict(tokens=[25, 31], experts_lt=4),        # the second rank's experts receive no rows
    dict(tokens=[40, 33], placement="random"),  # experts placed by an arbitrary permutation
    dict(tokens=[48, 41], placement="balanced", calls=2),
    dict(tokens=[40, 33], placement="random", combine="fp16"),
])
def test_expert_parallel_host_logic_matches_single_process_pipeline(case):
    mp.spawn(_worker, args=(2, _rendezvous_file(), case), nprocs=2, join=True)


def test_expert_ranges_cover_all_experts_once():
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import ep
    for E in (8, 16, 288, 1024):
        for world in (1, 2, 3, 4, 8):
            ranges = [ep.expert_range(r, world, E) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == E
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert all(e1 > e0 for e0, e1 in ranges)
            # owner_rank (the reduce kernel's rank_of) inverts expert_range
            assert all(ep.owner_rank(e, E, world) == r for r, (e0, e1) in enumerate(ranges) for e in range(e0, e1))


def test_balanced_placement_is_a_partition_and_balances_zipf_load():
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import ep
    import synth
    E, world = 288, 8
    ids, _ = synth.routing("zipf", 8192, E, 8, seed=1, popularity_seed=9)
    counts = torch.bincount(ids.flatten(), minlength=E).tolist()
    pl = ep.balanced_placement(counts, world)
    assert sorted(pl) == list(range(E))

    def loads(order):
        return [sum(counts[e] for e in order[slice(*ep.expert_range(r, world, E))]) for r in range(world)]
    contiguous, balanced = loads(list(range(E))), loads(pl)
    # the hottest expert alone holds 0.87 of a rank's average rows and its rank still takes E/N - 1 more
    # experts, so about 1.08x the average is the floor without replicating experts
    assert max(balanced) <= 1.10 * (sum(counts) / world)
    assert max(balanced) < 0.8 * max(contiguous)
    # a later batch of the same router stays balanced with the placement fitted on the first
    ids2, _ = synth.routing("zipf", 8192, E, 8, seed=2, popularity_seed=9)
    counts = torch.bincount(ids2.flatten(), minlength=E).tolist()
    assert max(loads(pl)) <= 1.15 * (sum(counts) / world)
