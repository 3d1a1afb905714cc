"""Expert-parallel prefill of one routed-expert MoE layer over N GPUs, one process per GPU.

No reference counterpart: the reference refuses expert-parallel layers (kernel/exl3_grouped_runtime.py:96-98,
``layer.expert_map is not None`` falls back to the original path).  This module adds it, B200-first:

* experts are split into ranges of E/N, rank r owning positions [r*E/N, (r+1)*E/N) of a placement (a
  permutation of the expert ids; the identity by default); tokens live on the rank that produced them, in
  a buffer of ``tokens_per_rank`` rows.  A global token index t is row t % tokens_per_rank of rank
  t // tokens_per_rank;
* routing: every rank all-gathers the (small) routing of all ranks and sorts, with the GPU expert sort,
  the list of N*tokens_per_rank*topk routing slots (slot s = t*topk + j) keeping only the slots that go
  to its own experts (positions [e0, e1) become local expert ids, every other slot is left unrouted).
  No index exchange is needed, every sorted row knows both its token (s // topk) and its slot, and the
  sort's work grows with this rank's experts, not with all E.  The number of this rank's rows stays on
  the device (the sort's meta[1]): stages 2 and 4 read it there and the workspace is sized for the worst
  case, so the layer issues without a host synchronisation;
* dispatch: ``ep_pull_rows`` copies each remote token row that has a route to this rank's experts into a
  local buffer, once (a token routed to several of this rank's experts crosses NVLink once), reading
  the owners' token buffers in place (mapped with CUDA IPC), on a side stream beside the routing sort;
  stage 2 (``ep_row_had``) then gathers locally and records where each routing slot's row went;
* stages 3 and 4 run locally on this rank's expert slice;
* combine: stage 5 (``ep_gemm_store``) stores the weighted output rows locally; ``ep_combine_push``
  sums, per token, the rows of this rank's experts and writes that ONE row (fp16 by default, or fp32)
  into the token owner's staging buffer over NVLink, one warp per row so the link carries full packets;
  ``ep_combine_reduce`` then sums each token's rows over the contributing ranks in rank order
  (deterministic).  NVLink carries one row per (token, rank) pair each way instead of one per
  routing slot.

Per layer the ranks exchange only two collectives: the routing all-gather (which also orders every
rank's token-buffer writes, and the end of its previous reduce, before any peer access) and a barrier
after the pushes (after which every rank's staging buffer holds all of its rows).  The device work goes
through a backend object; ``CudaBackend`` (the sm_100a library) is the product, and the CPU tests drive
the same host logic with a backend built on the oracle.
"""
from __future__ import annotations

import types

import torch
import torch.distributed as dist

import b200_ext

MAX_RANKS = b200_ext.MAX_RANKS


def expert_range(rank: int, world: int, n_experts: int):
    """Contiguous expert slice [e0, e1) of `rank`."""
    return rank * n_experts // world, (rank + 1) * n_experts // world


def balanced_placement(counts, world: int, tile_rows: int = 256):
    """Expert placement that balances the ranks' work, from per-expert routed-row counts measured on a
    calibration batch (experts' popularity is a property of the model's router, stable across batches).

    Every rank keeps E/world experts (the contiguous-range sizes of ``expert_range``); experts are taken
    heaviest first and given to the least-loaded rank with room, with cost = rows + tile_rows/2 per
    256-row M-tile (each tile also decodes the expert's weights once).  Returns the E global expert ids
    in rank order: rank r owns placement[e0:e1] with (e0, e1) = expert_range(r, world, E)."""
    counts = [int(c) for c in counts]
    E = len(counts)
    room = [expert_range(r, world, E)[1] - expert_range(r, world, E)[0] for r in range(world)]
    cost = [c + (tile_rows // 2) * ((c + tile_rows - 1) // tile_rows) for c in counts]
    load = [0] * world
    members = [[] for _ in range(world)]
    for e in sorted(range(E), key=lambda e: (-cost[e], e)):
        r = min((r for r in range(world) if len(members[r]) < room[r]), key=lambda r: (load[r], r))
        members[r].append(e)
        load[r] += cost[e]
    return [e for r in range(world) for e in sorted(members[r])]


def layer_take(layer, experts):
    """Copy of a stacked layer holding `experts` (global ids) in that order."""
    idx = torch.as_tensor(list(experts), dtype=torch.long, device=layer.w13_trellis.device)
    out = types.SimpleNamespace()
    for name in ("w13_trellis", "w13_suh", "w13_svh", "w2_trellis", "w2_suh", "w2_svh"):
        setattr(out, name, getattr(layer, name).index_select(0, idx).contiguous())
    out._exl3_intermediate_local = layer._exl3_intermediate_local
    return out


def layer_slice(layer, e0: int, e1: int):
    """View of a stacked layer restricted to experts [e0, e1) (same attribute names and layouts)."""
    out = types.SimpleNamespace()
    for name in ("w13_trellis", "w13_suh", "w13_svh", "w2_trellis", "w2_suh", "w2_svh"):
        setattr(out, name, getattr(layer, name)[e0:e1])
    out._exl3_intermediate_local = layer._exl3_intermediate_local
    return out


class _DeviceArray:
    """Zero-copy view of a raw device allocation (for torch.as_tensor)."""

    def __init__(self, addr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(addr), False),
                                         "version": 3, "strides": None}


def owner_rank(position: int, n_experts: int, world: int) -> int:
    """Rank owning expert position `position` (the inverse of ``expert_range``)."""
    r = 0
    while r + 1 < world and position >= (r + 1) * n_experts // world:
        r += 1
    return r


class CudaBackend:
    """The product backend: buffers from exl3_ep_alloc shared through CUDA IPC; stages from the library."""

    def __init__(self, group, rank: int, world: int, tokens_per_rank: int, hidden: int, topk: int,
                 device: torch.device, combine_dtype: torch.dtype = torch.float16):
        self.group, self.rank, self.world, self.device = group, rank, world, device
        self.tpr, self.topk, self.d = tokens_per_rank, topk, hidden
        self.combine_f16 = combine_dtype == torch.float16
        self._own = []
        self._opened = []
        x_addr = b200_ext.ep_alloc(tokens_per_rank * hidden * 2, device)
        self._own.append(x_addr)
        esz = 2 if self.combine_f16 else 4
        st_addr = b200_ext.ep_alloc(tokens_per_rank * world * hidden * esz, device)
        self._own.append(st_addr)
        self.x = torch.as_tensor(_DeviceArray(x_addr, (tokens_per_rank, hidden), "<f2"), device=device)
        self.staging = torch.as_tensor(_DeviceArray(st_addr, (tokens_per_rank * world, hidden),
                                                    "<f2" if self.combine_f16 else "<f4"), device=device)
        self.out = torch.empty(tokens_per_rank, hidden, dtype=torch.float32, device=device)
        # every routing slot's sorted row (written by stage 2 for this rank's slots, read by the push)
        self.slot_row = torch.empty(world * tokens_per_rank * topk, dtype=torch.int32, device=device)
        # remote token rows this rank needs, at their global token rows
        self.x_pulled = (torch.empty(world * tokens_per_rank, hidden, dtype=torch.float16, device=device)
                         if world > 1 else None)
        # exchange the IPC handles of both buffers (NCCL all-gather of 128 bytes per rank)
        mine = torch.frombuffer(bytearray(b200_ext.ep_ipc_handle(x_addr, device) +
                                          b200_ext.ep_ipc_handle(st_addr, device)), dtype=torch.uint8).to(device)
        allh = torch.empty(world, mine.numel(), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.cpu()
        self.x_addrs, self.staging_addrs = [], []
        h = b200_ext.IPC_HANDLE_BYTES
        for r in range(world):
            if r == rank:
                self.x_addrs.append(x_addr)
                self.staging_addrs.append(st_addr)
                continue
            row = bytes(allh[r].tolist())
            xa = b200_ext.ep_ipc_open(row[:h], device)
            self._opened.append(xa)
            oa = b200_ext.ep_ipc_open(row[h:], device)
            self._opened.append(oa)
            self.x_addrs.append(xa)
            self.staging_addrs.append(oa)
        # stage 2 reads this rank's tokens in place and every other rank's from the pulled copy
        row_bytes = tokens_per_rank * hidden * 2
        self.row_src = [x_addr if r == rank else self.x_pulled.data_ptr() + r * row_bytes for r in range(world)]
        # the pull runs on its own stream, beside the routing sort (it needs only the gathered routing)
        self.pull_stream = torch.cuda.Stream(device) if world > 1 else None
        self._pulled = None

    def all_gather(self, dst, src):
        dist.all_gather_into_tensor(dst, src, group=self.group)

    def publish(self):
        # nothing to move: peers read this rank's token buffer in place (the pull), ordered by the routing
        # all-gather that precedes this call on every rank
        pass

    def pull(self, ids_pos, e0, e1):
        if self.world > 1:
            self.pull_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.pull_stream):
                b200_ext.ep_pull_rows(self.x_addrs, self.rank, self.tpr, ids_pos, e0, e1, self.x_pulled)
            self._pulled = torch.cuda.Event()
            self._pulled.record(self.pull_stream)

    def _join_pull(self):
        if self._pulled is not None:
            torch.cuda.current_stream(self.device).wait_event(self._pulled)
            self._pulled = None

    def barrier(self):
        # a one-element all-reduce on the current stream orders every rank's pushes before any later
        # read of this rank's staging buffer, and this rank's pull before any peer rewrites its tokens
        self._join_pull()
        t = torch.ones(1, dtype=torch.int32, device=self.device)
        dist.all_reduce(t, group=self.group)

    def reduce(self, ids_pos, n_experts, T):
        b200_ext.ep_combine_reduce(self.staging, ids_pos[:T], n_experts, self.world, self.out[:T])

    def local_ids(self, ids_pos, e0, e1, out):
        # this rank's routing slots: expert positions in [e0, e1) -> local ids, every other slot unrouted
        torch.where((ids_pos >= e0) & (ids_pos < e1), ids_pos - e0, torch.full_like(ids_pos, -1), out=out)

    def route_sort(self, ids, w, n_experts, bufs):
        b200_ext.route_sort(ids, w, n_experts, bufs.token_sorted, bufs.weight_sorted, bufs.expert_of_row,
                            bufs.counts, bufs.expert_row0, bufs.block_expert, bufs.block_row0, bufs.meta,
                            scratch=bufs.scratch)

    def row_had(self, h13, slot_sorted, expert_of_row, rows_dev, suh):
        self._join_pull()
        b200_ext.ep_row_had(self.row_src, self.tpr, self.topk, h13, slot_sorted, expert_of_row, 0, suh,
                            slot_row=self.slot_row, rows_dev=rows_dev)

    def gemm_gate_up(self, h13, layer, counts, row0, gu):
        b200_ext.grouped_gemm(h13, layer.w13_trellis[:, 0], layer.w13_trellis[:, 1], layer.w13_svh[:, 0],
                              layer.w13_svh[:, 1], None, None, counts, row0, None, None, gu, 0)

    def act_had(self, gu, act, expert_of_row, rows_dev, suh, limit):
        b200_ext.ep_act_had(gu, act, expert_of_row, 0, suh, limit, rows_dev=rows_dev)

    def gemm_down(self, act, layer, counts, row0, weight_sorted, y):
        b200_ext.ep_gemm_store(act, layer.w2_trellis, layer.w2_svh, counts, row0, weight_sorted, y)

    def push(self, y, ids_pos, e0, e1):
        b200_ext.ep_combine_push(y, ids_pos, e0, e1, self.slot_row, self.staging_addrs, self.rank, self.tpr,
                                 self.combine_f16)

    def close(self):
        torch.cuda.synchronize(self.device)
        for a in self._opened:
            b200_ext.ep_ipc_close(a, self.device)
        self._opened = []
        self.x = self.staging = self.out = self.x_pulled = self.slot_row = None
        for a in self._own:
            b200_ext.ep_free(a, self.device)
        self._own = []


class ExpertParallel:
    """Per-rank expert-parallel MoE prefill.

    ``prefill(x, ids, weights, layer_local, limit)``: x [T, d] (T <= tokens_per_rank) this rank's tokens,
    ids [T, topk] global expert ids, weights [T, topk]; layer_local holds this rank's experts.  Without
    ``placement`` rank r owns the contiguous experts [e0, e1) = ``expert_range(r, N, E)`` (``layer_slice``);
    with ``placement`` (a permutation of the E expert ids, e.g. from ``balanced_placement``) it owns
    ``placement[e0:e1]`` in that order (``layer_take``): the ids are mapped to placement positions before
    the sort, so every rank's rows stay one contiguous slice.  Returns the fp32 [T, d] output of
    this rank's tokens: a view of the shared output buffer, valid until the next ``prefill`` (pass
    ``copy=True`` for a fresh tensor).  Every rank must call ``prefill`` the same number of times.

    ``combine_dtype``: the type of the per-(token, rank) partial sums sent back to the token owners.
    fp16 (default) halves the NVLink bytes of the combine and rounds each partial sum once (about 2.8e-4
    relative, the same order as the fp16 cast the serving path applies to the layer output); fp32
    matches the single-GPU pipeline up to the fp32 summation order.
    """

    def __init__(self, tokens_per_rank: int, hidden: int, n_experts: int, topk: int, intermediate: int,
                 group=None, device: torch.device | None = None, backend=None, placement=None,
                 combine_dtype: torch.dtype = torch.float16):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 1 <= self.world <= MAX_RANKS:
            raise RuntimeError(f"expert parallelism supports 1..{MAX_RANKS} ranks")
        if n_experts < self.world:
            raise RuntimeError("fewer experts than ranks")
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.tpr, self.d, self.E, self.topk, self.I = int(tokens_per_rank), int(hidden), int(n_experts), int(topk), \
            int(intermediate)
        self.e0, self.e1 = expert_range(self.rank, self.world, self.E)
        self.position = None
        if placement is not None:
            placement = [int(e) for e in placement]
            if sorted(placement) != list(range(self.E)):
                raise RuntimeError("placement must be a permutation of the expert ids")
            pos = torch.empty(self.E, dtype=torch.int64)
            pos[torch.tensor(placement)] = torch.arange(self.E)
            self.position = pos.to(self.device)
            self.experts = placement[self.e0:self.e1]
        else:
            self.experts = list(range(self.e0, self.e1))
        if combine_dtype not in (torch.float16, torch.float32):
            raise RuntimeError("combine_dtype must be torch.float16 or torch.float32")
        self.combine_dtype = combine_dtype
        self.be = backend if backend is not None else CudaBackend(group, self.rank, self.world, self.tpr, self.d,
                                                                  self.topk, self.device, combine_dtype)
        dev = self.device
        Rg = self.world * self.tpr * self.topk
        b = types.SimpleNamespace()
        b.ids_pad = torch.full((self.tpr, self.topk), -1, dtype=torch.int64, device=dev)
        b.w_pad = torch.zeros(self.tpr, self.topk, dtype=torch.float32, device=dev)
        b.ids_g = torch.empty(self.world * self.tpr, self.topk, dtype=torch.int64, device=dev)
        b.w_g = torch.empty(self.world * self.tpr, self.topk, dtype=torch.float32, device=dev)
        El = self.e1 - self.e0
        b.ids_loc = torch.empty(self.world * self.tpr, self.topk, dtype=torch.int64, device=dev)
        b.token_sorted = torch.empty(Rg, dtype=torch.int64, device=dev)
        b.weight_sorted = torch.empty(Rg, dtype=torch.float16, device=dev)
        b.expert_of_row = torch.empty(Rg, dtype=torch.int32, device=dev)
        b.counts = torch.empty(El, dtype=torch.int32, device=dev)
        b.expert_row0 = torch.empty(El, dtype=torch.int32, device=dev)
        max_blocks = Rg // 128 + El
        b.block_expert = torch.empty(max_blocks, dtype=torch.int32, device=dev)
        b.block_row0 = torch.empty(max_blocks, dtype=torch.int32, device=dev)
        b.meta = torch.zeros(2, dtype=torch.int32, device=dev)
        b.scratch = (torch.empty(b200_ext.route_sort_scratch_elems(Rg, El), dtype=torch.int32, device=dev)
                     if dev.type == "cuda" else None)
        self.bufs = b
        # Stage workspace for the worst case, every routing slot of every rank on this rank's experts
        # (Rg rows: 2.2 GB per 65536 rows at d = 4096, f = 1536), so no host read of the row count is needed.
        self._h13 = torch.empty(Rg, self.d, dtype=torch.float16, device=dev)
        self._gu = torch.empty(Rg, 2 * self.I, dtype=torch.float16, device=dev)
        self._act = torch.empty(Rg, self.I, dtype=torch.float16, device=dev)
        self._y = torch.empty(Rg, self.d, dtype=torch.float32, device=dev)

    @property
    def x_buffer(self) -> torch.Tensor:
        """This rank's token buffer [tokens_per_rank, d] fp16: write tokens here to skip the copy."""
        return self.be.x

    @property
    def last_rows(self) -> int:
        """Routed rows this rank processed in the last prefill (reads the device count: synchronises)."""
        return int(self.bufs.meta[1].item())

    def prefill(self, x, ids, weights, layer_local, limit: float, copy: bool = False, stage_hook=None):
        hook = stage_hook if stage_hook is not None else (lambda name: None)
        b, be = self.bufs, self.be
        T = int(x.shape[0])
        if T > self.tpr:
            raise RuntimeError(f"{T} tokens exceed tokens_per_rank={self.tpr}")
        if tuple(ids.shape) != (T, self.topk) or tuple(weights.shape) != (T, self.topk):
            raise RuntimeError("ids / weights must be [T, topk]")
        if int(layer_local.w13_trellis.shape[0]) != self.e1 - self.e0:
            raise RuntimeError("layer_local must hold this rank's experts")
        hook("dispatch_setup")
        if x.data_ptr() != be.x.data_ptr():
            be.x[:T].copy_(x)
        if self.position is None:
            b.ids_pad[:T].copy_(ids)
        else:
            # expert id -> placement position (ids outside [0, E) stay unrouted)
            idl = ids.to(device=self.device, dtype=torch.int64)
            valid = (idl >= 0) & (idl < self.E)
            b.ids_pad[:T].copy_(torch.where(valid, self.position[idl.clamp(0, self.E - 1)], -1))
        b.ids_pad[T:].fill_(-1)
        b.w_pad[:T].copy_(weights)
        # the all-gathers follow this rank's token-buffer copy and its previous reduce on its stream, so when
        # they complete on any rank, every rank's token buffer is ready for peer reads and its staging
        # buffer free for the pushes
        be.all_gather(b.ids_g, b.ids_pad)
        be.all_gather(b.w_g, b.w_pad)
        be.publish()
        hook("pull")
        be.pull(b.ids_g, self.e0, self.e1)
        hook("route_sort")
        # one list of routing slots, only this rank's experts routed (local ids 0 .. e1 - e0 - 1); its rows
        # come first, their number stays on the device (meta[1])
        be.local_ids(b.ids_g, self.e0, self.e1, b.ids_loc)
        be.route_sort(b.ids_loc.view(-1, 1), b.w_g.view(-1, 1), self.e1 - self.e0, b)
        rows_dev = b.meta[1:]
        hook("row_had")
        be.row_had(self._h13, b.token_sorted, b.expert_of_row, rows_dev, layer_local.w13_suh[:, 0])
        hook("gemm_gate_up")
        be.gemm_gate_up(self._h13, layer_local, b.counts, b.expert_row0, self._gu)
        hook("act_had")
        be.act_had(self._gu, self._act, b.expert_of_row, rows_dev, layer_local.w2_suh, limit)
        hook("gemm_down")
        be.gemm_down(self._act, layer_local, b.counts, b.expert_row0, b.weight_sorted, self._y)
        hook("combine_push")
        be.push(self._y, b.ids_g, self.e0, self.e1)        # tokens without a route here are skipped
        hook("combine_barrier")
        be.barrier()
        hook("combine_reduce")
        be.reduce(b.ids_pad, self.E, T)
        hook("end")
        out = be.out[:T]
        return out.clone() if copy else out

    def close(self):
        self.be.close()
