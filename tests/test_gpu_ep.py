"""GPU: the expert-parallel path (ep.ExpertParallel with the CUDA backend), through the C ABI.

* one rank (NCCL world of 1): the stage-2 gather, the weighted-row GEMM, the push and the reduce with this
  GPU's own buffers must reproduce grouped_prefill on the same inputs;
* two ranks (skipped with fewer than 2 GPUs): rows cross NVLink in both directions (pull and push); every
  rank's output must equal grouped_prefill over all tokens with all experts, computed on GPU 0.

Tolerances: fp32 combine rel-L2 < 1e-5 (only the fp32 summation order differs); fp16 combine < 1e-3, the
layer bar (one fp16 rounding per (token, rank) partial sum, about 3e-4).

Every rank runs in its own process with a 60 s process-group timeout."""
import os
import tempfile
import sys
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
PATHS = [os.path.join(REPO, "glm53-exl3-prefill_b200"), os.path.join(REPO, "oracle")]


def _rendezvous_file():
    """A fresh file for a file:// rendezvous (no TCP port that a previous run may still hold)."""
    fd, path = tempfile.mkstemp(prefix="exl3_ep_rdzv_")
    os.close(fd)
    os.unlink(path)
    return path


def _worker(rank, world, rdzv, cfg):
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import b200_ext
    import ep
    import exl3_grouped_runtime as rt
    import synth
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method="file://" + rdzv, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        E, d, f, k = cfg["E"], cfg["d"], cfg["f"], cfg["k"]
        tokens = cfg["tokens"]
        tpr = max(tokens)
        T_all = sum(tokens)
        layer = synth.make_layer(E, d, f, seed=11, device=dev, sv_scale=0.05)
        x_all = synth.make_x(T_all, d, seed=12, device=dev)
        ids_all, w_all = synth.routing(cfg["routing"], T_all, E, k, seed=13, device=dev)
        off = sum(tokens[:rank])
        mine = slice(off, off + tokens[rank])
        e0, e1 = ep.expert_range(rank, world, E)
        f16 = cfg.get("combine", "fp16") == "fp16"
        placement = None
        if cfg.get("placement") == "random":
            placement = torch.randperm(E, generator=torch.Generator().manual_seed(3)).tolist()
        eng = ep.ExpertParallel(tpr, d, E, k, f, device=dev, placement=placement,
                                combine_dtype=torch.float16 if f16 else torch.float32)
        lay = ep.layer_slice(layer, e0, e1) if placement is None else ep.layer_take(layer, placement[e0:e1])
        outs = []
        for _ in range(2):
            outs.append(eng.prefill(x_all[mine], ids_all[mine], w_all[mine], lay, 7.0, copy=True))
        torch.cuda.synchronize(dev)
        assert b200_ext.read_status(dev) == 0
        got = torch.zeros(tpr, d, dtype=torch.float32, device=dev)
        got[:tokens[rank]] = outs[1]
        allgot = torch.empty(world * tpr, d, dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(allgot, got)
        allgot = allgot.view(world, tpr, d)
        if rank == 0:
            want = rt.grouped_prefill(x_all, ids_all, w_all, layer, 7.0)
            for r in range(world):
                o = sum(tokens[:r])
                g = allgot[r, :tokens[r]]
                w = want[o:o + tokens[r]]
                rel = float((g - w).norm() / w.norm())
                assert rel < (1e-3 if f16 else 1e-5), (r, rel)
            # the EP combine has no atomics: a repeated call gives the same bits
            assert torch.equal(outs[0], outs[1])
        eng.close()
    finally:
        dist.destroy_process_group()


def _run(world, cfg):
    mp.spawn(_worker, args=(world, _rendezvous_file(), cfg), nprocs=world, join=True)


def test_ep_single_rank_matches_grouped_prefill(cuda_device):
    _run(1, dict(E=32, d=1024, f=512, k=4, tokens=[1000], routing="zipf", combine="fp32"))
    _run(1, dict(E=32, d=1024, f=512, k=4, tokens=[1000], routing="zipf", combine="fp16"))


def test_ep_single_rank_config1_shapes(cuda_device):
    _run(1, dict(E=288, d=4096, f=1536, k=8, tokens=[2048], routing="zipf"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_ranks_match_grouped_prefill(cuda_device):
    _run(2, dict(E=32, d=1024, f=512, k=4, tokens=[700, 613], routing="zipf", combine="fp32"))
    _run(2, dict(E=32, d=1024, f=512, k=4, tokens=[700, 613], routing="uniform", combine="fp16",
                 placement="random"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_ranks_config1_shapes(cuda_device):
    _run(2, dict(E=288, d=4096, f=1536, k=8, tokens=[2048, 2048], routing="zipf"))
