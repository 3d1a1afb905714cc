#!/usr/bin/env python3
"""Benchmark of the routed-expert EXL3 MoE prefill layer on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--tokens T] [--routing zipf|uniform]

A step is one MoE layer (all five stages) over one chunk of synthetic tokens: BASELINE.json config 1 by
default (E=288, d=4096, f=1536, top-8, T=8192, Zipf(1.1) routing).  `value` is tokens/s with the inputs
resident in HBM; `e2e` is the same metric through the public call (the installed apply_exl3_experts)
with host buffers, the H2D copies of x / ids / weights and the D2H copy of the output inside the timed
region.  `roofline` covers the dominant kernel (the gate|up grouped GEMM), timed with CUDA events on
its own stream inside the timed region, against the measured burst bf16 peak.  `cpu_baseline` times the
reference per-expert loop (the oracle's port of harness/proto_fp8.py:123-134 with decoded fp32 weights,
built once as the reference builds them) over the whole layer on this host's cores.  The N=1 line also
carries `chunk_sweep` (configs 2 and 3: per-stage ms at 256..8192 tokens, Zipf and uniform routing) and
`small_batch_ms` (1 / 8 / 32-token calls through the installed entry point with
EXL3_GROUPED_SMALL_BATCH=1); --no-extra skips them.

With N > 1 (torchrun, one rank per GPU) the layer runs expert-parallel (glm53-exl3-prefill_b200/ep.py):
each rank owns 288/N experts and T tokens (weak scaling: N*T tokens per step; at N=4 this is config 4's
32768-token chunk); each remote token row a GPU needs is pulled once over NVLink, and one partial-sum
row per (token, GPU) is pushed back to the token's owner (fp16 by default, --combine fp32).  Timed as
the max over ranks.

--workload moe-block / glm-block / dense-mlp (1 GPU) time the routed experts plus the shared expert, the
same from hidden states through the router front-end, or a dense SwiGLU MLP, on the same kernels;
--graph replays the layer from a CUDA graph (the small-batch path, for decode-sized --tokens).  These are
extra lines; the headline is the default workload.

--impl reference times the reference's own algorithm on the host CPU: the per-expert loop of the
reference (restated in oracle/, because the reference's CUDA path needs exllamav3 and sm_121a and the
overlay's loop is not available) over the whole layer per step, all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "glm53-exl3-prefill_b200")
ORACLE = os.path.join(REPO, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "MoE-layer prefill tokens/s (ms/layer) at 1K-8K chunk, 1/2/4/8 B200, % roofline"
UNIT = "tokens/s"
E_, D_, F_, K_ = 288, 4096, 1536, 8
LIMIT = 7.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=8192, help="tokens per GPU (weak scaling)")
    ap.add_argument("--total-tokens", type=int, default=0,
                    help="strong scaling: this many tokens per step in all, split evenly over the GPUs "
                         "(32768 = BASELINE.json config 4); overrides --tokens")
    ap.add_argument("--routing", default="zipf", choices=["zipf", "uniform"])
    ap.add_argument("--experts", type=int, default=E_, help="routed experts (288 = config 1; fewer for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--deterministic", action="store_true",
                    help="down stage as slot rows + a fixed-order combine (bit-repeatable) instead of fp32 atomics")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the chunk sweep (configs 2-3) and small-batch latencies added to the N=1 line")
    ap.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                    help="expert placement with N > 1 (balanced: fitted on a calibration batch)")
    ap.add_argument("--workload", default="moe", choices=["moe", "moe-block", "glm-block", "dense-mlp"],
                    help="1 GPU: moe = routed experts (the headline); moe-block = routed + shared expert; "
                         "glm-block = router front-end + routed + shared expert from hidden states; "
                         "dense-mlp = a dense SwiGLU MLP (d=4096, f=--dense-inter) on the same kernels")
    ap.add_argument("--dense-inter", type=int, default=12288, help="intermediate size of --workload dense-mlp")
    ap.add_argument("--graph", action="store_true",
                    help="1 GPU, --workload moe: replay the layer from a CUDA graph (the small-batch path)")
    ap.add_argument("--combine", default="fp16", choices=["fp16", "fp32"],
                    help="with N > 1: type of the per-(token, rank) partial sums sent back to the token owners")
    return ap.parse_args()


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm=float(d["hbm_gbs"]), tflops=float(d["bf16_tflops"]),
                    tflops_sustained=float(d["bf16_tflops_sustained"]), source="measured")
    return dict(hbm=6650.0, tflops=1590.0, tflops_sustained=1400.0, source="fallback")


GEMM_SOURCES = ("csrc/trellis_gemm.cu", "csrc/trellis_thin.cu", "csrc/trellis_common.cuh", "csrc/common.cuh")


def gemm_sources_sha16() -> str:
    """Hash of the trellis GEMM's sources, recorded beside the DRAM traffic in its ncu summary."""
    import hashlib
    h = hashlib.sha256()
    for rel in GEMM_SOURCES:
        with open(os.path.join(PKG, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def profiled_traffic():
    """(dram bytes of the gate|up GEMM stage at config 1, note) from the committed ncu summary: the sum
    over the stage's launches (two-block and thin kernels).  The figure counts only if the summary was
    captured on the current GEMM sources (same hash)."""
    p = os.path.join(REPO, "profiles", "trellis_gemm_gate_up_cfg1.md")
    if not os.path.exists(p):
        return None, "no ncu summary"
    vals = {}
    for line in open(p):
        for key in ("dram_bytes_gate_up_stage_cfg1:", "kernel_sources_sha16:"):
            if line.strip().startswith(key):
                vals[key] = line.split(":", 1)[1].strip().split()[0]
    sha = gemm_sources_sha16()
    if vals.get("kernel_sources_sha16:") != sha:
        return None, f"profiles/trellis_gemm_gate_up_cfg1.md was captured on other GEMM sources (now {sha})"
    try:
        return (float(vals["dram_bytes_gate_up_stage_cfg1:"]),
                f"ncu dram__bytes_read+write of the stage's launches, sources {sha}")
    except (KeyError, ValueError):
        return None, "no traffic line in the ncu summary"


# ------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=lambda: self.lines.extend(iter(self.proc.stdout.readline, "")), daemon=True)
        self.thread.start()

    def wait_first(self, timeout_s: float = 5.0) -> bool:
        """Block until the sampler has produced a line (nvidia-smi can take a second to start)."""
        t_end = time.time() + timeout_s
        while self.proc is not None and not self.lines and time.time() < t_end:
            time.sleep(0.05)
        return bool(self.lines)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------ CPU baseline
class CpuReferenceLayer:
    """The reference per-expert loop (harness/proto_fp8.py:123-134, ``ref_fp16``) on the host cores.

    As in the reference (which builds every expert's real-domain weights once, ``Wfull``,
    harness/proto_fp8.py:106-117), the set-up decodes each routed expert's packed weights once (the
    oracle's C trellis decode, threaded) and applies the exllamav3 convention
    W = diag(suh) H W' H diag(svh) (:66-76); ``step`` then runs the loop itself: per expert, gather its
    tokens, gate and up matmuls, clamped SwiGLU, down matmul, route-weighted index_add.  The host has no
    fast fp16 matmul, so the weights (the fp16 values) and activations are held in fp32."""

    def __init__(self, layer, experts, threads: int):
        import oracle
        torch.set_num_threads(threads)
        self.threads = threads
        H = torch.from_numpy(oracle.had128_matrix())
        t0 = time.perf_counter()
        self.decode_s = 0.0
        self.w = {}
        for e in experts:
            t1 = time.perf_counter()
            pk = (layer.w13_trellis[e, 0].cpu().numpy(), layer.w13_trellis[e, 1].cpu().numpy(),
                  layer.w2_trellis[e].cpu().numpy())
            dec = [torch.from_numpy(oracle.reconstruct(p, np.float32)) for p in pk]
            self.decode_s += time.perf_counter() - t1
            sv = ((layer.w13_suh[e, 0], layer.w13_svh[e, 0]), (layer.w13_suh[e, 1], layer.w13_svh[e, 1]),
                  (layer.w2_suh[e], layer.w2_svh[e]))
            self.w[e] = tuple(self._full(H, wq, su, svv) for wq, (su, svv) in zip(dec, sv))
        self.setup_s = time.perf_counter() - t0

    @staticmethod
    def _full(H, wq, suh, svh):
        K, N = wq.shape
        t = (H @ wq.view(-1, 128, N)).view(K, N) * suh.cpu().float()[:, None]
        return ((t.view(K, -1, 128) @ H).view(K, N) * svh.cpu().float()[None, :]).contiguous()

    def step(self, xf, ids_np, w_cpu):
        out = torch.zeros(xf.shape[0], xf.shape[1])
        for e, (g, u, dn) in self.w.items():
            tok, kpos = np.nonzero(ids_np == e)
            if tok.size == 0:
                continue
            tok_t = torch.from_numpy(tok)
            h = xf.index_select(0, tok_t)
            gate, up = h @ g, h @ u
            act = torch.nn.functional.silu(gate.clamp(max=LIMIT)) * up.clamp(-LIMIT, LIMIT)
            out.index_add_(0, tok_t, (act @ dn) * w_cpu[tok_t, torch.from_numpy(kpos)][:, None])
        return out


def cpu_host():
    model = ""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return f"{os.cpu_count()} host cpus ({model or 'unknown model'})"


def cpu_baseline(layer, x16, ids, w, threads: int, steps: int = 1):
    """The reference loop timed over the WHOLE layer (every routed expert, all tokens) on this host's
    cores, after the one-time weight set-up; value = tokens / median step time."""
    ids_np = ids.cpu().numpy()
    E = layer.w13_trellis.shape[0]
    counts = np.bincount(ids_np.reshape(-1)[ids_np.reshape(-1) >= 0], minlength=E)
    ref = CpuReferenceLayer(layer, [int(e) for e in np.nonzero(counts)[0]], threads)
    xf = x16.cpu().float()
    w_cpu = w.cpu().float()
    times = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        ref.step(xf, ids_np, w_cpu)
        times.append(time.perf_counter() - t0)
    t_layer = statistics.median(times)
    T = xf.shape[0]
    return {"value": T / t_layer, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"the whole layer ({len(ref.w)} routed experts, {int(counts.sum())} routed rows, {T} tokens), "
                      f"{len(times)} timed step(s) of the per-expert loop after a one-time set-up of "
                      f"{ref.setup_s:.1f} s (trellis decode {ref.decode_s:.1f} s, not timed, as the reference "
                      f"builds its weights once); {cpu_host()}",
            "step_s": times, "setup_s": ref.setup_s}


# ------------------------------------------------------------------------------------ ours
def make_inputs(dev, T, routing, seed=100, E=E_):
    import synth
    layer = synth.make_layer(E, D_, F_, seed=seed, device=dev)
    x = synth.make_x(T, D_, seed=seed + 1, device=dev)
    ids, w = synth.routing(routing, T, E, K_, seed=seed + 2, device=dev)
    return layer, x, ids, w


def stage_times(run, x, ids, w, stage_names, stream, warmup=3, steps=5):
    """Median per-stage ms of `run(x, ids, w, hook)` (CUDA events between stage launches) and layer ms."""
    for _ in range(warmup):
        run(x, ids, w, None)
    per = []
    for _ in range(steps):
        evs = []

        def hook(name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            evs.append((name, ev))
        run(x, ids, w, hook)
        per.append(evs)
    torch.cuda.synchronize()
    st = {}
    for evs in per:
        for (n, a), (_, b) in zip(evs[:-1], evs[1:]):
            st.setdefault(n, []).append(a.elapsed_time(b))
    med = {n: statistics.median(v) for n, v in st.items()}
    return med, statistics.median([evs[0][1].elapsed_time(evs[-1][1]) for evs in per])


def chunk_sweep(layer, dev, stream, peak_tflops):
    """BASELINE.json configs 2 and 3 on the config-1 layer: T = 1K..8K under Zipf(1.1) and uniform routing,
    and the thin-expert case (uniform, T = 256 / 512).  Per-stage ms, layer ms, and each GEMM's achieved
    TFLOP/s and fraction of the burst bf16 peak (tensor-pipe % comes from ncu, not from this run)."""
    import exl3_grouped_runtime as rt
    import synth
    names = ["route_sort", "row_had", "gemm_gate_up", "act_had", "gemm_down", "combine", "end"]
    res = {}
    for routing, toks in (("zipf", (1024, 2048, 4096, 8192)), ("uniform", (256, 512, 1024, 2048, 4096, 8192))):
        for T in toks:
            x = synth.make_x(T, D_, seed=101, device=dev)
            ids, w = synth.routing(routing, T, E_, K_, seed=102, device=dev)
            st, layer_ms = stage_times(lambda xx, ii, ww, hook: rt.grouped_prefill(xx, ii, ww, layer, LIMIT,
                                                                                    stage_hook=hook),
                                       x, ids, w, names, stream)
            R = T * K_
            fl_gu, fl_dn = 4.0 * R * D_ * F_, 2.0 * R * D_ * F_
            tf_gu = fl_gu / (st["gemm_gate_up"] * 1e-3) / 1e12
            tf_dn = fl_dn / (st["gemm_down"] * 1e-3) / 1e12
            res[f"{routing}_{T}"] = {"layer_ms": layer_ms, "tokens_per_s": T / (layer_ms * 1e-3),
                                     "stages_ms": st, "gemm_gate_up_tflops": tf_gu,
                                     "gemm_gate_up_frac": tf_gu / peak_tflops, "gemm_down_tflops": tf_dn,
                                     "gemm_down_frac": tf_dn / peak_tflops}
    return res


def small_batch_latency(layer, dev, stream, cap=64, tokens=(1, 8, 32), reps=20):
    """Decode-sized calls through the installed apply_exl3_experts with EXL3_GROUPED_SMALL_BATCH=1 (the
    small-batch path a serving engine reaches for tokens <= the fused kernel's row cap): median ms per call,
    device-timed, inputs already on the GPU."""
    import exl3_grouped_runtime as rt
    import synth
    ov = type(sys)("exl3_overlay_stub_small")
    ov.SWIGLU_LIMIT_DEFAULT = LIMIT
    ov.apply_exl3_experts = lambda *a, **k: (_ for _ in ()).throw(RuntimeError("original path not expected"))
    old = os.environ.get("EXL3_GROUPED_SMALL_BATCH")
    os.environ["EXL3_GROUPED_SMALL_BATCH"] = "1"
    try:
        rt.install(ov)
    finally:
        if old is None:
            os.environ.pop("EXL3_GROUPED_SMALL_BATCH")
        else:
            os.environ["EXL3_GROUPED_SMALL_BATCH"] = old
    layer._exl3_fused_temps = [torch.zeros(1, cap, device=dev)]
    out = {}
    for T in tokens:
        x = synth.make_x(T, D_, seed=500 + T, device=dev)
        ids, w = synth.routing("zipf", T, E_, K_, seed=600 + T, device=dev)
        for _ in range(3):
            ov.apply_exl3_experts(x, ids, w, layer, limit=LIMIT)
        torch.cuda.synchronize()
        ms = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ov.apply_exl3_experts(x, ids, w, layer, limit=LIMIT)
            b.record(stream)
            b.synchronize()
            ms.append(a.elapsed_time(b))
        out[str(T)] = statistics.median(ms)
    assert layer._exl3_last_apply == "grouped-small-batch"
    layer._exl3_fused_temps = None
    return out


def run_ours(args, rank, world, local_rank):
    import exl3_grouped_runtime as rt
    import synth
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T = args.tokens
    E = args.experts
    stream = torch.cuda.current_stream(dev)
    rt._load_ext()
    f_gemm = F_                                     # intermediate size of the timed gate|up GEMM
    if world == 1 and args.workload == "dense-mlp":
        import exl3_dense
        f_gemm = args.dense_inter
        layer = synth.make_layer(1, D_, f_gemm, seed=100, device=dev)
        x = synth.make_x(T, D_, seed=101, device=dev)
        ids = torch.zeros(T, 1, dtype=torch.int64, device=dev)
        w = torch.ones(T, 1, dtype=torch.float16, device=dev)
        stage_names = ["route_sort", "row_had", "gemm_gate_up", "act_had", "gemm_down", "combine", "end"]

        def run_layer(xx, ii, ww, hook=None):
            return exl3_dense.dense_mlp_prefill(xx, layer, LIMIT, stage_hook=hook)

        def gate_up_rows():
            return T
    elif world == 1 and args.workload == "glm-block":
        import exl3_router
        layer, x, ids, w = make_inputs(dev, T, args.routing, seed=100, E=E)
        shared = synth.make_layer(1, D_, F_, seed=200, device=dev)
        g = torch.Generator(device=dev).manual_seed(300)
        wr = (torch.randn(E, D_, generator=g, device=dev) * (2.0 / D_ ** 0.5)).half()
        # a skewed router: e_score_correction_bias tilted toward Zipf(1.1)-popular experts
        pop = torch.arange(1, E + 1, device=dev, dtype=torch.float32).pow(-1.1)
        pop = pop[torch.randperm(E, generator=g, device=dev)]
        bias = 0.05 * torch.log(pop / pop.max())
        router = exl3_router.NoauxTcRouter(wr, bias, topk=K_, norm=True, scale=2.5)
        stage_names = ["route_front", "row_had", "gemm_gate_up", "act_had", "gemm_down", "combine"]
        stage_names = stage_names + ["shared_" + n for n in ["route_sort"] + stage_names[1:]] + ["end"]

        def run_layer(xx, ii, ww, hook=None):
            return exl3_router.moe_prefill_from_hidden(xx, router, layer, LIMIT, shared=shared, stage_hook=hook)

        def gate_up_rows():
            return T * K_
    elif world == 1:
        layer, x, ids, w = make_inputs(dev, T, args.routing, seed=100, E=E)
        stage_names = ["route_sort", "row_had", "gemm_gate_up", "act_had", "gemm_down", "combine", "end"]
        shared = None
        if args.workload == "moe-block":
            import exl3_dense
            shared = synth.make_layer(1, D_, F_, seed=200, device=dev)
            stage_names = stage_names[:-1] + ["shared_" + n for n in stage_names[:-1]] + ["end"]

        graphed = None
        if args.graph and args.workload == "moe":
            import exl3_decode
            graphed = exl3_decode.GraphedPrefill(layer, LIMIT, K_, max_tokens=T, device=dev)
            stage_names = ["layer", "end"]           # one replay: no per-stage events inside the graph

        def run_layer(xx, ii, ww, hook=None):
            if graphed is not None:
                if hook:
                    hook("layer")
                o = graphed(xx, ii, ww)
                if hook:
                    hook("end")
                return o
            if shared is not None:
                return exl3_dense.moe_block_prefill(xx, ii, ww, layer, shared, LIMIT, stage_hook=hook)
            return rt.grouped_prefill(xx, ii, ww, layer, LIMIT, stage_hook=hook, deterministic=args.deterministic)

        def gate_up_rows():
            return T * K_
    else:
        import ep
        e0, e1 = ep.expert_range(rank, world, E)
        layer = synth.make_layer(e1 - e0, D_, F_, seed=100 + 1000 * rank, device=dev)   # this rank's experts
        x = synth.make_x(T, D_, seed=101 + rank, device=dev)
        # one routing for the whole chunk of world*T tokens (one expert-popularity order, as one router
        # produces), sharded by token: rank r routes tokens [r*T, (r+1)*T)
        ids_all, w_all = synth.routing(args.routing, world * T, E, K_, seed=102, device=dev, popularity_seed=102)
        ids, w = ids_all[rank * T:(rank + 1) * T].contiguous(), w_all[rank * T:(rank + 1) * T].contiguous()
        del ids_all, w_all
        placement = None
        if args.placement == "balanced":
            # placement from a separate calibration batch of the same router (never the timed batch)
            cal, _ = synth.routing(args.routing, world * T, E, K_, seed=7, device=dev, popularity_seed=102)
            placement = ep.balanced_placement(torch.bincount(cal.flatten(), minlength=E).tolist(), world)
        eng = ep.ExpertParallel(T, D_, E, K_, F_, device=dev, placement=placement,
                                combine_dtype=torch.float16 if args.combine == "fp16" else torch.float32)
        eng.x_buffer.copy_(x)                      # this rank's tokens live in the peer-readable buffer
        x = eng.x_buffer
        stage_names = ["dispatch_setup", "pull", "route_sort", "row_had", "gemm_gate_up", "act_had", "gemm_down",
                       "combine_push", "combine_barrier", "combine_reduce", "end"]

        def run_layer(xx, ii, ww, hook=None):
            return eng.prefill(xx, ii, ww, layer, LIMIT, stage_hook=hook)

        def gate_up_rows():
            return eng.last_rows

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def step(events=None):
        hook = None
        if events is not None:
            def hook(name):
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(stream)
                events.append((name, ev))
        return run_layer(x, ids, w, hook)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # ---- device-resident timed region
    # Clock samples (rank 0's GPU, every 200 ms) must come from the load being timed: wait for the sampler's
    # first line, then keep the GPU busy with the same steps (the same count on every rank, since the
    # expert-parallel step holds collectives) for ~0.25 s before the timed region, long enough for a
    # sample under load and short of the seconds-long load that brings the 1 kW power cap in, and stop
    # the sampler right after.
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks is not None:
        clocks.start()
        clocks.wait_first()
    t_pre = time.perf_counter()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    per_step_s = (time.perf_counter() - t_pre) / max(1, args.warmup)
    n_pre = torch.tensor([min(100, max(3, int(0.25 / max(per_step_s, 1e-4))))], device=dev)
    if world > 1:
        torch.distributed.all_reduce(n_pre, op=torch.distributed.ReduceOp.MIN)
    for _ in range(int(n_pre.item())):
        step()
    per_step_events = [[] for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(per_step_events[i])
    t1.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop() if clocks is not None else None
    barrier()
    elapsed_ms = t0.elapsed_time(t1)
    rows_gate_up = gate_up_rows()
    if world > 1:
        tt = torch.tensor([elapsed_ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
    stages = {n: [] for n in stage_names[:-1]}
    for evs in per_step_events:
        for (n, a), (_, b) in zip(evs[:-1], evs[1:]):
            stages.setdefault(n, []).append(a.elapsed_time(b))
    stage_ms = {n: statistics.mean(v) for n, v in stages.items() if v}

    # ---- end to end through the public call with host buffers
    x_h = x[:T].cpu().pin_memory()
    ids_h = ids.cpu().pin_memory()
    w_h = w.cpu().pin_memory()
    out_h = torch.empty(T, D_, dtype=torch.float16).pin_memory()
    if world == 1 and (args.workload != "moe" or args.graph):
        e2e_path = f"{args.workload} call with pinned host x in, fp16 out to host (copies overlapped as below)"

        def public_call(xd, idd, wd):
            return run_layer(xd, idd, wd).to(torch.float16)
    elif world == 1:
        ov = type(sys)("exl3_overlay_stub")
        ov.SWIGLU_LIMIT_DEFAULT = LIMIT
        ov.apply_exl3_experts = lambda *a, **k: (_ for _ in ()).throw(RuntimeError("decode path not expected"))
        rt.install(ov)
        layer._exl3_fused_temps = None
        e2e_path = ("installed apply_exl3_experts with pinned host x/ids/weights in, fp16 out to host; "
                    "H2D of the next step and D2H of the previous one overlap the layer on two copy streams")

        def public_call(xd, idd, wd):
            return ov.apply_exl3_experts(xd, idd, wd, layer, limit=LIMIT)
    else:
        e2e_path = ("ExpertParallel.prefill per rank with pinned host x/ids/weights in, fp16 out to host; "
                    "H2D of the next step and D2H of the previous one overlap the layer on two copy streams")

        def public_call(xd, idd, wd):
            # fp16 copy of this step's output: the next step's reduce rewrites the output buffer while the
            # D2H of this one may still run
            return eng.prefill(xd, idd, wd, layer, LIMIT).to(torch.float16)

    # Pipelined like a serving loop: the H2D copies of step i+1 (copy stream) and the D2H copy of step
    # i-1 (second copy stream) overlap the layer of step i; every step's copies are inside the timed
    # region, which ends when the last D2H has landed.
    h2d_stream = torch.cuda.Stream(dev)
    d2h_stream = torch.cuda.Stream(dev)
    in_bufs = [(torch.empty_like(x_h, device=dev), torch.empty_like(ids_h, device=dev),
                torch.empty_like(w_h, device=dev)) for _ in range(2)]
    out_hs = [out_h, torch.empty_like(out_h).pin_memory()]
    in_free = [None, None]

    def issue_h2d(i, start_ev=None):
        b = i % 2
        with torch.cuda.stream(h2d_stream):
            if start_ev is not None:
                h2d_stream.wait_event(start_ev)
            if in_free[b] is not None:
                h2d_stream.wait_event(in_free[b])
            for dst, src in zip(in_bufs[b], (x_h, ids_h, w_h)):
                dst.copy_(src, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d_stream)
        return ev

    def run_e2e(nsteps, start_ev=None):
        ready = issue_h2d(0, start_ev)
        for i in range(nsteps):
            nxt = issue_h2d(i + 1) if i + 1 < nsteps else None
            stream.wait_event(ready)
            xd, idd, wd = in_bufs[i % 2]
            o = public_call(xd, idd, wd)
            done = torch.cuda.Event()
            done.record(stream)
            in_free[i % 2] = done
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(done)
                out_hs[i % 2].copy_(o, non_blocking=True)
                o.record_stream(d2h_stream)
            ready = nxt
        stream.wait_stream(d2h_stream)

    run_e2e(max(2, args.warmup))
    torch.cuda.synchronize(dev)
    barrier()
    e0_ev = torch.cuda.Event(enable_timing=True)
    e1_ev = torch.cuda.Event(enable_timing=True)
    e0_ev.record(stream)
    run_e2e(args.steps, e0_ev)
    e1_ev.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0_ev.elapsed_time(e1_ev)
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(tt.item())
        barrier()
        eng.close()
    h2d = x_h.numel() * x_h.element_size() + ids_h.numel() * ids_h.element_size() + w_h.numel() * w_h.element_size()
    d2h = out_h.numel() * out_h.element_size()

    if rank != 0:
        return None, None
    pk = peaks()
    extra = {}
    if world == 1 and args.workload == "moe" and not args.graph and E == E_ and not args.no_extra:
        extra["chunk_sweep"] = chunk_sweep(layer, dev, stream, pk["tflops"])
        extra["small_batch_ms"] = small_batch_latency(layer, dev, stream)
        # the same layer with the other down stage (bit-repeatable combine, or the atomic scatter)
        other = not args.deterministic
        st, lay_ms = stage_times(lambda xx, ii, ww, hook: rt.grouped_prefill(xx, ii, ww, layer, LIMIT, stage_hook=hook,
                                                                            deterministic=other),
                                 x, ids, w, None, stream)
        extra["deterministic_down" if other else "atomic_down"] = {"layer_ms": lay_ms, "stages_ms": st}
    gemm_flops = 2.0 * rows_gate_up * D_ * 2 * f_gemm
    thin_on = os.environ.get("EXL3_B200_THIN_KERNEL", "1") != "0"
    thin_max = max(0, min(128, int(os.environ.get("EXL3_B200_THIN_MAX_ROWS", "96") or 96)))
    roof_kernel = ("gate|up GEMM stage (mode 0): " + (f"trellis_gemm (M-tiles of {thin_max + 1}..256 rows) + trellis_thin "
                                                      f"(M-tiles of 1..{thin_max} rows)" if thin_on else "trellis_gemm")
                   + ("" if world == 1 else ", rank 0"))
    roof_alg = f"2*R*d*2f = {gemm_flops:.4g} FLOP per stage, R={rows_gate_up}"
    if "gemm_gate_up" in stage_ms:
        gemm_ms = stage_ms["gemm_gate_up"]
    else:                                        # graph replay: the whole layer is one timed unit
        gemm_flops = 6.0 * rows_gate_up * D_ * f_gemm
        gemm_ms = stage_ms["layer"]
        roof_kernel = "whole layer (CUDA graph replay)"
        roof_alg = f"6*R*d*f = {gemm_flops:.4g} FLOP per layer, R={rows_gate_up}"
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12
    traffic, traffic_note = (profiled_traffic() if world == 1 and args.workload == "moe" and not args.graph
                             and args.tokens == 8192 and E == E_ else (None, "captured for config 1 only"))
    ms_step = elapsed_ms / args.steps
    metric, config = workload_config(args, world, E, T, f_gemm)
    res = {
        "metric": metric, "value": world * T * args.steps / (elapsed_ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if args.total_tokens else "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded EXL3 4-bpw trellis words, su/sv, x~N(0,1), Zipf(1.1) top-8 routing)",
        "config": config,
        "roofline": {"bound": "tensor", "kernel": roof_kernel,
                     "achieved": achieved, "peak": pk["tflops"], "unit": "TFLOP/s",
                     "frac": achieved / pk["tflops"],
                     "peak_note": (f"bf16 dense cuBLAS burst, {pk['source']}: the kernel runs inside a timed region "
                                   f"of well under a second at full clocks (frac of the sustained "
                                   f"{pk['tflops_sustained']:.0f}: {achieved / pk['tflops_sustained']:.3f})"),
                     "algorithmic": roof_alg,
                     "traffic": traffic, "traffic_note": traffic_note},
        "stages_ms": stage_ms,
        "clocks": clk,
        "e2e": {"value": world * T * args.steps / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms / args.steps,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "path": e2e_path},
        **extra,
        # route_hist + route_scatter + row_had + gemm + act_had + gemm + combine per layer (the router front-end
        # is router + scatter); with EP: pull, hist, scatter, row_had, gemm, act_had, gemm, push, reduce
        # with the atomic down stage there is no combine launch; each GEMM stage is two launches (two-block
        # tiles and thin tiles) unless EXL3_B200_THIN_KERNEL=0
        "gpu_launches": ((({"moe": 7, "dense-mlp": 7, "moe-block": 14, "glm-block": 14}[args.workload]
                           - (0 if args.deterministic else (2 if args.workload in ("moe-block", "glm-block") else 1))
                           + (2 if os.environ.get("EXL3_B200_THIN_KERNEL", "1") != "0" else 0)
                           * (2 if args.workload in ("moe-block", "glm-block") else 1))
                          if world == 1 else 9 + (2 if os.environ.get("EXL3_B200_THIN_KERNEL", "1") != "0" else 0))
                         * args.steps),
        "down_stage": "slot rows + fixed-order combine" if args.deterministic else "fp32 atomic scatter",
    }
    return res, (layer, x, ids, w)


def workload_config(args, world: int, E: int, T: int, f_gemm: int = F_):
    """(metric, config dict) of a run: the same for both arms (--impl ours / reference)."""
    metric = METRIC
    if world == 1 and args.workload == "dense-mlp":
        metric = "dense SwiGLU MLP prefill tokens/s (EXL3 4-bpw, same kernels)"
        workload = f"dense-mlp: one SwiGLU MLP, d={D_} f={f_gemm}, T={T} tokens"
        parallelism = "single GPU"
    elif world == 1 and args.workload == "glm-block":
        metric = "GLM MoE-block prefill tokens/s from hidden states (router + routed + shared expert)"
        workload = (f"glm-block: noaux_tc router (synthetic, Zipf-tilted bias) + E={E} routed experts + 1 shared "
                    f"expert, d={D_} f={F_} top-{K_}, T={T} tokens")
        parallelism = "single GPU"
    elif world == 1 and args.workload == "moe-block":
        metric = "MoE-block prefill tokens/s (routed experts + shared expert)"
        workload = (f"moe-block: E={E} routed experts + 1 shared expert, d={D_} f={F_} top-{K_}, T={T} tokens, "
                    f"{args.routing} routing")
        parallelism = "single GPU"
    elif world == 1:
        workload = (f"{'config1' if E == E_ and T == 8192 else 'custom'}: one MoE layer, E={E} d={D_} f={F_} "
                    f"top-{K_}, T={T} tokens/GPU, {args.routing} routing"
                    + (", replayed from a CUDA graph" if args.graph else ""))
        parallelism = "single GPU"
    else:
        total = T * world
        workload = (f"{'config4' if E == E_ and total == 32768 else 'expert-parallel'}: one MoE layer, "
                    f"E={E} d={D_} f={F_} top-{K_}, {T} tokens on each of {world} GPUs ({total} per step), "
                    f"{args.routing} routing")
        parallelism = (f"expert parallel: {E // world} experts per GPU ({args.placement} placement); over NVLink "
                       f"peer memory, each needed token row pulled once per GPU and one {args.combine} partial-sum "
                       f"row per (token, GPU) pushed back")
    config = {"workload": workload, "tokens_per_gpu": T, "experts": E, "hidden": D_, "intermediate": F_,
              "topk": K_, "routing": args.routing, "parallelism": parallelism,
              "l2": ("inputs larger than L2: 2.72 GB of packed expert weights stream every step"
                     if not (world == 1 and args.workload == "dense-mlp") else
                     f"activations larger than L2 ({T * 2 * f_gemm * 2 / 1e6:.0f} MB of gate|up rows per "
                     f"step); the {D_ * f_gemm * 3 / 2 / 1e6:.0f} MB of packed weights may stay in L2")}
    return metric, config


def run_reference(args, rank):
    """The reference's per-expert loop (the oracle's port of harness/proto_fp8.py:123-134) on the host
    cores, on the same config / metric as --impl ours: set-up once (every routed expert's weights
    decoded, as the reference does), then W warm-up and K timed steps, each step the loop over the
    whole layer (all routed experts, all T tokens).  With N > 1 ranks only rank 0 runs: one rank's
    T-token share of the N*T-token step, the loop being per token anyway."""
    if rank != 0:
        return None
    world = int(os.environ.get("WORLD_SIZE", "1"))
    threads = max(1, os.cpu_count() or 1)
    torch.set_num_threads(threads)
    T = args.tokens
    layer, x, ids, w = make_inputs(torch.device("cpu"), T, args.routing, E=args.experts)
    ids_np = ids.numpy()
    counts = np.bincount(ids_np.reshape(-1), minlength=args.experts)
    ref = CpuReferenceLayer(layer, [int(e) for e in np.nonzero(counts)[0]], threads)
    xf, w_cpu = x.float(), w.float()
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        ref.step(xf, ids_np, w_cpu)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    step_s = statistics.mean(times)
    v = T / step_s
    metric, config = workload_config(args, world, args.experts, T)
    sample = (f"the whole layer per step ({len(ref.w)} routed experts, {int(counts.sum())} routed rows, {T} tokens"
              + (f": one GPU's share of the {T * world}-token step" if world > 1 else "")
              + f"); one-time set-up {ref.setup_s:.1f} s (trellis decode {ref.decode_s:.1f} s) not timed, as the "
                f"reference builds its weights once; {cpu_host()}")
    return {"metric": metric, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (same seeds as --impl ours)",
            "impl": "reference", "config": config,
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "step_s": times, "setup_s": ref.setup_s}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.total_tokens:
        if args.total_tokens % world:
            raise SystemExit(f"--total-tokens {args.total_tokens} does not split evenly over {world} GPUs")
        args.tokens = args.total_tokens // world
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    res, inputs = run_ours(args, rank, world, local_rank)
    if rank == 0 and world == 1 and args.workload == "moe" and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(*inputs, max(1, os.cpu_count() or 1))
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
