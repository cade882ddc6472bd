#!/usr/bin/env python
"""SmolVLA action-chunk inference benchmark on 1..8 B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Workload (benchmark configuration C4, end-to-end): per observation one 512x512
image through the 12-layer SigLIP tower and the pixel-shuffle connector, 48
text tokens + 1 state token, a 113-token prefix through 16 text layers, then
the 16-layer action expert for 10 Euler steps -> one 50x32 action chunk.  One
step = one batch of B observations per GPU (default 256, the largest C4 batch);
observations are partitioned across ranks with no collective on the data path
(weak scaling: every rank runs B).  Weights are random and seeded, inputs are
synthetic with the benchmark's distributions.

The default arm times the CUDA path: the whole chunk forward is one CUDA graph
replay, timed with CUDA events between a barrier + synchronize on both sides,
max over ranks.  ``e2e`` times the public host API (host->device copies of
the observations and device->host copy of the actions inside the timed
region).  ``roofline`` comes from an eager pass with the library's launch
profiler.  ``cpu_baseline`` and ``--impl reference`` time the reference's own
CPU path (the oracle's bf16 restatement of its torch modules) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vla-to-npu_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "SmolVLA action chunks/sec"
UNIT = "chunks/s"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=256, help="observations per GPU per step")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip block timings, batch sweep and CPU baseline")
    ap.add_argument("--cpu-threads", type=int, default=0)
    ap.add_argument("--kernel-case", default="",
                    help="run one kernel of the step on a fixed small case (for ncu captures) and print its timing: "
                         + ", ".join(KERNEL_CASES))
    ap.add_argument("--ctas", type=int, default=0, choices=[0, 1, 2],
                    help="GEMM kernel cases: force one CTA (1) or a CTA pair (2) per tile; 0 = automatic")
    ap.add_argument("--tile-n", type=int, default=0, help="GEMM kernel cases: force the tile width BN; 0 = automatic")
    ap.add_argument("--splits", type=int, default=None,
                    help="GEMM kernel cases: one-CTA tiles with the K split over this many CTAs (1 = none, 0 = auto)")
    ap.add_argument("--attn-impl", type=int, default=0,
                    help="attention kernel cases: VLA_ATTN_* kernel choice (0 = automatic)")
    return ap.parse_args()


# name -> description; shapes are one GPU's share of the C4 step at 16 observations
# (inputs larger than L2, a few hundred MB on the device)
KERNEL_CASES = {
    "gemm_fc1": "SigLIP fc1 GEMM + bias + GELU, M=16384 N=3072 K=768",
    "gemm_qkv": "SigLIP QKV GEMM + bias, M=16384 N=2304 K=768",
    "gemm_fc2": "SigLIP fc2 GEMM + bias + residual, M=16384 N=768 K=3072",
    "gemm_plain": "plain GEMM (no epilogue work) at the fc1 shape, M=16384 N=3072 K=768",
    "gemm_plain_k3072": "plain GEMM, M=16384 N=3072 K=3072",
    "gemm_exp_down": "action-expert down projection + residual, M=12800 N=720 K=2048",
    "gemm_exp_o": "action-expert output projection + residual, M=12800 N=720 K=960",
    "gemm_exp_qkv": "action-expert self-attention QKV + RoPE on Q and K, M=12800 N=1600 K=720",
    "gemm_exp_gu": "action-expert gate/up + SwiGLU, M=12800 N=4096 K=720",
    "attn_vision": "SigLIP non-causal attention, 16 x 12 heads x 1024 x 1024",
    "attn_text": "text-prefix causal GQA attention (short-sequence tcgen05 kernel), 256 x 15 q / 5 kv heads x 113 x 113",
    "layer_norm": "SigLIP LayerNorm, 16384 x 768",
    "layer_norm_full": "SigLIP LayerNorm at the B = 256 step's shape, 262144 x 768 (805 MB moved, larger than L2)",
    "rms_norm": "text-width RMSNorm, 131072 x 960 (250 MB in, larger than L2)",
    "attn_exp_self": "action-expert causal self-attention, 512 x 15 q / 5 kv heads x 50 x 50 (AUTO kernel choice)",
    "attn_exp_cross": "action-expert cross-attention to the prefix, 512 x 15 q / 5 kv heads x 50 x 113 (AUTO)",
    "gemm_fc1_full": "SigLIP fc1 GEMM + bias + GELU at the bench step's shape, M=262144 N=3072 K=768 (2 GB)",
    "gemm_b1_down": "one observation's action-expert down projection + residual, M=50 N=720 K=2048",
    "gemm_b1_o": "one observation's action-expert output projection + residual, M=50 N=720 K=960",
    "gemm_b1_qkv": "one observation's action-expert QKV + RoPE, M=50 N=1600 K=720",
    "gemm_b1_gu": "one observation's action-expert gate/up + SwiGLU, M=50 N=4096 K=720",
}


def run_kernel_case(args):
    from vla_b200 import _lib
    from vla_b200 import device as dev
    from vla_b200 import weights as W
    torch.cuda.set_device(0)
    name = args.kernel_case
    if name not in KERNEL_CASES:
        raise SystemExit(f"unknown kernel case {name!r}; choose from {list(KERNEL_CASES)}")
    bf = torch.bfloat16
    if name.startswith("gemm"):
        M, N, K = {"gemm_fc1": (16384, 3072, 768), "gemm_fc1_full": (262144, 3072, 768), "gemm_qkv": (16384, 2304, 768),
                   "gemm_fc2": (16384, 768, 3072), "gemm_plain": (16384, 3072, 768),
                   "gemm_plain_k3072": (16384, 3072, 3072), "gemm_exp_down": (12800, 720, 2048),
                   "gemm_exp_o": (12800, 720, 960), "gemm_exp_qkv": (12800, 1600, 720),
                   "gemm_exp_gu": (12800, 4096, 720), "gemm_b1_down": (50, 720, 2048), "gemm_b1_o": (50, 720, 960),
                   "gemm_b1_qkv": (50, 1600, 720), "gemm_b1_gu": (50, 4096, 720)}[name]
        a = W.randn((M, K), 0, "kc.a").cuda()
        w = W.randn((N, K), 0, "kc.w", std=0.02).cuda()
        b = W.randn((N,), 0, "kc.b", std=0.01).cuda()
        swiglu = name in ("gemm_exp_gu", "gemm_b1_gu")
        c = torch.empty(M, N // 2 if swiglu else N, dtype=bf, device="cuda")
        res = (W.randn((M, N), 0, "kc.r").cuda()
               if name in ("gemm_fc2", "gemm_exp_down", "gemm_exp_o", "gemm_b1_down", "gemm_b1_o") else None)
        plain = name.startswith("gemm_plain") or name.startswith("gemm_exp") or name.startswith("gemm_b1")
        epi = dev.make_epilogue(bias=None if plain else b, residual=res,
                                act=_lib.ACT_GELU_TANH if name.startswith("gemm_fc1") else 0)
        if name in ("gemm_exp_qkv", "gemm_b1_qkv"):
            from vla_b200.model import rope_table
            cs = rope_table(50, 64, 10_000.0).cuda()
            epi = dev.make_epilogue(act=_lib.ACT_ROPE, rope_cs=cs, rope_seq=50, rope_ncols=1280)
        elif swiglu:
            epi = dev.make_epilogue(act=_lib.ACT_SWIGLU)
        if args.splits is not None:
            fn = lambda: dev.gemm(a, w, c, epi, tile_n=args.tile_n, splits=args.splits)  # noqa: E731
        else:
            fn = lambda: dev.gemm(a, w, c, epi, tile_n=args.tile_n, ctas=args.ctas)  # noqa: E731
        out_cols = c.shape[1]
        flops, nbytes = 2.0 * M * N * K, 2.0 * (M * K + N * K + M * out_cols * (2 if res is not None else 1))
    elif name == "attn_vision":
        B, L, H = 16, 1024, 12
        qkv = W.randn((B * L, 3 * H * 64), 0, "kc.qkv").cuda()
        o = torch.empty(B * L, H * 64, dtype=bf, device="cuda")
        fn = lambda: dev.attention(qkv[:, :H * 64], qkv[:, H * 64:2 * H * 64], qkv[:, 2 * H * 64:], o,  # noqa: E731
                                   batch=B, Lq=L, Lk=L, Hq=H, Hkv=H, q_batch=L * 3 * H * 64, k_batch=L * 3 * H * 64,
                                   v_batch=L * 3 * H * 64, o_batch=L * H * 64)
        flops, nbytes = 4.0 * B * H * L * L * 64, 2.0 * B * L * H * 64 * 4
    elif name == "attn_text":
        # the step's own shape (256 observations, 148 MB): 16 would leave most SMs idle
        B, L, Hq, Hkv = 256, 113, 15, 5
        cols = (Hq + 2 * Hkv) * 64
        qkv = W.randn((B * L, cols), 0, "kc.qkv").cuda()
        o = torch.empty(B * L, Hq * 64, dtype=bf, device="cuda")
        fn = lambda: dev.attention(qkv[:, :Hq * 64], qkv[:, Hq * 64:(Hq + Hkv) * 64],  # noqa: E731
                                   qkv[:, (Hq + Hkv) * 64:], o, batch=B, Lq=L, Lk=L, Hq=Hq, Hkv=Hkv,
                                   q_batch=L * cols, k_batch=L * cols, v_batch=L * cols, o_batch=L * Hq * 64,
                                   causal=True, impl=args.attn_impl)
        flops, nbytes = 4.0 * B * Hq * L * L * 64, 2.0 * B * L * (2 * Hq + 2 * Hkv) * 64
    elif name in ("attn_exp_self", "attn_exp_cross"):
        B, Lq, Hq, Hkv = 512, 50, 15, 5
        Lk = Lq if name == "attn_exp_self" else 113
        if name == "attn_exp_self":
            cols = (Hq + 2 * Hkv) * 64
            qkv = W.randn((B * Lq, cols), 0, "kc.qkv").cuda()
            q, k, v = qkv[:, :Hq * 64], qkv[:, Hq * 64:(Hq + Hkv) * 64], qkv[:, (Hq + Hkv) * 64:]
            qb = kb = Lq * cols
        else:
            q = W.randn((B * Lq, Hq * 64), 0, "kc.q").cuda()
            kv = W.randn((B * Lk, 2 * Hkv * 64), 0, "kc.kv").cuda()
            k, v = kv[:, :Hkv * 64], kv[:, Hkv * 64:]
            qb, kb = Lq * Hq * 64, Lk * 2 * Hkv * 64
        o = torch.empty(B * Lq, Hq * 64, dtype=bf, device="cuda")
        fn = lambda: dev.attention(q, k, v, o, batch=B, Lq=Lq, Lk=Lk, Hq=Hq, Hkv=Hkv, q_batch=qb,  # noqa: E731
                                   k_batch=kb, v_batch=kb, o_batch=Lq * Hq * 64, causal=name == "attn_exp_self",
                                   impl=args.attn_impl)
        flops, nbytes = 4.0 * B * Hq * Lq * Lk * 64, 2.0 * B * (2 * Lq * Hq + 2 * Lk * Hkv) * 64
    elif name == "rms_norm":
        x = W.randn((131072, 960), 0, "kc.x").cuda()
        g = torch.ones(960, dtype=bf, device="cuda")
        y = torch.empty_like(x)
        fn = lambda: dev.rms_norm(x, g, 1e-5, out=y)  # noqa: E731
        flops, nbytes = 0.0, 4.0 * 131072 * 960
    else:
        rows = 262144 if name == "layer_norm_full" else 16384
        x = W.randn((rows, 768), 0, "kc.x").cuda()
        g, bb = torch.ones(768, dtype=bf, device="cuda"), torch.zeros(768, dtype=bf, device="cuda")
        y = torch.empty_like(x)
        fn = lambda: dev.layer_norm(x, g, bb, 1e-6, out=y)  # noqa: E731
        flops, nbytes = 0.0, 4.0 * rows * 768
    for _ in range(max(args.warmup, 1)):
        fn()
    torch.cuda.synchronize()
    # the timed launches replay as one CUDA graph, so that host launch cost (ctypes,
    # tensor-map encoding) does not set the pace of short kernels
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(args.steps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    dev.sync_check()
    print(json.dumps({"kernel_case": name, "what": KERNEL_CASES[name], "ms": ms,
                      "tflops": flops / ms / 1e9 if flops else None, "gbs": nbytes / ms / 1e6}), flush=True)


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(backend="nccl"):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def gather_floats(vals, world: int) -> list:
    """Every rank's list of floats, gathered to every rank (rank order)."""
    if world == 1:
        return [list(vals)]
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    outs = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(outs, t)
    return [o.tolist() for o in outs]


def strong_scaling(model, dev_in, world, global_batches=(8, 64, 256), reps=10) -> dict:
    """Fixed global batch split evenly across the ranks (benchmark configuration
    C4: B observations sharded by batch over the GPUs): chunks/s of the whole job,
    timed per rank with CUDA events over graph replays, max over ranks."""
    res = {}
    for G in global_batches:
        if G % world:
            continue
        b = G // world
        model.allocate(b)
        model.load_inputs(dev_in["images"][:b], dev_in["token_ids"][:b], dev_in["state"][:b], dev_in["noise"][:b])
        model.capture()
        for _ in range(3):
            model.replay()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            model.replay()
        e1.record()
        e1.synchronize()
        t = max_over_ranks(e0.elapsed_time(e1) / reps, world)
        res[str(G)] = {"per_gpu_batch": b, "ms_per_step": round(t, 4), "chunks_per_s": round(G / (t / 1e3), 2)}
    B = dev_in["images"].shape[0]
    model.allocate(B)
    model.load_inputs(dev_in["images"], dev_in["token_ids"], dev_in["state"], dev_in["noise"])
    return res


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,clocks.mem")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.25)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        power = [num(r[3]) for r in rows if num(r[3]) is not None]
        loaded = [num(r[1]) for r in rows if num(r[3]) is not None and num(r[3]) > 300 and num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(loaded or sm) if (loaded or sm) else None,
                "sm_max_mhz": num(rows[0][2]), "reasons": reasons, "samples": len(rows),
                "samples_under_load": len(loaded), "power_w_max": max(power) if power else None,
                "mem_mhz": statistics.median([num(r[9]) for r in rows if num(r[9]) is not None] or [0])}


# ---------------------------------------------------------------------------
# the CPU path (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
def cpu_chunk_seconds(n_obs: int, threads: int) -> tuple:
    """Time the reference's own bf16 CPU path (oracle restatement of its torch modules)
    for ``n_obs`` full action chunks (one observation each); returns (seconds, threads)."""
    from oracle import smolvla_ref as R
    from vla_b200 import weights as W
    from vla_b200.configs import SmolVLACfg
    if threads > 0:
        torch.set_num_threads(threads)
    cfg = SmolVLACfg()
    params = W.smolvla_params(cfg, seed=0)
    obs = W.observation_batch(cfg, 1, seed=1)
    with torch.no_grad():
        t0 = time.perf_counter()
        for _ in range(n_obs):
            R.smolvla_chunk(obs, params, cfg, dt=torch.bfloat16)
        dt = time.perf_counter() - t0
    return dt, torch.get_num_threads()


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = args.cpu_threads or os.cpu_count()
    torch.set_num_threads(threads)
    from oracle import smolvla_ref as R
    from vla_b200 import weights as W
    from vla_b200.configs import SmolVLACfg
    cfg = SmolVLACfg()
    params = W.smolvla_params(cfg, seed=0)
    obs = W.observation_batch(cfg, 1, seed=1)
    with torch.no_grad():
        for _ in range(args.warmup):
            R.smolvla_chunk(obs, params, cfg, dt=torch.bfloat16)
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            R.smolvla_chunk(obs, params, cfg, dt=torch.bfloat16)
            times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    value = 1.0 / sec
    sample = ("1 observation per step (one full action chunk: vision tower, prefix, 16 text layers, "
              "10 Euler steps of the 16-layer expert) through the bf16 CPU restatement of the reference's "
              "torch modules")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random weights and observations)",
        "config": workload_config(args, args.batch, world),
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample, "cpu_model": cpu_model(), "host_logical_cpus": os.cpu_count()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args, batch, world):
    return {
        "workload": "C4 end-to-end SmolVLA action-chunk inference: 512x512 image -> 12 SigLIP layers -> "
                    "pixel-shuffle connector; 113-token prefix -> 16 text layers; 16-layer action expert x 10 "
                    "Euler steps -> 50x32 action chunk",
        "global_batch": batch * world, "per_gpu_batch": batch, "prefix_tokens": 113, "image": 512,
        "vision_layers": 12, "text_layers": 16, "expert_layers": 16, "euler_steps": 10, "chunk": 50,
        "parallelism": f"dp{world} (observations partitioned, no collective on the data path)",
        "l2_policy": "working set larger than L2 (0.8 GB of weights + per-step activations), no flush",
    }


# ---------------------------------------------------------------------------
# the CUDA path
# ---------------------------------------------------------------------------
# The step's GEMMs with their fused epilogues: (name, M, N, K, epilogue)
STEP_GEMMS = [
    ("vision fc1 +bias +GELU", 262144, 3072, 768, "gelu"),
    ("vision fc2 +bias +residual", 262144, 768, 3072, "bias_res"),
    ("vision qkv +bias", 262144, 2304, 768, "bias"),
    ("vision o +bias +residual", 262144, 768, 768, "bias_res"),
    ("text gate/up SwiGLU", 28928, 5120, 960, "swiglu"),
    ("text down +residual", 28928, 960, 2560, "res"),
    ("text qkv RoPE", 28928, 1600, 960, "rope"),
    ("text o +residual", 28928, 960, 960, "res"),
    ("expert gate/up SwiGLU", 12800, 4096, 720, "swiglu"),
    ("expert down +residual", 12800, 720, 2048, "res"),
    ("expert qkv RoPE", 12800, 1600, 720, "rope"),
    ("expert cross q RoPE", 12800, 960, 720, "rope"),
    ("expert o +residual", 12800, 720, 960, "res"),
]


def gemm_shape_rates(peak_tflops: float, reps: int = 20) -> list:
    """Each GEMM of the B = 256 step at its shape and epilogue, timed as a CUDA graph
    of `reps` back-to-back launches (launch overlap between them as inside the step's
    graph).  The launch profile's per-launch events instead cut that overlap and
    charge each launch its ramp and tail, which costs the short expert GEMMs 30-60 %."""
    from vla_b200 import _lib
    from vla_b200 import device as dev
    from vla_b200.model import rope_table
    bf = torch.bfloat16
    out = []
    g = torch.Generator(device="cpu").manual_seed(5)
    for name, M, N, K, kind in STEP_GEMMS:
        a = (torch.randn(M, K, generator=g, dtype=torch.float32)).to(bf).cuda()
        w = (torch.randn(N, K, generator=g, dtype=torch.float32) * 0.02).to(bf).cuda()
        oc = N // 2 if kind == "swiglu" else N
        c = torch.empty(M, oc, dtype=bf, device="cuda")
        bias = torch.zeros(N, dtype=bf, device="cuda")
        res = torch.randn(M, oc, generator=g, dtype=torch.float32).to(bf).cuda() if "res" in kind else None
        if kind == "gelu":
            epi = dev.make_epilogue(bias=bias, act=_lib.ACT_GELU_TANH)
        elif kind == "bias":
            epi = dev.make_epilogue(bias=bias)
        elif kind == "bias_res":
            epi = dev.make_epilogue(bias=bias, residual=res)
        elif kind == "res":
            epi = dev.make_epilogue(residual=res)
        elif kind == "swiglu":
            epi = dev.make_epilogue(act=_lib.ACT_SWIGLU)
        else:
            seq = 113 if M == 28928 else 50
            cs = rope_table(seq, 64, 1e4).cuda()
            epi = dev.make_epilogue(act=_lib.ACT_ROPE, rope_cs=cs, rope_seq=seq, rope_ncols=min(N, 1280))
        dev.gemm(a, w, c, epi)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                dev.gemm(a, w, c, epi)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) / reps * 1e3
        tf = 2.0 * M * N * K / (us * 1e-6) / 1e12
        out.append({"gemm": name, "mnk": [M, N, K], "us": round(us, 2), "tflops": round(tf, 1),
                    "frac_of_bf16_peak": round(tf / peak_tflops, 3)})
        del a, w, c, res, graph
    torch.cuda.empty_cache()
    return out


def norm_rates(hbm_peak: float, reps: int = 20) -> list:
    """The step's row norms at their B = 256 shapes, timed like gemm_shape_rates."""
    from vla_b200 import device as dev
    bf = torch.bfloat16
    out = []
    for name, M, N, ln in (("expert RMSNorm", 12800, 720, False), ("text RMSNorm", 28928, 960, False),
                           ("vision LayerNorm", 262144, 768, True)):
        x = torch.randn(M, N, device="cuda").to(bf)
        y = torch.empty_like(x)
        g = torch.ones(N, dtype=bf, device="cuda")
        b = torch.zeros(N, dtype=bf, device="cuda")
        fn = (lambda: dev.layer_norm(x, g, b, 1e-6, out=y)) if ln else (lambda: dev.rms_norm(x, g, 1e-5, out=y))
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) / reps * 1e3
        gbs = 4.0 * M * N / (us * 1e-6) / 1e9
        out.append({"norm": name, "shape": [M, N], "us": round(us, 2), "gbs": round(gbs, 1),
                    "frac_of_hbm": round(gbs / hbm_peak, 3),
                    "l2_resident": 4.0 * M * N < 126e6})
        del x, y, graph
    return out


def profile_pass(model) -> dict:
    """Eager forward under the launch profiler; the queue is pre-filled behind a
    sleep kernel so launch gaps do not enter the per-kernel device times."""
    from vla_b200 import _lib
    import ctypes
    lib = _lib.load()
    cap = 8192
    _lib.call("vla_profile_start", cap)
    torch.cuda._sleep(400_000_000)
    model.forward_device()
    recs = (_lib.ProfileRecord * cap)()
    n = ctypes.c_int32(0)
    _lib.call("vla_profile_stop", recs, cap, ctypes.byref(n))
    agg = {}
    shapes = {}
    for i in range(min(n.value, cap)):
        r = recs[i]
        k = _lib.KIND_NAMES[r.kind]
        a = agg.setdefault(k, {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
        a["launches"] += 1
        a["ms"] += r.ms
        a["flops"] += r.flops
        a["bytes"] += r.bytes
        if r.kind == 0:
            sh = shapes.setdefault((r.m, r.n, r.k, r.tile_n, r.ctas), [0, 0.0, 0.0])
            sh[0] += 1
            sh[1] += r.ms
            sh[2] += r.flops
    del lib
    top = sorted(shapes.items(), key=lambda kv: -kv[1][1])[:12]
    agg["_gemm_shapes"] = [{"mnk": list(s[:3]), "tile_n": s[3], "ctas": s[4], "launches": v[0], "ms": round(v[1], 3),
                            "tflops": round(v[2] / (v[1] * 1e-3) / 1e12, 1)} for s, v in top]
    return agg


# DRAM bytes (read + write) of one launch of a step GEMM, from an ncu capture of
# that GEMM alone at the step's own shape:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none \
#       -k regex:gemm -s 3 -c 1 python bench.py --kernel-case gemm_fc1_full --steps 2 --warmup 3
# (M N K) -> bytes.  Algorithmic minimum for the fc1 shape: A 402.7 MB + W 4.7 MB +
# C 1610.6 MB = 2018 MB.
DRAM_TRAFFIC_PER_LAUNCH = {(262144, 3072, 768): 445.34e6 + 1.56e9}


# Algorithmic work of the benchmark blocks at B = 1 (valid tokens only; attention
# counted dense over the unmasked region, causal at full L^2): FLOPs, and the
# bytes a B = 1 pass must move from HBM (weights once per pass, plus the
# activations in and out).  C3 re-reads the expert's weights on each of its 10
# Euler steps (196 MB > the 126 MB L2).
BLOCK_WORK = {
    # C0: q 235.93 M + k,v 157.29 M + o 235.93 M + gate/up 1258.29 M + down 629.15 M + QK^T, PV 2 x 31.46 M
    "C0_text_block": (2.580e9, 20.3e6),
    # C1: qkvo 4.832 G + MLP 9.664 G + attention 3.221 G; 14.17 MB weights + 3.15 MB in/out
    "C1_siglip_block": (17.72e9, 17.3e6),
    # C2: patch 1.208 G + 12 x 17.72 G + connector 1.510 G; 197 MB of weights (+1.6 MB image in)
    "C2_vision_tower_connector": (215.3e9, 198.8e6),
    # C3: 10 steps x (8 self x 636.29 M + 8 cross x 602.30 M) + cross K/V 0.37 G; 10 x 196 MB weights
    "C3_action_expert_10_steps": (99.5e9, 1.96e9),
}


def block_timings(model, peaks, reps=20) -> dict:
    """Per-block device time (us) at B = 1 via CUDA-graph replay, and the fraction
    of the block's roofline time max(FLOPs / bf16 peak, bytes / HBM peak) that it
    reaches (blocks timed alone: the burst bf16 peak).  C0 / C1 are one layer at the
    benchmark configurations; C2 (vision tower + connector) and C3 (16-layer expert
    x 10 Euler steps against the cached prefix K/V, key padding on) run inside the
    model at one observation."""
    from vla_b200 import device as dev
    from vla_b200 import weights as W
    from vla_b200.configs import SmolVLACfg, TextCfg, VisionCfg
    from vla_b200.model import LlamaLayerWeights, VisionLayerWeights, rope_table
    out = {}

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / reps * 1e3

    ws = dev.Workspace()
    t = TextCfg()
    lw = LlamaLayerWeights(W.text_block_params(t), t, "cuda")
    x = W.randn((128, t.hidden), 0, "b.x").cuda()
    cs = rope_table(128, 64, t.rope_theta).cuda()
    qkv = torch.empty(128, t.q_dim + 2 * t.kv_dim, dtype=torch.bfloat16, device="cuda")
    out["C0_text_block"] = timed(lambda: dev.llama_self_layer(lw.struct, x, 1, 128, cs, ws, qkv_out=qkv))
    v = VisionCfg()
    vw = VisionLayerWeights(W.vision_block_params(v), v, "cuda")
    xv = W.randn((1024, v.hidden), 0, "b.xv").cuda()
    out["C1_siglip_block"] = timed(lambda: dev.vision_layer(vw.struct, xv, 1, 1024, ws))
    cfg = SmolVLACfg()
    obs = W.observation_batch(cfg, 1, seed=7)
    model.allocate(1)
    model.load_inputs(*(obs[k].cuda() for k in ("images", "token_ids", "state", "noise")))
    model.forward_device()  # fills the prefix K/V the expert attends to
    out["C2_vision_tower_connector"] = timed(model.vision_tower)
    model.action.set_kv_len(torch.tensor([113], dtype=torch.int32, device="cuda"))
    out["C3_action_expert_10_steps"] = timed(model.action_expert)
    model.action.set_kv_len(None)
    torch.cuda.synchronize()
    tf = peaks.get("bf16_tflops") or 1590.0
    bw = peaks.get("hbm_gbs") or 6650.0
    res = {}
    for k, us in out.items():
        flops, nbytes = BLOCK_WORK[k]
        t_tensor, t_hbm = flops / (tf * 1e12), nbytes / (bw * 1e9)
        roof_us = max(t_tensor, t_hbm) * 1e6
        res[k] = {"us": round(us, 2), "roofline_us": round(roof_us, 2), "bound": "tensor" if t_tensor >= t_hbm else "hbm",
                  "frac_of_roofline": round(roof_us / us, 4), "gflop": flops / 1e9, "mbytes": nbytes / 1e6}
    res["peaks"] = {"bf16_tflops": tf, "hbm_gbs": bw,
                    "source": "measured (MEASURED_PEAKS.json, burst bf16)" if peaks else "fallback"}
    return res


def run_ours(args, rank, world, local):
    from vla_b200 import _lib
    from vla_b200 import weights as W
    from vla_b200.configs import SmolVLACfg
    from vla_b200.model import SmolVLA

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = SmolVLACfg()
    B = args.batch
    params = W.smolvla_params(cfg, seed=0)
    model = SmolVLA(cfg, params, dev)
    del params
    obs = W.observation_batch(cfg, B, seed=1 + rank)
    host = {
        "images": obs["images"].pin_memory(),
        "token_ids": obs["token_ids"].pin_memory(),
        "state": obs["state"].pin_memory(),
        "noise": obs["noise"].pin_memory(),
    }
    dev_in = {k: v.to(dev) for k, v in host.items()}
    model.load_inputs(dev_in["images"], dev_in["token_ids"], dev_in["state"], dev_in["noise"])
    # count this library's launches in one eager forward
    lib = _lib.load()
    c0 = lib.vla_launch_count()
    model.forward_device()
    launches_per_step = lib.vla_launch_count() - c0
    torch.cuda.synchronize()
    model.capture()

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        model.replay()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        model.replay()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = max_over_ranks(ms, world)

    # end to end through the public host API
    out_host = torch.empty((B, cfg.expert.chunk, cfg.expert.action_dim), dtype=torch.float32, pin_memory=True)
    for _ in range(2):
        model.infer_host(host["images"], host["token_ids"], host["state"], host["noise"], out=out_host)
    barrier(world)
    torch.cuda.synchronize()
    # streamed host APIs: every step moves its observations in and its actions
    # out; infer_host_stream overlaps step k+1's host->device copies with step
    # k's compute, infer_overlapped also runs step k+1's vision / text half
    # concurrently with step k's action expert.  The faster one is the e2e figure.
    batches = [(host["images"], host["token_ids"], host["state"], host["noise"])] * args.steps
    outs = [torch.empty_like(out_host).pin_memory() for _ in range(args.steps)]

    def e2e_ms(api):
        api(batches[:2], outs[:2])
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        api(batches, outs)
        e1.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / args.steps * 1e3
        barrier(world)
        return max(e0.elapsed_time(e1) / args.steps, wall)

    e2e_apis = {"SmolVLA.infer_host_stream": e2e_ms(model.infer_host_stream),
                "SmolVLA.infer_overlapped": e2e_ms(model.infer_overlapped)}
    e2e_api = min(e2e_apis, key=e2e_apis.get)
    ms_e2e = e2e_apis[e2e_api]
    out_host = outs[-1]
    ms_e2e_max = max_over_ranks(ms_e2e, world)
    e2e_all = {k: round(world * B / (max_over_ranks(v, world) / 1e3), 3) for k, v in e2e_apis.items()}
    e2e_camera = None
    if not args.no_extras:
        # the same observations as uint8 camera frames [B, 512, 512, 3]: the GPU
        # resizes / normalises them and writes the patch operand in one kernel
        frames = ((host["images"].float() + 1.0) * 127.5).round().clamp(0, 255).to(torch.uint8)
        frames = frames.permute(0, 2, 3, 1).contiguous().pin_memory()
        batches = [(frames, host["token_ids"], host["state"], host["noise"])] * args.steps
        ms_cam = max_over_ranks(e2e_ms(model.infer_overlapped), world)
        e2e_camera = {"value": round(world * B / (ms_cam / 1e3), 3), "unit": UNIT,
                      "h2d_bytes_per_step": frames.numel() + sum(host[k].numel() * host[k].element_size()
                                                                 for k in ("token_ids", "state", "noise")),
                      "d2h_bytes_per_step": out_host.numel() * out_host.element_size(),
                      "api": "SmolVLA.infer_overlapped with uint8 camera frames"}
        model.load_inputs(dev_in["images"], dev_in["token_ids"], dev_in["state"], dev_in["noise"])
        del frames, batches
    clk = clocks.stop()
    per_rank = gather_floats([ms, clk.get("sm_mhz") or 0.0, ms_e2e], world)
    strong = strong_scaling(model, dev_in, world) if (world > 1 and not args.no_extras) else None
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = out_host.numel() * out_host.element_size()
    assert torch.isfinite(out_host).all(), "non-finite actions"

    extras = {}
    roofline = None
    kernels = None
    cpu_base = None
    if rank == 0:
        agg = profile_pass(model)
        extras["gemm_shapes"] = agg.pop("_gemm_shapes")
        total_ms = sum(a["ms"] for a in agg.values())
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except (OSError, ValueError):
            pass
        tflops_peak = peaks.get("bf16_tflops_sustained") or 1400.0
        hbm_peak = peaks.get("hbm_gbs") or 6650.0
        peak_src = "measured" if peaks else "fallback"
        kernels = {}
        for k, a in sorted(agg.items(), key=lambda kv: -kv[1]["ms"]):
            ent = {"launches": a["launches"], "ms_per_step": round(a["ms"], 4),
                   "share": round(a["ms"] / total_ms, 4) if total_ms else None}
            if a["flops"] > 0:
                ach = a["flops"] / (a["ms"] * 1e-3) / 1e12
                ent.update(achieved_tflops=round(ach, 1), frac_of_bf16_peak=round(ach / tflops_peak, 3))
            if a["bytes"] > 0:
                gbs = a["bytes"] / (a["ms"] * 1e-3) / 1e9
                ent.update(achieved_gbs=round(gbs, 1), frac_of_hbm=round(gbs / hbm_peak, 3))
            kernels[k] = ent
        # dominant single kernel: the GEMM shape with the largest share of the step
        top = extras["gemm_shapes"][0] if extras.get("gemm_shapes") else None
        traffic = DRAM_TRAFFIC_PER_LAUNCH.get(tuple(top["mnk"])) if top else None
        if top:
            ach = 2.0 * top["mnk"][0] * top["mnk"][1] * top["mnk"][2] * top["launches"] / (top["ms"] * 1e-3) / 1e12
            roofline = {"bound": "tensor",
                        "kernel": (f"{'gemm_bf16_tc2_kernel' if top['ctas'] == 2 else 'gemm_bf16_tc_kernel'}<{top['tile_n']}"
                                   f"{', 2' if top['ctas'] == 2 else ''}> "
                                   f"M,N,K={top['mnk']} ({top['launches']} launches per step)"),
                        "achieved": round(ach, 1), "peak": tflops_peak, "unit": "TFLOP/s",
                        "frac": round(ach / tflops_peak, 4), "traffic": traffic,
                        "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this "
                                        "GEMM at the step's shape (bench.py --kernel-case gemm_fc1_full); null "
                                        "for shapes without a capture",
                        "peak_source": f"{peak_src} bf16_tflops_sustained",
                        "algorithmic_flops_per_launch": 2.0 * top["mnk"][0] * top["mnk"][1] * top["mnk"][2],
                        "avg_launch_ms": top["ms"] / top["launches"]}
        if not args.no_extras and world == 1:
            try:
                extras["blocks"] = block_timings(model, peaks)
            except Exception as exc:  # extras never fail the benchmark line
                extras["blocks_error"] = repr(exc)
            try:
                extras["gemm_rates_graph"] = {
                    "peak": tflops_peak, "peak_source": f"{peak_src} bf16_tflops_sustained",
                    "note": "each step GEMM alone at the B = 256 shape and epilogue, 20 launches in one CUDA "
                            "graph, operands L2-warm across the launches",
                    "shapes": gemm_shape_rates(tflops_peak)}
            except Exception as exc:
                extras["gemm_rates_graph_error"] = repr(exc)
            try:
                extras["norm_rates_graph"] = {"peak_gbs": hbm_peak, "shapes": norm_rates(hbm_peak),
                                              "note": "algorithmic bytes (read + write) over graph-replay time; "
                                                      "shapes under L2 size stay L2-resident across the launches"}
            except Exception as exc:
                extras["norm_rates_graph_error"] = repr(exc)
            sweep = {}
            for b in (1, 8, 64):
                model.allocate(b)
                model.load_inputs(dev_in["images"][:b], dev_in["token_ids"][:b], dev_in["state"][:b],
                                  dev_in["noise"][:b])
                model.capture()
                for _ in range(3):
                    model.replay()
                torch.cuda.synchronize()
                a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = 10
                a_.record()
                for _ in range(reps):
                    model.replay()
                b_.record()
                b_.synchronize()
                sweep[str(b)] = round(b / (a_.elapsed_time(b_) / reps / 1e3), 2)
            sweep[str(B)] = round(B / (ms / 1e3), 2)
            extras["batch_sweep_chunks_per_s"] = sweep
            # a stream of small batches through the overlapped host API: batch k+1's
            # vision / text half runs beside batch k's action expert
            ov = {}
            for b in (1, 8):
                hb = [(host["images"][i * b:(i + 1) * b].pin_memory(), host["token_ids"][i * b:(i + 1) * b].pin_memory(),
                       host["state"][i * b:(i + 1) * b].pin_memory(), host["noise"][i * b:(i + 1) * b].pin_memory())
                      for i in range(20)]
                hout = [torch.empty(b, cfg.expert.chunk, cfg.expert.action_dim).pin_memory() for _ in range(20)]
                model.infer_overlapped(hb[:3], hout[:3])
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                model.infer_overlapped(hb, hout)
                ov[str(b)] = round(20 * b / (time.perf_counter() - t0), 2)
            extras["stream_overlapped_chunks_per_s"] = ov
            # where one observation's chunk spends its time: the launch profile at B = 1
            try:
                model.allocate(1)
                model.load_inputs(dev_in["images"][:1], dev_in["token_ids"][:1], dev_in["state"][:1],
                                  dev_in["noise"][:1])
                agg1 = profile_pass(model)
                shapes1 = agg1.pop("_gemm_shapes")
                extras["b1_profile"] = {
                    "kinds": {k: {"launches": a["launches"], "ms": round(a["ms"], 4),
                                  "us_per_launch": round(1e3 * a["ms"] / a["launches"], 2)}
                              for k, a in sorted(agg1.items(), key=lambda kv: -kv[1]["ms"])},
                    "top_gemm_shapes": shapes1[:6],
                    "note": "eager forward at B = 1 with CUDA events around every launch (launch overlap "
                            "between kernels is lost to the events, so the sum exceeds the graph replay time)"}
            except Exception as exc:
                extras["b1_profile_error"] = repr(exc)
            try:
                n_obs = 2
                sec, thr = cpu_chunk_seconds(n_obs, args.cpu_threads or os.cpu_count())
                cpu_base = {"value": n_obs / sec, "unit": UNIT, "cores": thr, "kind": "port", "cpu_model": cpu_model(),
                            "host_logical_cpus": os.cpu_count(),
                            "sample": f"{n_obs} observations (full action chunks, B=1 each) through the bf16 CPU "
                                      "restatement of the reference's torch modules"}
            except Exception as exc:
                cpu_base = {"value": None, "unit": UNIT, "cores": None, "kind": "port", "error": repr(exc)}

    if rank == 0:
        value = world * B / (ms_max / 1e3)
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights; images U(-1,1), token ids U[0,49152), state/noise N(0,1))",
            "config": workload_config(args, B, world),
            "e2e": {"value": round(world * B / (ms_e2e_max / 1e3), 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "api": e2e_api, "by_api": e2e_all,
                    "note": "the public streamed host API over K batches: pinned host observations (bf16 images, "
                            "int32 ids, bf16 state, fp32 noise) copied in and fp32 actions copied out every step; "
                            "the slower of CUDA events and the wall clock"},
            "gpu_launches": int(launches_per_step) * args.steps,
            "per_rank": [{"rank": i, "ms_per_step": round(r[0], 4), "sm_mhz_median": r[1], "e2e_ms_per_step": round(r[2], 4)}
                         for i, r in enumerate(per_rank)],
            "clocks": clk,
            "roofline": roofline,
            "kernels": kernels,
            "cpu_baseline": cpu_base,
        }
        if strong is not None:
            line["strong_scaling"] = strong
        if e2e_camera is not None:
            line["e2e_camera_u8"] = e2e_camera
        line.update(extras)
        print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.kernel_case:
        run_kernel_case(args)
        return
    if args.impl == "reference":
        # the CPU reference path runs on rank 0 only; other ranks exit without work
        run_reference(args, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, world, local = dist_setup("nccl")
    if world != args.gpus:
        log(f"note: --gpus {args.gpus} but WORLD_SIZE {world}; using WORLD_SIZE")
    run_ours(args, rank, world, local)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
