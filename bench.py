#!/usr/bin/env python
"""Benchmark: decode tok/s at the Qwen3-30B-A3B shape on B200.

Default workload (the metric's config): one decode
token of the 48-layer 30B-A3B-shaped model with random weights -- embedding
row, 48 x (attention half, 32 q / 4 kv heads of 128, + MoE block: hidden
2048, 128 experts, top-8, expert FFN 768, gate/up q4_K, down q6_K), output
norm, LM head (151,936 x 2048 q6_K), greedy pick -- with --ctx cache rows
already filled, batch 1.  Every expert resident in HBM (18.8 GB); router
rows carry a Zipf(1.1) popularity bias.  Synthetic data, generated on the
device.  At N > 1 (torchrun) the same sequence runs with its experts split
over the ranks (expert parallelism, e % N == rank) and one cross-rank sum
of the k x H slot buffer per layer (--ep-comm fused, the default: the
block's own kernel pushes its rows over NVLink peer memory and adds the
ranks' sum into x; p2p: one kernel after the block does the exchange and
the combine; nccl: an NCCL all-reduce): strong scaling of one sequence.

`value`: tokens/s, device-timed with CUDA events (a CUDA graph at N = 1).
`e2e`: a greedy chain through the C ABI with host buffers (token id in,
pick out, fed back).  `roofline`: the MoE block (25,550,848 algorithmic
bytes) over its own time measured in the same run, against the measured HBM
copy bandwidth; `step_roofline`: the whole token's bytes.  `check`: the
greedy picks, equal at every N (expert parallelism is bit-exact).

Other workloads: --workload cfg3 (the 48 MoE blocks alone; replicas at
N > 1), --workload cfg4 (6 GiB expert budget, the rest streamed from pinned
host memory), --workload batch (--batch B tokens per step through the 48 MoE
blocks on the tensor-core batch path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload ...]
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (30B-A3B shape, q4_K) at 1/2/4/8 B200; MoE-layer % of HBM peak"
H, F, E, K_TOP, N_LAYERS = 2048, 768, 128, 8, 48
Q4_K, Q6_K = 12, 14
QD = Q6_K                          # down projection format
SG = (H // 256) * 144 * F          # gate / up slab bytes per expert
SD = (F // 256) * 210 * H          # down slab bytes per expert
ALG_BYTES_LAYER = K_TOP * (2 * SG + SD) + E * H * 4 + 3 * H * 4   # 25,550,848
SHAPE = "cfg2"


def set_shape(name: str) -> None:
    """The MoE stack's shape: cfg2 (the 30B-A3B layer of configs[1] / [2],
    48 layers, down q6_K) or cfg5 (configs[4]'s 235B-A22B layer: H 4096, F
    1536, 128 experts top-8, every matrix q4_K, 94 layers)."""
    global H, F, N_LAYERS, QD, SG, SD, ALG_BYTES_LAYER, SHAPE
    if name == "cfg5":
        H, F, N_LAYERS, QD = 4096, 1536, 94, Q4_K
    SG = (H // 256) * 144 * F
    SD = (F // 256) * (210 if QD == Q6_K else 144) * H
    ALG_BYTES_LAYER = K_TOP * (2 * SG + SD) + E * H * 4 + 3 * H * 4
    SHAPE = name


def shape_desc() -> str:
    qd = "q6_K" if QD == Q6_K else "q4_K"
    return f"H{H} E{E} top{K_TOP} F{F}, gate/up q4_K, down {qd}"


ZIPF_S, ZIPF_TAU, ZIPF_KAPPA = 1.1, 0.25, 4.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def zipf_bias(layer: int) -> np.ndarray:
    """a_e = tau * ln p_pi(e), p_j ~ j^-s, pi a seeded permutation."""
    rng = np.random.default_rng(9000 + layer)
    p = np.arange(1, E + 1, dtype=np.float64) ** -ZIPF_S
    p /= p.sum()
    perm = rng.permutation(E)
    return (ZIPF_TAU * np.log(p[perm])).astype(np.float32)


def zipf_dir() -> np.ndarray:
    m = np.random.default_rng(8999).normal(0, 1, H)
    return (m / np.linalg.norm(m)).astype(np.float32)


def token_bank(n: int) -> np.ndarray:
    rng = np.random.default_rng(102)
    return (rng.normal(0, 1, (n, H)) + ZIPF_KAPPA * zipf_dir()[None, :]).astype(np.float32)


def router_host(layer: int) -> np.ndarray:
    rng = np.random.default_rng(5000 + layer)
    r = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    return r + zipf_bias(layer)[:, None] * zipf_dir()[None, :]


# -------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampled during the timed region."""

    def __init__(self, dev: int):
        self.dev = dev
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,utilization.gpu")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            time.sleep(0.2)
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        self.f.flush()
        rows = []
        try:
            with open(self.f.name) as f:
                for line in f:
                    parts = [x.strip() for x in line.split(",")]
                    if len(parts) >= 7:
                        rows.append(parts)
        except Exception:
            pass
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        busy = [r for r in rows if r[6].isdigit() and int(r[6]) > 0] or rows
        sm = [float(r[0]) for r in busy if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in busy if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i in range(4) if r[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(busy)}


# ---------------------------------------------------------- CPU legs
def cpu_layer(seed: int = 0):
    """One 30B-shaped MoE layer on the host (same shapes and value
    distribution as the device workload), quantised by the oracle."""
    from oracle import oracle as O
    rng = np.random.default_rng(7000 + seed)
    gate = np.empty(E * SG, np.uint8)
    up = np.empty(E * SG, np.uint8)
    down = np.empty(E * SD, np.uint8)
    for e in range(E):
        gate[e * SG:(e + 1) * SG] = O.quantize(Q4_K, rng.standard_normal((F, H), np.float32) * np.float32(0.02)).reshape(-1)
        up[e * SG:(e + 1) * SG] = O.quantize(Q4_K, rng.standard_normal((F, H), np.float32) * np.float32(0.02)).reshape(-1)
        down[e * SD:(e + 1) * SD] = O.quantize(QD, rng.standard_normal((H, F), np.float32) * np.float32(0.02)).reshape(-1)
    return router_host(0), np.ones(H, np.float32), gate, up, down


def time_cpu(budget_s: float, nthreads: int):
    """Times the oracle MoE block (C, OpenMP over rows) for ~budget_s.
    Returns (tok/s for the 48-layer stack, seconds per layer, reps)."""
    from oracle import oracle as O
    router, norm, gate, up, down = cpu_layer()
    toks = token_bank(16)
    O.moe_block_mt(toks[0], norm, 1e-6, router, K_TOP, True, (Q4_K, Q4_K, QD), gate, up, down, F, nthreads)
    t0 = time.perf_counter()
    reps = 0
    while True:
        O.moe_block_mt(toks[reps % 16], norm, 1e-6, router, K_TOP, True, (Q4_K, Q4_K, QD), gate, up, down, F,
                       nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 2000:
            break
    per_layer = el / reps
    return 1.0 / (N_LAYERS * per_layer), per_layer, reps


def run_reference(args, rank: int) -> int:
    """--impl reference: the reference's CPU implementation of the path (the
    C restatement in oracle/, all host threads) on the same workload, each
    step a bounded sample of it scaled to one token.  decode: one layer's
    attention half (args.ctx cache rows) and MoE block plus 1/48 of
    the LM head per step, i.e. 1/48 of a token; cfg3: two MoE layers."""
    if rank != 0:
        return 0
    from oracle import oracle as O
    O.build()
    nth = os.cpu_count() or 1
    router, norm, gate, up, down = cpu_layer()
    toks = token_bank(16)
    qts = (Q4_K, Q4_K, Q6_K)
    if args.workload == "decode":
        rng = np.random.default_rng(11)
        qd, kvd, ctx = N_HEADS * HD, N_KV * HD, args.ctx

        def q(qt, r, c):
            return O.quantize(qt, rng.standard_normal((r, c), np.float32) * np.float32(0.02)).reshape(-1)
        ws = [(Q4_K, q(Q4_K, qd, H)), (Q4_K, q(Q4_K, kvd, H)), (Q6_K, q(Q6_K, kvd, H)), (Q4_K, q(Q4_K, H, qd))]
        kc = rng.standard_normal((ctx + 1, kvd), np.float32)
        vc = rng.standard_normal((ctx + 1, kvd), np.float32)
        ones_h, ones_d = np.ones(H, np.float32), np.ones(HD, np.float32)
        head_rows = -(-N_VOCAB // N_LAYERS)
        head = q(Q6_K, head_rows, H)

        def step(i):
            x = toks[i % 16].copy()
            x = O.attn_block(x, ones_h, 1e-6, N_HEADS, N_KV, HD, ones_d, ones_d, 1e6, ws, ctx, kc, vc)
            x = O.moe_block_mt(x, norm, 1e-6, router, K_TOP, True, qts, gate, up, down, F, nth)
            O.matvec_q(Q6_K, head, head_rows, H, x)
        per_step_tokens = 1.0 / N_LAYERS
        sample = (f"per step one layer of the whole decode step (attention half at {ctx} cache rows, one thread; "
                  f"MoE block, {nth} threads) and 1/48 of the LM head ({head_rows} q6_K rows), i.e. 1/48 of a "
                  f"token; scaled to the token")
        workload = decode_config(args.layers, ctx, int(os.environ.get("WORLD_SIZE", "1")), args.ep_comm)
        metric = METRIC
    else:
        def step(i):
            for j in range(2):
                O.moe_block_mt(toks[(i + j) % 16], norm, 1e-6, router, K_TOP, True, qts, gate, up, down, F, nth)
        per_step_tokens = 2.0 / N_LAYERS
        sample = "2 of the 48 MoE layers per step (one 30B-shaped layer re-run), scaled to the 48-layer token"
        workload = workload_config(args.gpus)
        metric = METRIC
    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    el = time.perf_counter() - t0
    v = args.steps * per_step_tokens / el
    line = {"impl": "reference", "metric": metric, "value": v, "unit": "tok/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", str(args.gpus))),
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload,
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": nth, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference = C restatement of the reference CPU path (oracle/); the reference itself is "
                    "Rust+Vulkan and cannot run here (no Rust toolchain, no graphics stack)"}
    print(json.dumps(line), flush=True)
    return 0


def workload_config(n: int):
    name = "cfg2 MoE layer" if SHAPE == "cfg2" else "cfg5 (configs[4]) MoE layer"
    return {"workload": f"{name} ({shape_desc()}) stacked x{N_LAYERS} (cfg3 MoE path), batch-1 decode, "
                        "all experts resident",
            "n_layers": N_LAYERS, "n_embd": H, "n_expert": E, "n_expert_used": K_TOP, "n_ff": F,
            "global_batch": n, "parallelism": f"replicas x{n}" if n > 1 else "single",
            "l2": f"inputs larger than L2 ({N_LAYERS * K_TOP * (2 * SG + SD) / 1e9:.1f} GB of expert slabs per "
                  "token vs 126 MB L2)",
            "router": "Zipf(1.1) popularity bias"}


# ------------------------------------------------------------- GPU arm
def build_model(dev: int, n_layers: int, unique: int = 4):
    import torch

    from styx_b200 import ops
    torch.cuda.set_device(dev)
    d = f"cuda:{dev}"
    base = []
    for u in range(min(unique, n_layers)):
        g = ops.synth_quant(Q4_K, E * F, H, 1000 + 3 * u, 0.02, device=dev)
        up = ops.synth_quant(Q4_K, E * F, H, 1001 + 3 * u, 0.02, device=dev)
        dn = ops.synth_quant(QD, E * H, F, 1002 + 3 * u, 0.02, device=dev)
        base.append((g, up, dn))
    torch.cuda.synchronize()
    layers = []
    norm = torch.ones(H, dtype=torch.float32, device=d)
    for layer in range(n_layers):
        if layer < len(base):
            g, up, dn = base[layer]
        else:   # distinct copies: every layer streams its own bytes
            g, up, dn = (t.clone() for t in base[layer % len(base)])
        router = torch.from_numpy(router_host(layer)).to(d)
        layers.append(ops.LayerWeights(norm, router, ops.Experts(Q4_K, g, SG), ops.Experts(Q4_K, up, SG),
                                       ops.Experts(QD, dn, SD)))
    torch.cuda.synchronize()
    return layers


# ---------------------------------------------------------- whole decode step
N_HEADS, N_KV, HD, N_VOCAB = 32, 4, 128, 151936   # Qwen3-30B-A3B attention and vocabulary


def ep_moe_layers(dev: int, n_layers: int, world: int, rank: int, unique: int = 4):
    """This rank's MoE layers under expert parallelism: the experts e with
    e % world == rank of each layer as dense hot buffers in ascending id
    order (remap: expert -> local slot, SKIP for the others), no full tensor.
    The bytes are the ones build_model generates for world 1."""
    import torch

    from styx_b200 import ops
    d = f"cuda:{dev}"
    owned = [e for e in range(E) if e % world == rank]
    remap = torch.full((E,), -1, dtype=torch.int32)
    remap[owned] = torch.arange(len(owned), dtype=torch.int32)
    remap = remap.to(d)
    base = []
    for u in range(min(unique, n_layers)):
        base.append((ops.synth_quant(Q4_K, E * F, H, 1000 + 3 * u, 0.02, device=dev),
                     ops.synth_quant(Q4_K, E * F, H, 1001 + 3 * u, 0.02, device=dev),
                     ops.synth_quant(QD, E * H, F, 1002 + 3 * u, 0.02, device=dev)))
    torch.cuda.synchronize()
    norm = torch.ones(H, dtype=torch.float32, device=d)

    def mine(t, slab):
        return torch.cat([t[e * slab:(e + 1) * slab] for e in owned])
    layers = []
    for layer in range(n_layers):
        g, up, dn = base[layer % len(base)]
        router = torch.from_numpy(router_host(layer)).to(d)
        layers.append(ops.LayerWeights(norm, router, ops.Experts(Q4_K, None, SG, hot=mine(g, SG)),
                                       ops.Experts(Q4_K, None, SG, hot=mine(up, SG)),
                                       ops.Experts(QD, None, SD, hot=mine(dn, SD)), remap=remap))
    del base
    torch.cuda.synchronize()
    return layers


def decode_config(L: int, ctx: int, world: int, comm: str = "fused") -> dict:
    """The decode workload's config (both arms)."""
    return {"workload": f"whole decode step at the 30B-A3B shape (configs[2]): embedding row, {L} x "
                        f"(attention {N_HEADS}q/{N_KV}kv x {HD} + MoE block H{H} E{E} top{K_TOP} F{F}, "
                        f"gate/up q4_K, down q6_K), LM head {N_VOCAB} x {H} q6_K, greedy pick; batch 1; "
                        f"{ctx} cache rows before the token",
            "ctx": ctx, "global_batch": 1,
            "parallelism": (f"expert-parallel x{world}: experts e % {world} == rank, per layer one cross-rank "
                            f"sum of the {K_TOP} x {H} slot buffer ("
                            + {"fused": "over NVLink peer memory, inside the block's kernel",
                               "p2p": "one kernel over NVLink peer memory",
                               "nccl": "NCCL all-reduce"}[comm] + ")"
                            if world > 1 else "single"),
            "l2": "inputs larger than L2 (%.2f GB read per token)" % (decode_bytes_per_token(L, ctx) / 1e9)}


def decode_model(local: int, L: int, ctx: int, world: int, rank: int, allreduce=None, ep_comm=None,
                 ep_fused: bool = True):
    """The 30B-shaped decode model with random weights: attention q/k/o q4_K,
    v q6_K (four generated layer bases, copied to every layer), the MoE
    layers (every expert at world 1, this rank's experts under expert
    parallelism), embedding q4_K, LM head q6_K; ctx cache rows filled."""
    import torch

    from styx_b200 import ops
    from styx_b200.decode import DecodeLayer, DecodeModel, DecodeParams
    dev = f"cuda:{local}"
    qd, kvd = N_HEADS * HD, N_KV * HD
    moe = build_model(local, L) if world == 1 else ep_moe_layers(local, L, world, rank)
    ones = lambda n: torch.ones(n, dtype=torch.float32, device=dev)   # noqa: E731
    base = []
    for u in range(min(4, L)):
        base.append((ops.synth_quant(Q4_K, qd, H, 2000 + 4 * u, 0.02, device=local),
                     ops.synth_quant(Q4_K, kvd, H, 2001 + 4 * u, 0.02, device=local),
                     ops.synth_quant(Q6_K, kvd, H, 2002 + 4 * u, 0.02, device=local),
                     ops.synth_quant(Q4_K, H, qd, 2003 + 4 * u, 0.02, device=local)))
    layers = []
    for li in range(L):
        wq, wk, wv, wo = base[li] if li < len(base) else (t.clone() for t in base[li % len(base)])
        attn = ops.AttnWeights(ones(H), ops.DenseWeight(Q4_K, wq), ops.DenseWeight(Q4_K, wk),
                               ops.DenseWeight(Q6_K, wv), ops.DenseWeight(Q4_K, wo), q_norm=ones(HD), k_norm=ones(HD))
        layers.append(DecodeLayer(attn, moe[li]))
    embd = ops.DenseWeight(Q4_K, ops.synth_quant(Q4_K, N_VOCAB, H, 3000, 0.5, device=local))
    head = ops.DenseWeight(Q6_K, ops.synth_quant(Q6_K, N_VOCAB, H, 3001, 0.02, device=local))
    p = DecodeParams(L, H, N_HEADS, N_KV, HD, F, E, K_TOP, N_VOCAB)
    model = DecodeModel(p, embd, layers, ones(H), head, ctx + 1, local, allreduce=allreduce, ep_comm=ep_comm,
                        ep_fused=ep_fused)
    model.kcache[:, :ctx].copy_(ops.synth_f32(L * ctx * kvd, 4000, 0, 1.0, device=local).view(L, ctx, kvd))
    model.vcache[:, :ctx].copy_(ops.synth_f32(L * ctx * kvd, 4001, 0, 1.0, device=local).view(L, ctx, kvd))
    model.n_past = ctx
    torch.cuda.synchronize()
    return model


def run_decode(args, local: int, rank: int, world: int) -> int:
    """The whole decode step at the 30B shape: embedding row,
    48 x (attention half + MoE block), output norm, LM head (q6_K, 151,936
    rows), greedy pick, with args.ctx cache rows already filled.  One
    sequence; at N > 1 its experts are split over the ranks (expert
    parallelism: every rank runs the step on the same token, holds the
    experts e % N == rank, and one NCCL all-reduce per layer sums the slot
    contributions), so the scaling is strong.  The token is a CUDA graph
    recorded through the C ABI at N = 1 and, with the peer-memory combine
    (--ep-comm fused / p2p: only this library's kernels), at N > 1 too; with
    --ep-comm nccl the step runs eagerly (its all-reduces go through
    torch.distributed)."""
    import ctypes as C
    import zlib

    import torch

    from styx_b200 import _lib, ops
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device(dev))
        pg = dist
    L, ctx = args.layers, args.ctx
    p2p = pg is not None and args.ep_comm in ("fused", "p2p")
    ep_comm = None
    if p2p:   # the cross-rank sum and the combine as one kernel over NVLink peer memory
        ep_comm = ops.EpComm(rank, world, K_TOP, H, local)
        ep_comm.connect_with(pg)
    allreduce = (lambda t: pg.all_reduce(t)) if pg and not p2p else None
    model = decode_model(local, L, ctx, world, rank, allreduce, ep_comm, args.ep_comm == "fused")
    blk_ctx = model.moe.ctx
    blk_ctx.set_option(_lib.OPT_EXCLUSIVE, 0 if args.shared_device else 1)
    blk_ctx.set_option(_lib.OPT_ATTN_KERNELS, args.attn_kernels)
    blk_ctx.set_option(_lib.OPT_MOE_KERNELS, args.moe_kernels)
    lib, cx = _lib.lib(), blk_ctx.handle
    stream = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(stream.cuda_stream)
    rng = np.random.default_rng(7)
    toks = torch.from_numpy(rng.integers(0, N_VOCAB, 4096).astype(np.int32)).to(dev)
    with torch.cuda.stream(stream):
        model.tok.copy_(toks[:1])
        model.pos.fill_(ctx)
    model.step(stream)                      # eager once
    stream.synchronize()
    blk_ctx.check_device_error(stream)
    attn_path, moe_path = model.attn.last_path(), blk_ctx.last_moe_path()
    graph = None
    if world == 1 or p2p:
        graph = C.c_void_p()
        _lib.check(lib.styx_graph_begin(cx, sp))
        model.step(stream)
        _lib.check(lib.styx_graph_end(cx, sp, C.byref(graph)))

    def run_step():
        if graph is not None:
            _lib.check(lib.styx_graph_launch(cx, graph, sp))
        else:
            model.step(stream)

    def replay(i):
        with torch.cuda.stream(stream):
            model.tok.copy_(toks[i % toks.numel():i % toks.numel() + 1])
        run_step()

    def barrier():
        if pg:
            pg.barrier()

    def max_over_ranks(v):
        if not pg:
            return v
        t = torch.tensor([v], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    for i in range(args.warmup):
        replay(i)
    stream.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            replay(i)
        ev1.record(stream)
        stream.synchronize()
    barrier()
    el_ms = max_over_ranks(ev0.elapsed_time(ev1))
    blk_ctx.check_device_error(stream)
    ms = el_ms / args.steps

    # e2e: a real greedy chain through the C ABI with host buffers -- the
    # token id uploaded from pinned memory, the step, the greedy pick read
    # back into pinned memory and fed in as the next token; the picks are
    # also the cross-N identity check (expert parallelism is bit-exact)
    hin, hout = ops.HostBuffer(4, local), ops.HostBuffer(4, local)
    n_e2e = args.e2e_steps or args.steps
    tok_host = 1234
    picks = []
    barrier()
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n_e2e):
        hin.tensor.view(torch.int32)[0] = tok_host
        _lib.check(lib.styx_upload(cx, C.c_void_p(model.tok.data_ptr()), 0, C.c_void_p(hin.ptr), 4, sp))
        run_step()
        _lib.check(lib.styx_download(cx, C.c_void_p(hout.ptr), C.c_void_p(model.next.data_ptr()), 0, 4, sp))
        stream.synchronize()
        tok_host = int(hout.tensor.view(torch.int32)[0])
        picks.append(tok_host)
    e1.record(stream)
    stream.synchronize()
    t_wall = time.perf_counter() - t_wall
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    x_bytes = model.x.cpu().numpy().tobytes()
    check = {"greedy_tokens": picks[:8], "greedy_crc32": zlib.crc32(np.array(picks, np.int32).tobytes()),
             "x_crc32": zlib.crc32(x_bytes), "steps": n_e2e}
    if graph is not None:
        _lib.check(lib.styx_graph_destroy(cx, graph))
        graph = None

    # the MoE block's roofline, measured in the same run: at N = 1 the 48
    # blocks alone as a graph (the kernel the block runs, nothing else); at
    # N > 1 the per-layer compute (styx_moe_block_ep) and all-reduce apart
    def timed(fn, reps):
        fn()
        stream.synchronize()
        barrier()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        z.record(stream)
        stream.synchronize()
        barrier()
        return max_over_ranks(a.elapsed_time(z)) / reps

    peak, peak_kind = peaks()
    reps = max(3, args.steps // 4)
    ep = None
    if world == 1:
        g2 = C.c_void_p()
        _lib.check(lib.styx_graph_begin(cx, sp))
        for li, ly in enumerate(model.layers):
            model.moe.forward(model.x, ly.moe, li, model.ids, stream=stream)
        _lib.check(lib.styx_graph_end(cx, sp, C.byref(g2)))
        t_layer = timed(lambda: _lib.check(lib.styx_graph_launch(cx, g2, sp)), reps) / L * 1e-3
        _lib.check(lib.styx_graph_destroy(cx, g2))
        achieved = ALG_BYTES_LAYER / t_layer / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_kind": peak_kind, "alg_bytes": ALG_BYTES_LAYER, "us_per_layer": t_layer * 1e6,
                "unit_of_work": "one MoE block (one k_moe_fused launch), timed as 48 blocks in a graph in this run"}
    else:
        fused = args.ep_comm == "fused"

        def moe_ep_only():
            for li, ly in enumerate(model.layers):
                model.moe.forward_ep(model.x, ly.moe, li, model.ids, model.partial, stream=stream)

        def allreduce_only():
            if p2p:
                for _ in range(L):
                    ep_comm.combine(model.partial, model.x, stream=stream)
                return
            with torch.cuda.stream(stream):
                for _ in range(L):
                    pg.all_reduce(model.partial)

        def ep_blocks():
            for li, ly in enumerate(model.layers):
                ep_comm.moe_block(model.moe, model.x, ly.moe, li, model.ids, stream=stream)

        def as_graph(fn):
            # fused / p2p: the pieces as recorded graphs, as the step runs them
            if not p2p:
                return fn, None
            g = C.c_void_p()
            _lib.check(lib.styx_graph_begin(cx, sp))
            fn()
            _lib.check(lib.styx_graph_end(cx, sp, C.byref(g)))
            return (lambda: _lib.check(lib.styx_graph_launch(cx, g, sp))), g

        graphs = []
        f_moe, g = as_graph(moe_ep_only)
        graphs.append(g)
        f_ar, g = as_graph(ep_blocks if fused else allreduce_only)
        graphs.append(g)
        t_moe = timed(f_moe, reps) / L
        t_ar = timed(f_ar, reps) / L
        for g in graphs:
            if g is not None:
                _lib.check(lib.styx_graph_destroy(cx, g))
        if fused:   # t_ar timed the block and its exchange together
            t_layer = t_ar * 1e-3
            t_ar = t_ar - t_moe
        else:
            t_layer = (t_moe + t_ar) * 1e-3
        achieved = ALG_BYTES_LAYER / t_layer / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak * world, "unit": "GB/s",
                "frac": achieved / (peak * world), "peak_kind": peak_kind + f" x{world}",
                "alg_bytes": ALG_BYTES_LAYER, "us_per_layer": t_layer * 1e6,
                "unit_of_work": "one MoE layer over all ranks: " + (
                    "styx_ep_moe_block on every rank (the block with the exchange and the combine as its "
                    "epilogue: one k_moe_fused launch)" if fused else
                    "styx_moe_block_ep on every rank + the cross-rank sum of the k x H slot buffer" +
                    (" and the combine (styx_ep_combine)" if p2p else ""))}
        ep = {"moe_ep_us_per_layer": t_moe * 1e3, "allreduce_us_per_layer": t_ar * 1e3,
              "allreduce_bytes": K_TOP * H * 4, "limiter": "all-reduce latency" if t_ar > t_moe else
              "the block's compute", "ranks": world,
              "collective": {"fused": "styx_ep_moe_block: each CTA of the block's kernel stores its rows of every "
                                      "slot into the peers' inboxes over NVLink (CUDA IPC), release adds / acquire "
                                      "loads of arrival counters, the ranks' sum added into x in the same kernel "
                                      "(allreduce_us_per_layer: the block with its exchange minus the block alone)",
                             "p2p": "styx_ep_combine: plain stores into the peers' inboxes over NVLink (CUDA IPC), "
                                    "release adds / acquire loads of arrival counters, the sum and the combine in "
                                    "one kernel after the block",
                             "nccl": "NCCL all-reduce (torch.distributed) + styx_moe_combine"}[args.ep_comm]}
    bytes_tok = decode_bytes_per_token(L, ctx)
    step_achieved = bytes_tok / (ms * 1e-3) / 1e9
    one_attn, one_moe = attn_path in (1, 3), moe_path in (1, 6)
    ep_launch = 1 if world > 1 and not (args.ep_comm == "fused" and moe_path == 1) else 0
    launches = 1 + L * ((1 if one_attn else 8) + (1 if one_moe else 3) + ep_launch) + 3
    attn_form = {1: "one cooperative kernel per layer", 3: "one launch of thread-block clusters per layer "
                 "(a cluster per kv head)"}.get(attn_path, "eight kernels per layer")
    moe_form = {1: "single cooperative kernel per layer", 6: "one launch of thread-block clusters per layer "
                "(a cluster per selected slot)"}.get(moe_path, "three kernels per layer")
    line = {
        "metric": METRIC, "value": 1e3 / ms, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "int8-dp4a/f32 (q4_K,q6_K weights)",
        "data": "synthetic (random weights of the 30B-A3B shapes, random cache rows)",
        "config": decode_config(L, ctx, world, args.ep_comm),
        "kernels": {"launch": ("CUDA graph" if world == 1 or p2p else "eager (NCCL all-reduces between the kernels)") +
                              (", cooperative" if args.shared_device else
                               ", plain single kernels (STYX_OPT_EXCLUSIVE: the bench owns its GPU)"),
                    "attention": attn_form, "moe": moe_form},
        "e2e": {"value": n_e2e / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                "wall_s": t_wall, "form": "greedy chain: each step's pick read back and fed in as the next token"},
        "gpu_launches": args.steps * launches,
        "roofline": roof,
        "step_roofline": {"bytes": bytes_tok, "achieved": step_achieved, "peak": peak * world, "unit": "GB/s",
                          "frac": step_achieved / (peak * world)},
        "check": check,
        "clocks": clk.summary(),
    }
    if ep:
        line["ep"] = ep
    tp = os.path.join(ROOT, "profiles", "moe_layer_traffic.json")
    if world == 1 and os.path.exists(tp):
        try:
            roof["traffic"] = json.load(open(tp)).get("dram_bytes_per_layer")
        except Exception:
            roof["traffic"] = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            nth = os.cpu_count() or 1
            v, desc = time_cpu_decode(args.cpu_seconds, nth, ctx)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": nth, "kind": "port", "sample": desc}
        except Exception as e:  # the CPU leg must not sink the GPU number
            line["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": 0, "kind": "port",
                                    "sample": f"failed: {e}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    hin.free()
    hout.free()
    if pg:
        pg.barrier()
        if ep_comm is not None:
            ep_comm.close()
            pg.barrier()   # no rank unmaps an inbox a peer still writes
        pg.destroy_process_group()
    return 0


def time_cpu_decode(budget_s: float, nthreads: int, ctx: int):
    """The decode step's CPU leg on the oracle: the MoE block (C, OpenMP over
    rows, time_cpu), the attention half of a layer (C, one thread; 30B shapes,
    ctx cache rows) and a 4,096-row sample of the LM head (C, one thread),
    scaled to 48 layers + the whole head.  Returns (tok/s, description)."""
    from oracle import oracle as O
    _, moe_layer, reps = time_cpu(budget_s * 0.6, nthreads)
    rng = np.random.default_rng(11)
    qd, kvd = N_HEADS * HD, N_KV * HD

    def q(qt, r, c):
        return O.quantize(qt, rng.standard_normal((r, c), np.float32) * np.float32(0.02)).reshape(-1)
    ws = [(Q4_K, q(Q4_K, qd, H)), (Q4_K, q(Q4_K, kvd, H)), (Q6_K, q(Q6_K, kvd, H)), (Q4_K, q(Q4_K, H, qd))]
    kc = rng.standard_normal((ctx + 1, kvd), np.float32)
    vc = rng.standard_normal((ctx + 1, kvd), np.float32)
    x = rng.standard_normal(H, np.float32)
    ones_h, ones_d = np.ones(H, np.float32), np.ones(HD, np.float32)
    t0 = time.perf_counter()
    n_attn = 0
    while n_attn < 3 or time.perf_counter() - t0 < budget_s * 0.2:
        O.attn_block(x, ones_h, 1e-6, N_HEADS, N_KV, HD, ones_d, ones_d, 1e6, ws, ctx, kc, vc)
        n_attn += 1
    attn_layer = (time.perf_counter() - t0) / n_attn
    rows = 4096
    head = q(Q6_K, rows, H)
    t0 = time.perf_counter()
    O.matvec_q(Q6_K, head, rows, H, x)
    head_s = (time.perf_counter() - t0) * N_VOCAB / rows
    per_tok = N_LAYERS * (moe_layer + attn_layer) + head_s
    return 1.0 / per_tok, (f"oracle: MoE block {moe_layer * 1e3:.2f} ms/layer ({reps} runs, {nthreads} threads), "
                           f"attention half {attn_layer * 1e3:.2f} ms/layer at {ctx} rows ({n_attn} runs, 1 thread), "
                           f"LM head {head_s * 1e3:.1f} ms (4,096-row sample, 1 thread); scaled to 48 layers")


def decode_bytes_per_token(n_layers: int, ctx: int) -> int:
    """Algorithmic bytes of one decode step: per layer the MoE block's bytes,
    the attention weights (q, k, o q4_K; v q6_K), the norms and the cache
    rows read (ctx + 1 of K and of V) and written (1 each); then the output
    norm, the LM head (q6_K) and the embedding row (q4_K)."""
    q4 = lambda r, c: r * (c // 256) * 144   # noqa: E731
    q6 = lambda r, c: r * (c // 256) * 210   # noqa: E731
    qd, kvd = N_HEADS * HD, N_KV * HD
    attn = q4(qd, H) + q4(kvd, H) + q6(kvd, H) + q4(H, qd) + (H + 2 * HD) * 4
    cache = 2 * (ctx + 1) * kvd * 4 + 2 * kvd * 4
    return n_layers * (ALG_BYTES_LAYER + attn + cache) + H * 4 + q6(N_VOCAB, H) + q4(1, H)


# ---------------------------------------------------------- cfg4 arm
def zipf_hist(n_layers: int, n_tok: int = 4096):
    """Synthetic (layer, expert, hits) histogram: n_tok * k draws per layer
    from the same Zipf(1.1) popularity the layer's router carries (the
    permutation of zipf_bias), seeded by rng(104)."""
    rng = np.random.default_rng(104)
    L_, E_, H_ = [], [], []
    p = np.arange(1, E + 1, dtype=np.float64) ** -ZIPF_S
    p /= p.sum()
    for l in range(n_layers):
        perm = np.random.default_rng(9000 + l).permutation(E)
        counts = rng.multinomial(n_tok * K_TOP, p[perm])
        L_ += [l] * E
        E_ += list(range(E))
        H_ += counts.tolist()
    return np.array(L_, np.int32), np.array(E_, np.int32), np.array(H_, np.uint64)


def run_streaming(args, local: int) -> int:
    """the 30B-shaped stack with a 6 GiB HBM expert budget; every
    full expert tensor in pinned host memory, popularity pinning from a
    Zipf(1.1) hit histogram, the next token's predicted cold experts copied
    into the HBM arena on a side stream, online repinning every 128 tokens
    (at most 2 swaps per layer), unpredicted cold experts read in place."""
    import torch

    from styx_b200 import ops
    from styx_b200.streaming import ExpertStreamer
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    L = args.layers
    budget = 6 << 30
    host = []
    hbufs = []
    for l in range(L):
        trio = []
        u = l % 4
        for t, (qt, rows, cols, slab) in enumerate(((Q4_K, E * F, H, SG), (Q4_K, E * F, H, SG),
                                                      (Q6_K, E * H, F, SD))):
            d = ops.synth_quant(qt, rows, cols, 1000 + 3 * u + t, 0.02, device=local)
            hb = ops.HostBuffer(E * slab, local)
            hb.tensor.copy_(d.view(torch.uint8))   # device -> pinned host
            hbufs.append(hb)
            trio.append(hb.tensor)
            del d
        host.append(tuple(trio))
    torch.cuda.synchronize()
    hist = zipf_hist(L)
    st = ExpertStreamer(ops.Dims(H, F, E, K_TOP), L, (Q4_K, Q4_K, Q6_K), (SG, SG, SD), host, hist, budget,
                        device=local, repin_interval=128, repin_max=2, prefetch=not args.no_prefetch,
                        prefetch_min_hit=args.prefetch_min_hit, prefetch_probe=16)
    norm = torch.ones(H, dtype=torch.float32, device=dev)
    routers = [torch.from_numpy(router_host(l)).to(dev) for l in range(L)]
    layers = [st.layer_weights(l, norm, routers[l]) for l in range(L)]
    blk = ops.MoeBlock(ops.Dims(H, F, E, K_TOP), local)
    bank = torch.from_numpy(token_bank(64)).to(dev)
    x = torch.empty(H, dtype=torch.float32, device=dev)
    ids = torch.zeros(L * 64, dtype=torch.int32, device=dev)
    evA = [torch.cuda.Event(enable_timing=True) for _ in range(L)]
    evB = [torch.cuda.Event(enable_timing=True) for _ in range(L + 1)]
    prev = None
    n_warm = args.warmup
    tok_ms, wait_ms, kern_ms = [], [], []
    t_wall = 0.0
    for t in range(n_warm + args.tokens):
        if t == n_warm:
            st.stats = type(st.stats)(cold_by_layer=[0] * L)
            torch.cuda.synchronize()
            t_wall = time.perf_counter()
        st.before_token(t, prev, layers)
        x.copy_(bank[t % 64])
        evB[0].record()
        w = 0.0
        for l in range(L):
            st.wait_layer(l)
            evA[l].record()
            blk.forward(x, layers[l], l, ids)
            evB[l + 1].record()
        prev = ids.cpu().numpy()        # the ids read back after the token (last_expert_ids)
        st.after_token(prev)
        if t >= n_warm:
            tok_ms.append(evB[0].elapsed_time(evB[L]))
            wait_ms.append(sum(evB[l].elapsed_time(evA[l]) for l in range(L)))
            kern_ms.append(sum(evA[l].elapsed_time(evB[l + 1]) for l in range(L)))
    t_wall = time.perf_counter() - t_wall
    blk.ctx.check_device_error()
    hud = st.hud()
    n = args.tokens
    copy_ms = st.stats.copy_ms / max(n, 1)
    exposed = sum(wait_ms) / max(n, 1)
    line = {"metric": "decode tok/s (30B-A3B shape, q4_K), 6 GiB HBM expert budget, cold experts streamed from "
                      "pinned host memory",
            "value": n / (sum(tok_ms) / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": n, "warmup": n_warm,
            "ms_per_step": sum(tok_ms) / n, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8-dp4a/f32 (q4_K,q6_K weights)", "data": "synthetic",
            "config": {"workload": "cfg4: cfg3 MoE stack, 6 GiB expert budget, Zipf(1.1) pinning histogram, "
                                   "repin every 128 tokens (max 2 per layer), copy-engine prefetch of the previous "
                                   "token's cold experts" + (
                                       "" if args.no_prefetch else
                                       f" while it pays (probe of 16 tokens after each repin; off below a "
                                       f"{args.prefetch_min_hit:.0%} hit rate)"),
                       "n_layers": L, "budget_bytes": budget, "tokens": n},
            "hud": hud,
            "streaming": {"copy_ms_per_tok": copy_ms, "exposed_wait_ms_per_tok": exposed,
                          "kernel_ms_per_tok": sum(kern_ms) / max(n, 1),
                          "overlap_pct": 100.0 * max(0.0, 1.0 - exposed / copy_ms) if copy_ms > 0 else None,
                          "hit_rate_pct": hud["hot_pct"],
                          "bytes_streamed_per_tok": (hud["prefetched_MiB_per_tok"] + hud["inplace_MiB_per_tok"]) * 2 ** 20,
                          "host_link_GBs": (hud["prefetched_MiB_per_tok"] + hud["inplace_MiB_per_tok"]) * 2 ** 20 /
                                           (sum(tok_ms) / n * 1e-3) / 1e9},
            "e2e": {"value": n / t_wall, "unit": "tok/s", "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": L * 256,
                    "wall_s": t_wall}}
    print(json.dumps(line), flush=True)
    for hb in hbufs:
        hb.free()
    return 0


def run_batch(args, local: int) -> int:
    """A batch of B decode tokens through the 48 MoE layers of the cfg3 stack
    (styx_moe_block_batch: per used expert a grouped GEMM on the tensor
    cores).  Step i takes tokens bank[(i * B + j) % 64].  Algorithmic bytes of
    a layer: the union of the experts the B tokens route to (each slab read
    once), the router, the norm, and x read and written; the union sizes come
    from an untimed pass over every phase of the token bank."""
    import ctypes as C
    from math import gcd

    import torch

    from styx_b200 import _lib, ops
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    L, B = args.layers, args.batch
    layers = build_model(local, L)
    blk = ops.MoeBatch(ops.Dims(H, F, E, K_TOP), B, local)
    lib, cx = _lib.lib(), blk.ctx.handle
    bank = torch.from_numpy(token_bank(64)).to(dev)
    x = torch.empty(B, H, dtype=torch.float32, device=dev)
    ids = torch.zeros(L, B * 64, dtype=torch.int32, device=dev)
    wts = torch.zeros(L, B * K_TOP, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    phases = 64 // gcd(64, B)
    sel = [torch.tensor([(p * B + j) % 64 for j in range(B)], device=dev) for p in range(phases)]

    def layers_pass():
        for l in range(L):
            blk.forward(x, layers[l], ids[l], wts[l])

    # union sizes per phase and layer (untimed), from the ids the kernels wrote
    uniq = []
    with torch.cuda.stream(stream):
        for p in range(phases):
            x.copy_(bank[sel[p]])
            layers_pass()
            stream.synchronize()
            got = ids.view(L, B, 64)[:, :, :K_TOP].cpu().numpy()
            uniq.append([len(np.unique(got[l])) for l in range(L)])
    blk.ctx.check_device_error(stream)

    graph = C.c_void_p()
    sp = C.c_void_p(stream.cuda_stream)
    _lib.check(lib.styx_graph_begin(cx, sp))
    with torch.cuda.stream(stream):
        layers_pass()
    _lib.check(lib.styx_graph_end(cx, sp, C.byref(graph)))

    def replay(i):
        with torch.cuda.stream(stream):
            x.copy_(bank[sel[i % phases]])
        _lib.check(lib.styx_graph_launch(cx, graph, sp))

    for i in range(args.warmup):
        replay(i)
    stream.synchronize()
    blk.ctx.check_device_error(stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            replay(i)
        ev1.record(stream)
        stream.synchronize()
    el_ms = ev0.elapsed_time(ev1)
    blk.ctx.check_device_error(stream)
    clocks = clk.summary()
    ms_step = el_ms / args.steps
    value = B * args.steps / (el_ms / 1e3)

    # e2e through the C ABI with host buffers: the batch's tokens up, the
    # hidden states and id blocks down, a ring of pinned buffers
    RING = 4
    hbank = token_bank(64)
    hxs = [ops.HostBuffer(B * H * 4, local) for _ in range(RING)]
    houts = [ops.HostBuffer(B * H * 4 + L * B * 256, local) for _ in range(RING)]
    done = [None] * RING
    xp, idp = C.c_void_p(x.data_ptr()), C.c_void_p(ids.data_ptr())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    e0.record(stream)
    for i in range(args.steps):
        r = i % RING
        if done[r] is not None:
            done[r].synchronize()
        rows = [(i % phases * B + j) % 64 for j in range(B)]
        hxs[r].tensor.view(torch.float32).view(B, H).copy_(torch.from_numpy(hbank[rows]))
        _lib.check(lib.styx_upload(cx, xp, 0, C.c_void_p(hxs[r].ptr), B * H * 4, sp))
        _lib.check(lib.styx_graph_launch(cx, graph, sp))
        _lib.check(lib.styx_download(cx, C.c_void_p(houts[r].ptr), xp, 0, B * H * 4, sp))
        _lib.check(lib.styx_download(cx, C.c_void_p(houts[r].ptr + B * H * 4), idp, 0, L * B * 256, sp))
        ev = torch.cuda.Event()
        ev.record(stream)
        done[r] = ev
    e1.record(stream)
    stream.synchronize()
    t_wall = time.perf_counter() - t_wall
    e2e_val = B * args.steps / (e0.elapsed_time(e1) / 1e3)
    last_x = houts[(args.steps - 1) % RING].tensor[:B * H * 4].view(torch.float32)
    finite = bool(torch.isfinite(last_x).all())

    # algorithmic bytes per layer: the mean over the timed steps' phases
    counts = [0] * phases
    for i in range(args.steps):
        counts[i % phases] += 1
    mean_union = sum(counts[p] * sum(uniq[p]) for p in range(phases)) / (args.steps * L)
    alg = mean_union * (2 * SG + SD) + E * H * 4 + H * 4 + 2 * B * H * 4
    peak, peak_kind = peaks()
    t_layer = ms_step / L * 1e-3
    achieved = alg / t_layer / 1e9
    line = {
        "metric": f"decode tok/s at batch {B} ({'30B-A3B' if SHAPE == 'cfg2' else '235B-A22B (configs[4])'} MoE "
                  f"stack, {'q4_K/q6_K' if QD == Q6_K else 'q4_K'} experts)", "value": value,
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 tensor-core operands (dequantised q4_K/q6_K), f32 accumulate", "data": "synthetic",
        "config": {"workload": f"batch {B}: the {SHAPE} MoE stack ({L} layers, {shape_desc()}) for {B} "
                               f"tokens per step, grouped expert GEMMs (tcgen05)", "global_batch": B,
                   "n_layers": L, "parallelism": "single",
                   "l2": "inputs larger than L2 (every layer's used experts stream from HBM)",
                   "mean_union_experts_per_layer": mean_union},
        "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": B * H * 4,
                "d2h_bytes_per_step": B * H * 4 + L * B * 256, "wall_s": t_wall, "ring": RING,
                "last_hidden_state_finite": finite},
        "gpu_launches": args.steps * 5 * L,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "unit_of_work": "one batched MoE layer (5 kernels); time = step / layers",
                     "alg_bytes": alg, "peak_kind": peak_kind, "us_per_layer": t_layer * 1e6},
        "cpu_baseline": None,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    _lib.check(lib.styx_graph_destroy(cx, graph))
    for hb in hxs + houts:
        hb.free()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="styx", choices=["styx", "reference"])
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--launch", choices=["block", "layers", "chain"], default="block",
                    help="block: one styx_moe_block call per layer (the fastest on B200); layers: every MoE "
                         "layer of a token in one persistent launch (STYX_OPT_MOE_LAYERS 1); chain: one launch "
                         "per layer without the grid-dependency wait, x passed as tagged words (2)")
    ap.add_argument("--shared-device", action="store_true",
                    help="cooperative launches (the library default); without it the bench, which owns its "
                         "GPU, sets STYX_OPT_EXCLUSIVE and the single kernel is a plain launch")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--e2e-steps", type=int, default=0, help="0 = same as --steps")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "cfg3", "cfg4", "batch"],
                    help="decode (default): the whole decode step at the 30B shape (attention + MoE per layer, LM "
                         "head, greedy pick; experts split over the ranks at N > 1); cfg3: the 48 MoE blocks "
                         "alone (replicas at N > 1); cfg4: 6 GiB HBM expert budget, the rest streamed from "
                         "pinned host memory; batch: --batch tokens per step through the cfg3 stack on the "
                         "tensor-core batch path")
    ap.add_argument("--ctx", type=int, default=640,
                    help="decode: cache rows before the token (640: the mean over configs[2]'s 256 decode "
                         "tokens after its 512-token prompt)")
    ap.add_argument("--tokens", type=int, default=1024, help="cfg4: timed decode tokens (configs[3]: 1024)")
    ap.add_argument("--prefetch-min-hit", type=float, default=0.25,
                    help="cfg4: the prefetch stays on while at least this share of prefetched slabs is used (0: always)")
    ap.add_argument("--no-prefetch", action="store_true", help="cfg4: no next-token prefetch")
    ap.add_argument("--batch", type=int, default=8, help="batch: tokens per step (1..64)")
    ap.add_argument("--moe-kernels", type=int, default=0, choices=[0, 1, 2, 3],
                    help="STYX_OPT_MOE_KERNELS: 0 auto, 1 single cooperative kernel, 2 three kernels, 3 cluster form")
    ap.add_argument("--ep-comm", default="fused", choices=["fused", "p2p", "nccl"],
                    help="decode at N > 1: the exchange over NVLink peer memory inside the block's kernel (fused, "
                         "styx_ep_moe_block), as one kernel after it (p2p, styx_ep_combine), or an NCCL all-reduce "
                         "+ styx_moe_combine")
    ap.add_argument("--attn-kernels", type=int, default=0, choices=[0, 1, 2, 3],
                    help="decode: STYX_OPT_ATTN_KERNELS: 0 auto, 1 cooperative kernel, 2 seven kernels, 3 cluster form")
    ap.add_argument("--shape", default="cfg2", choices=["cfg2", "cfg5"],
                    help="cfg3 / batch workloads: the 30B-A3B MoE layer (cfg2, 48 layers) or configs[4]'s "
                         "235B-A22B layer (cfg5: H 4096, F 1536, every matrix q4_K, 94 layers)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.shape != "cfg2":
        if args.workload not in ("cfg3", "batch") or args.impl != "styx":
            ap.error("--shape cfg5 applies to the device arm's --workload cfg3 and batch")
        set_shape(args.shape)
        if args.layers == 48:
            args.layers = N_LAYERS
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.workload == "cfg4":
        return run_streaming(args, local)
    if args.workload == "decode":
        return run_decode(args, local, rank, world)
    if args.workload == "batch":
        return run_batch(args, local)

    import ctypes as C

    import torch

    from styx_b200 import _lib, ops
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device(dev))
        pg = dist

    L = args.layers
    layers = build_model(local, L)
    blk = ops.MoeBlock(ops.Dims(H, F, E, K_TOP), local)
    lib, cx = _lib.lib(), blk.ctx.handle
    bank = torch.from_numpy(token_bank(64)).to(dev)
    x = torch.empty(H, dtype=torch.float32, device=dev)
    ids = torch.zeros(L * 64, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    blk.ctx.set_option(_lib.OPT_MOE_LAYERS, {"block": 0, "layers": 1, "chain": 2}[args.launch])
    blk.ctx.set_option(_lib.OPT_EXCLUSIVE, 0 if args.shared_device else 1)
    blk.ctx.set_option(_lib.OPT_MOE_KERNELS, args.moe_kernels)

    def moe_layers():
        if args.launch != "block":
            blk.forward_layers(x, layers, 0, ids)
        else:
            for layer in range(L):
                blk.forward(x, layers[layer], layer, ids)

    def token(i):
        x.copy_(bank[i % bank.shape[0]])
        moe_layers()

    with torch.cuda.stream(stream):
        token(0)
    stream.synchronize()
    blk.ctx.check_device_error(stream)

    # record one token through the C ABI's graph API
    graph = C.c_void_p()
    sp = C.c_void_p(stream.cuda_stream)
    _lib.check(lib.styx_graph_begin(cx, sp))
    with torch.cuda.stream(stream):
        moe_layers()
    _lib.check(lib.styx_graph_end(cx, sp, C.byref(graph)))

    def replay(i):
        with torch.cuda.stream(stream):
            x.copy_(bank[i % bank.shape[0]])
        _lib.check(lib.styx_graph_launch(cx, graph, sp))

    for i in range(args.warmup):
        replay(i)
    stream.synchronize()
    blk.ctx.check_device_error(stream)
    path = blk.ctx.last_moe_path()
    kernel_path = {1: "single cooperative kernel per MoE block", 2: "three kernels per MoE block",
                   4: "single cooperative kernel running every MoE layer of a token per launch",
                   5: "single cooperative kernel per MoE block, launches chained (x passed as tagged words)",
                   6: "one launch of thread-block clusters per MoE block (a cluster per selected slot)"
                   }.get(path, "unknown")
    launches_per_token = {1: L, 2: 3 * L, 4: -(-L // 80), 5: L, 6: L}.get(path, 0)

    def barrier():
        if pg:
            pg.barrier()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            replay(i)
        ev1.record(stream)
        stream.synchronize()
    barrier()
    el_ms = ev0.elapsed_time(ev1)
    blk.ctx.check_device_error(stream)
    if pg:
        t = torch.tensor([el_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        el_ms = float(t.item())
    clocks = clk.summary()
    ms_step = el_ms / args.steps
    value = world * args.steps / (el_ms / 1e3)

    # e2e: C ABI with host buffers -- every step uploads its own token from a
    # pinned buffer and downloads its hidden state + ids into its own pinned
    # buffer: a ring of RING slots, the host refilling a slot only after the
    # event recorded after that slot's last download has completed
    RING = 4
    n_e2e = args.e2e_steps or args.steps
    hxs = [ops.HostBuffer(H * 4, local) for _ in range(RING)]
    houts = [ops.HostBuffer(H * 4 + L * 256, local) for _ in range(RING)]
    done = [None] * RING
    hbank = token_bank(64)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    xp, idp = C.c_void_p(x.data_ptr()), C.c_void_p(ids.data_ptr())
    barrier()
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    e0.record(stream)
    for i in range(n_e2e):
        r = i % RING
        if done[r] is not None:
            done[r].synchronize()
        hxs[r].tensor.view(torch.float32).copy_(torch.from_numpy(hbank[i % 64]))
        _lib.check(lib.styx_upload(cx, xp, 0, C.c_void_p(hxs[r].ptr), H * 4, sp))
        _lib.check(lib.styx_graph_launch(cx, graph, sp))
        _lib.check(lib.styx_download(cx, C.c_void_p(houts[r].ptr), xp, 0, H * 4, sp))
        _lib.check(lib.styx_download(cx, C.c_void_p(houts[r].ptr + H * 4), idp, 0, L * 256, sp))
        ev = torch.cuda.Event()
        ev.record(stream)
        done[r] = ev
    e1.record(stream)
    stream.synchronize()
    t_wall = time.perf_counter() - t_wall
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if pg:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_val = world * n_e2e / (e2e_ms / 1e3)
    # the last step's result, read on the host
    last_x = houts[(n_e2e - 1) % RING].tensor[:H * 4].view(torch.float32)
    e2e_finite = bool(torch.isfinite(last_x).all())

    peak, peak_kind = peaks()
    t_layer = ms_step / L * 1e-3
    achieved = ALG_BYTES_LAYER / t_layer / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "moe_layer_traffic.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get("dram_bytes_per_layer")
        except Exception:
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            from oracle import oracle as O
            O.build()
            nth = os.cpu_count() or 1
            v, per_layer, reps = time_cpu(args.cpu_seconds, nth)
            cpu = {"value": v, "unit": "tok/s", "cores": nth, "kind": "port",
                   "sample": f"{reps} runs of one 30B-shaped MoE layer (C oracle, OpenMP), "
                             f"{per_layer * 1e3:.2f} ms/layer, scaled to 48 layers"}
        except Exception as e:  # the CPU leg must not sink the GPU number
            cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "port", "sample": f"failed: {e}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8-dp4a/f32 (q4_K,q6_K weights)", "data": "synthetic",
            "config": dict(workload_config(world), kernels=kernel_path,
                           launch="cooperative" if args.shared_device else
                           "plain (STYX_OPT_EXCLUSIVE: the bench owns its GPU)"),
            "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": H * 4,
                    "d2h_bytes_per_step": H * 4 + L * 256, "wall_s": t_wall, "ring": RING,
                    "last_hidden_state_finite": e2e_finite},
            "gpu_launches": args.steps * launches_per_token,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "unit_of_work": "one MoE layer (route + gate/up + down); time per layer = "
                                         "step time / layers",
                         "alg_bytes": ALG_BYTES_LAYER, "peak_kind": peak_kind,
                         "us_per_layer": t_layer * 1e6},
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    _lib.check(lib.styx_graph_destroy(cx, graph))
    for hb in hxs + houts:
        hb.free()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
