#!/usr/bin/env python
"""Leaf evaluations per second for GraphZero's Connect4 GAT (batch 4096 per
GPU), plus batched-search simulations per second, on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1|c0|c2|c3] [--mcts-moves M] [--no-other-configs]

One step = one forward pass over one batch of positions.  Multi-GPU runs
are launched with torchrun (one process per GPU); every rank evaluates its
own shard of positions with the network replicated (weak scaling), the
weights reach every GPU through one NCCL broadcast before timing, and the
reported time is the maximum over ranks.  Prints ONE JSON line on rank 0.
The c1 line also carries, under "configs", the other leaf-evaluation
workloads (c0 TicTacToe fp32, c2 Connect4 ResNet, c3 chess GAT) measured on
the same GPU, each with its roofline and CPU baseline (c3 also with the
batched search on chess positions under "search"), and under "train" the
training step time of the Connect4 GAT and ResNet at batch 64.

--impl reference times the CPU restatement of the same math (the reference's
own network code does not build) on the host cores with all threads; that
arm builds its weights and positions with the oracle's own generator and
never loads the product library.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "oracle")]

import numpy as np  # noqa: E402

# The product package (graphzero_b200, which loads libgraphzero_b200.so) is
# imported only by the product arm; the reference arm runs on the oracle alone.

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAK_TFLOPS = 1590.0
# fp32 CUDA-core peak for the TicTacToe fp32 workload: 148 SMs x 128 fp32
# lanes x 2 FLOP (FMA) x 1.965 GHz (nominal, computed; not measured here).
FP32_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
TICTACTOE, CONNECT4, CHESS = 0, 1, 2
GAT, RESNET = 0, 1
PREC_AUTO, PREC_FP32 = 0, 1
BASE_SEED = 0x6A5A
BOARD_BYTES = {TICTACTOE: 9, CONNECT4: 42, CHESS: 66}

CONFIGS = {
    "c0": dict(index=0, game=TICTACTOE, kind=GAT, batch=256, precision=PREC_FP32, steps=300,
               workload="TicTacToe GAT forward, 4 layers 8x32 heads, fp32, batch 256 per GPU"),
    "c1": dict(index=1, game=CONNECT4, kind=GAT, batch=4096, precision=PREC_AUTO, steps=2000,
               workload="Connect4 GAT leaf evaluation, 6 layers 8x32 heads, 16-bit tensor-core operands "
                        "(fp16 by default), fp32 accumulate, batch 4096 per GPU"),
    "c2": dict(index=2, game=CONNECT4, kind=RESNET, batch=4096, precision=PREC_AUTO, steps=300,
               workload="Connect4 ResNet leaf evaluation, 3x3 stem + 10 residual blocks of 128 channels, "
                        "16-bit tensor-core operands (fp16 by default), fp32 accumulate, batch 4096 per GPU"),
    "c3": dict(index=3, game=CHESS, kind=GAT, batch=8192, precision=PREC_AUTO, steps=100,
               workload="Chess GAT leaf evaluation, 64 nodes x 18 features, queen+knight graph (1856 edges), "
                        "8 layers 8x32 heads, 4672-way policy, 16-bit tensor-core operands (fp16 by default), "
                        "fp32 accumulate, batch 8192 per GPU"),
}


def rank_env() -> tuple[int, int, int]:
    """(rank, world, local_rank) from the torchrun environment."""
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def shard_seed(config_index: int, rank: int) -> int:
    """Per-rank input seed: base + 1000 x config + rank (graphzero_b200.dist)."""
    return BASE_SEED + 1000 * config_index + rank


def pool_batches(cfg: dict) -> int:
    """Distinct batches cycled by the device-timed loop: more board bytes
    than L2, so no batch is read from L2 twice in a row."""
    return max(8, math.ceil(1.05 * L2_BYTES / (cfg["batch"] * BOARD_BYTES[cfg["game"]])))


def config_block(cfg: dict, world: int) -> dict:
    """The workload description; identical in both arms."""
    B = cfg["batch"]
    nb = pool_batches(cfg)
    return {"workload": cfg["workload"], "batch_per_gpu": B, "global_batch": B * world,
            "positions": "uniform random legal playouts (seeded per rank)",
            "weights": "Glorot-uniform from seed, bf16-representable",
            "l2": f"inputs larger than L2: {nb} distinct batches ({nb * B * BOARD_BYTES[cfg['game']] / 2**20:.0f} "
                  f"MiB of boards) cycled on the GPU",
            "parallelism": f"dp{world} (independent shards, one NCCL weight broadcast)"}


def metric_name(cfg: dict) -> str:
    net = {TICTACTOE: "TicTacToe", CONNECT4: "Connect4", CHESS: "Chess"}[cfg["game"]]
    kind = "GAT" if cfg["kind"] == GAT else "ResNet"
    return f"leaf evals/sec ({net} {kind}, b={cfg['batch']})"


def resnet_gemm_flops() -> float:
    """Algorithmic FLOPs per position of the ResNet tower (implicit-GEMM
    convolutions + heads)."""
    conv = 2.0 * 42 * 128 * 128 * 9
    f = 20 * conv + 2.0 * 42 * 128 * 27       # blocks + stem
    f += 2.0 * 42 * 128 * 3                    # 1x1 head convolutions
    f += 2.0 * 84 * 7 + 2.0 * 42 * 128 + 2.0 * 128
    return f


GAT_SHAPES = {TICTACTOE: dict(nodes=9, features=4, layers=4, policy_per_node=1),
              CONNECT4: dict(nodes=42, features=4, layers=6, policy_per_node=1),
              CHESS: dict(nodes=64, features=18, layers=8, policy_per_node=73)}


def gat_gemm_flops(game: int) -> float:
    """Algorithmic GEMM FLOPs per position: projections + head GEMMs."""
    s = GAT_SHAPES[game]
    f = 2.0 * s["nodes"] * (s["features"] * 256 + (s["layers"] - 1) * 256 * 256)
    f += 2.0 * 256 * 64 + 2.0 * 64  # value head
    if game == CONNECT4:
        f += 2.0 * 7 * 256
    else:
        f += 2.0 * s["nodes"] * 256 * s["policy_per_node"]
    return f


def flops_per_position(cfg: dict) -> float:
    return gat_gemm_flops(cfg["game"]) if cfg["kind"] == GAT else resnet_gemm_flops()


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:  # noqa: BLE001
        return FALLBACK_PEAK_TFLOPS, "fallback 1.59 PFLOP/s"


def ncu_traffic(kernel: str, workload: str) -> float | None:
    p = ROOT / "profiles" / "ncu_traffic.json"
    try:
        d = json.loads(p.read_text())
        return float(d[kernel][workload]["dram_bytes_per_launch"])
    except Exception:  # noqa: BLE001
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML on a thread."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.dev = device_index
        self.period = period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # noqa: BLE001
            self.error = repr(e)
        return self

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
                rs = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, rs))
            except Exception as e:  # noqa: BLE001
                self.error = repr(e)
                return
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "error": self.error or "no samples"}
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = [name for b, name in self.REASONS.items() if bits & b and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


def oracle_inputs(cfg: dict, n: int, seed: int, first: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Positions from the oracle's own generator (bit-identical to the
    product's for TicTacToe and Connect4).  Chess has no legal-move generator
    in the oracle: random piece placements of the same record format stand
    in (the forward's cost does not depend on the position)."""
    import oracle

    if cfg["game"] != CHESS:
        return oracle.synth_positions(cfg["game"], n, seed, first)
    rng = np.random.default_rng(seed + first)
    b = np.zeros((n, 66), np.int8)
    for i in range(n):
        sq = rng.choice(64, size=int(rng.integers(2, 33)), replace=False)
        b[i, sq] = rng.choice([-6, -5, -4, -3, -2, -1, 1, 2, 3, 4, 5, 6], size=sq.size)
        b[i, 64] = rng.integers(0, 16)
        b[i, 65] = -1
    return b, rng.choice([-1, 1], size=n).astype(np.int8)


def oracle_weights(cfg: dict) -> np.ndarray:
    import oracle

    seed = shard_seed(cfg["index"], 0)
    return oracle.synth_gat_weights(cfg["game"], seed) if cfg["kind"] == GAT else oracle.synth_res_weights(seed)


def oracle_forward(cfg: dict, w: np.ndarray, threads: int):
    import oracle

    if cfg["kind"] == GAT:
        return lambda b, s: oracle.gat_forward(cfg["game"], w, b, s, threads=threads, native=True)
    return lambda b, s: oracle.resnet_forward(w, b, s, threads=threads, native=True)


def cpu_baseline(cfg: dict, seconds: float = 10.0) -> dict:
    """The oracle (C++ restatement of the same math, AVX2 build) on all host
    cores over a bounded sample of the same workload (inputs and weights
    from the oracle's generator)."""
    import oracle

    threads = oracle.cpu_threads()
    fwd = oracle_forward(cfg, oracle_weights(cfg), threads)
    chunk = 32 * threads
    done, t0, i = 0, time.perf_counter(), 0
    while True:
        boards, side = oracle_inputs(cfg, chunk, shard_seed(cfg["index"], 0) + 77, first=i * chunk)
        fwd(boards, side)
        done += chunk
        i += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 1 << 16:
            break
    return {"value": done / el, "unit": "leaf evals/s", "cores": threads, "kind": "port",
            "sample": f"{done} positions of the same workload in {el:.1f} s (oracle/oracle.cpp, "
                      f"-O3 -march=x86-64-v3, {threads} threads)"}


def reference_arm(args, cfg: dict) -> None:
    """The CPU restatement on the host cores (rank 0 only): the reference's
    own network code does not build.  Uses the oracle alone."""
    rank, _, _ = rank_env()
    if rank != 0:
        return
    import oracle

    threads = oracle.cpu_threads()
    fwd = oracle_forward(cfg, oracle_weights(cfg), threads)
    # size one step so the whole run stays within a couple of minutes
    probe_n = 4 * threads
    b, s = oracle_inputs(cfg, probe_n, 1)
    t0 = time.perf_counter()
    fwd(b, s)
    rate = probe_n / (time.perf_counter() - t0)
    per_step = int(max(threads, min(cfg["batch"], rate * min(2.0, 100.0 / max(1, args.steps + args.warmup)))))
    boards, side = oracle_inputs(cfg, per_step * (args.steps + args.warmup), shard_seed(cfg["index"], 0))
    for k in range(args.warmup):
        sl = slice(k * per_step, (k + 1) * per_step)
        fwd(boards[sl], side[sl])
    t0 = time.perf_counter()
    for k in range(args.warmup, args.warmup + args.steps):
        sl = slice(k * per_step, (k + 1) * per_step)
        fwd(boards[sl], side[sl])
    el = time.perf_counter() - t0
    value = per_step * args.steps / el
    sample = (f"{per_step} positions per step of the same workload (inputs and weights from the oracle's "
              f"generator); the reference's own network code does not build, so its CPU restatement "
              f"(oracle/oracle.cpp) runs")
    line = {
        "impl": "reference", "metric": metric_name(cfg), "value": value, "unit": "leaf evals/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(cfg, args.gpus),
        "cpu_baseline": {"value": value, "unit": "leaf evals/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "leaf evals/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def mcts_bench(net, device, game: int, trees: int, sims: int, leaves: int, moves: int, seed: int) -> dict:
    """Self-play throughput: `trees` games, `sims` simulations per move."""
    import torch

    m = gz.Mcts(game, trees, leaves, c_puct=1.5, virtual_loss=3, node_capacity=(sims + 1) * 3,
                dirichlet_alpha=1.0, dirichlet_eps=0.25, seed=seed, device=device)
    s = gz.game_shape(game)
    boards = torch.zeros((trees, s.nodes), dtype=torch.int8, device=f"cuda:{device}")
    side = torch.ones(trees, dtype=torch.int8, device=f"cuda:{device}")
    acts = torch.zeros(trees, dtype=torch.int32, device=f"cuda:{device}")
    m.reset_roots(boards, side)
    stream = torch.cuda.current_stream()

    def one_move():
        m.run(net, sims, stream)
        m.choose(15, acts, stream)
        m.play(acts, sims + 1, None, stream)

    one_move()  # warm-up
    torch.cuda.synchronize()
    gzd.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(moves):
        one_move()
    ev1.record(stream)
    torch.cuda.synchronize()
    el = ev0.elapsed_time(ev1) / 1e3
    el = gzd.max_over_ranks(el, device=f"cuda:{device}")
    m.check()
    waves = math.ceil(sims / leaves)
    world = gzd.rank_info().world
    out = {"sims_per_s": trees * waves * leaves * moves * world / el,
           "positions_per_s": trees * moves * world / el,
           "sims_per_s_per_gpu": trees * waves * leaves * moves / el,
           "positions_per_s_per_gpu": trees * moves / el,
           "config": f"{trees} games/GPU x {sims} sims/move, leaf batch {trees * leaves}, c_puct 1.5, "
                     f"virtual loss 3, Dirichlet(1.0, 0.25), {moves} timed moves",
           # per move: a selection, per wave a network pass and a backup fused
           # with the next wave's selection (the last backup alone), choose, play
           "gpu_launches_per_move": 2 * waves + 3}

    # Whole games through the self-play driver: every tree starts from the
    # empty board and plays until `trees` games have ended; examples are the
    # TrainingExample records the driver writes.
    m.reset_roots(boards, side)
    sp = gz.SelfPlay(m, max_examples=trees * s.nodes * 2)
    torch.cuda.synchronize()
    gzd.barrier()
    t0 = time.perf_counter()
    sp.run(net, trees, sims, 15, stream)
    el = gzd.max_over_ranks(time.perf_counter() - t0, device=f"cuda:{device}")
    ex, games = sp.take()
    m.check()
    out["selfplay"] = {"games_per_s": games * world / el, "examples_per_s": ex.size * world / el,
                       "games": games, "examples": int(ex.size), "seconds": el,
                       "call": f"gz_selfplay_run until {trees} games/GPU ended, from empty boards, "
                               f"{sims} sims/move, temperature moves 15"}
    sp.close()
    return out


def _import_product():
    """The product package and its multi-GPU helpers (loads libgraphzero_b200.so)."""
    global gz, gzd
    import graphzero_b200 as gz
    from graphzero_b200 import dist as gzd


def device_timed(cfg: dict, net, dev: int, rank: int, steps: int, warmup: int, stream) -> dict:
    """Device-timed forward passes over a pool of distinct batches (more
    board bytes than L2) resident in HBM: total time and the mean per-launch
    time from CUDA events on the launching stream, both max over ranks, and
    the SM clocks sampled during the timed region."""
    import torch

    game, B = cfg["game"], cfg["batch"]
    s = gz.game_shape(game)
    seed = shard_seed(cfg["index"], rank)
    base_n = 16384 if game == CHESS else 65536  # chess playouts are slow to generate
    base_b, base_s = gz.synth_positions(game, base_n, seed=seed)
    n_batches = pool_batches(cfg)
    g = torch.Generator(device="cpu").manual_seed(seed)
    idx = torch.randint(0, base_n, (n_batches * B,), generator=g).to(f"cuda:{dev}")
    pool_b = torch.from_numpy(base_b).to(f"cuda:{dev}")[idx].contiguous()
    pool_s = torch.from_numpy(base_s).to(f"cuda:{dev}")[idx].contiguous()
    pi = torch.empty((B, s.actions), device=f"cuda:{dev}")
    v = torch.empty(B, device=f"cuda:{dev}")

    def step(k):
        j = k % n_batches
        net.predict_batch(pool_b[j * B].data_ptr(), pool_s[j * B].data_ptr(), B, pi, v, stream)

    for k in range(warmup):
        step(k)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gzd.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev) as clocks:
        t_begin.record(stream)
        for k in range(steps):
            starts[k].record(stream)
            step(warmup + k)
            ends[k].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    gzd.barrier()
    net.check()
    elapsed = t_begin.elapsed_time(t_end) / 1e3
    kernel_s = statistics.mean(a.elapsed_time(b) for a, b in zip(starts, ends)) / 1e3
    del pool_b, pool_s
    return {"elapsed": gzd.max_over_ranks(elapsed, device=f"cuda:{dev}"),
            "kernel_s": gzd.max_over_ranks(kernel_s, device=f"cuda:{dev}"),
            "base": (base_b, base_s), "clocks": clocks.summary()}


def roofline(cfg: dict, kernel_name: str, kernel_s: float) -> dict:
    """Achieved GEMM FLOP/s of one launch against the measured bf16 tensor
    peak (the fp16 rate is the same), or the nominal fp32 CUDA-core peak for
    the fp32 SIMT kernel."""
    B = cfg["batch"]
    flops = flops_per_position(cfg) * B
    achieved = flops / kernel_s / 1e12
    if kernel_name.endswith("fp32"):
        peak, src, bound = FP32_PEAK_TFLOPS, "nominal fp32 CUDA-core peak (148 SMs x 128 lanes x 2 x 1.965 GHz)", "fp32"
    else:
        (peak, src), bound = measured_peak(), "tensor"
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "traffic": ncu_traffic(kernel_name, f"batch{B}"), "kernel": kernel_name, "kernel_ms": kernel_s * 1e3,
            "flops_per_launch": flops, "peak_source": src}


def chess_search_bench(net, dev: int, stream, trees: int = 1024, leaves: int = 4, sims: int = 200) -> dict:
    """Batched PUCT on chess positions with the chess net: `trees` roots made
    by the on-device position generator, `sims` simulations each from the
    roots (select, evaluate, backup), timed with CUDA events."""
    import torch

    m = gz.Mcts(CHESS, trees, leaves, c_puct=1.5, virtual_loss=3, node_capacity=sims + 8, dirichlet_alpha=0.3,
                dirichlet_eps=0.25, seed=0xC35, device=dev)
    boards, side = gz.synth_positions_device(CHESS, trees, seed=0xC36, device=dev, stream=stream)
    for _ in range(2):  # warm-up, then the timed search from fresh roots
        m.reset_roots(boards, side, stream)
        m.run(net, 3 * leaves if _ == 0 else sims, stream)
    torch.cuda.synchronize()
    m.reset_roots(boards, side, stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    m.run(net, sims, stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    el = ev0.elapsed_time(ev1) / 1e3
    m.check()
    nodes, edges = m.tree_sizes()
    waves = math.ceil(sims / leaves)
    m.close()
    return {"sims_per_s": trees * waves * leaves / el, "ms_per_wave": el / waves * 1e3,
            "config": f"{trees} chess roots (on-device random playouts) x {sims} sims, leaf batch {trees * leaves}, "
                      f"c_puct 1.5, virtual loss 3, Dirichlet(0.3, 0.25), the c3 net",
            "nodes_per_tree": float(nodes.mean()), "edges_per_node": float(edges.sum() / max(1, nodes.sum()))}


def other_config(name: str, dev: int, stream, with_cpu: bool) -> dict:
    """One more leaf-evaluation workload on this GPU (one rank): value,
    roofline and a bounded CPU baseline sample."""
    cfg = CONFIGS[name]
    net = gz.Net(cfg["game"], cfg["kind"], device=dev, precision=cfg["precision"], max_batch=cfg["batch"])
    net.load_weights(gz.synth_weights(cfg["game"], cfg["kind"], seed=shard_seed(cfg["index"], 0)))
    r = device_timed(cfg, net, dev, 0, cfg["steps"], 5, stream)
    out = {"metric": metric_name(cfg), "value": cfg["batch"] * cfg["steps"] / r["elapsed"], "unit": "leaf evals/s",
           "steps": cfg["steps"], "warmup": 5, "ms_per_step": r["elapsed"] / cfg["steps"] * 1e3,
           "config": config_block(cfg, 1), "roofline": roofline(cfg, net.kernel_name, r["kernel_s"]),
           "clocks": r["clocks"], "gpu_launches": cfg["steps"]}
    if cfg["game"] == CHESS:
        out["search"] = chess_search_bench(net, dev, stream)
    net.close()
    if with_cpu:
        out["cpu_baseline"] = cpu_baseline(cfg, seconds=8.0)
    return out


def train_bench(dev: int, stream, steps: int = 20, warmup: int = 3) -> dict:
    """Training steps (gz_net_train_step: loss, backward, Adam, repack) at the
    reference's batch of 64 (gat.cu:716) on device-resident synthetic
    batches, for the Connect4 GAT and ResNet, timed with CUDA events."""
    import torch

    out = {}
    for name, kind in (("connect4_gat", GAT), ("connect4_resnet", RESNET)):
        B = 64
        net = gz.Net(CONNECT4, kind, device=dev, max_batch=B)
        net.load_weights(gz.synth_weights(CONNECT4, kind, seed=0x7A1))
        boards, side = gz.synth_positions(CONNECT4, B, seed=0x7A2)
        rng = np.random.default_rng(0x7A3)
        pi = rng.dirichlet(np.full(7, 0.5), size=B).astype(np.float32)
        v = rng.uniform(-1, 1, B).astype(np.float32)
        d = [torch.from_numpy(np.ascontiguousarray(x)).cuda(dev) for x in (boards, side, pi, v)]
        cfg = gz.train_config()
        for _ in range(warmup):
            net.train_step(*d, B, cfg, stream=stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            net.train_step(*d, B, cfg, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        out[name] = {"batch": B, "steps": steps, "ms_per_step": ms, "positions_per_s": B / ms * 1e3,
                     "dtype": "f32", "optimizer": "Adam (lr 1e-3, weight decay 1e-4)"}
        net.close()
    return out


def ours(args, cfg: dict) -> None:
    import torch

    _import_product()
    info = gzd.rank_info()
    dev = info.local_rank
    torch.cuda.set_device(dev)
    multi = gzd.init_process_group("nccl", info)
    game, B = cfg["game"], cfg["batch"]
    s = gz.game_shape(game)
    stream = torch.cuda.current_stream()

    # ---- network, weights from rank 0 over NCCL ----
    net = gz.Net(game, cfg["kind"], device=dev, precision=cfg["precision"], max_batch=B)
    w = gz.synth_weights(game, cfg["kind"], seed=shard_seed(cfg["index"], 0))
    comm = None
    assert net.weight_count() == w.size
    if multi:
        if info.rank == 0:
            net.load_weights(w)
        uid = gzd.share_bytes(gz.nccl_unique_id() if info.rank == 0 else None)
        comm = gz.nccl_comm_init(uid, info.world, info.rank, dev)
        net.broadcast(comm, 0, stream)
        torch.cuda.synchronize()
        assert (net.save_weights() == w).all(), "weight broadcast mismatch"
    else:
        net.load_weights(w)

    # ---- timed region (device time, max over ranks) ----
    r = device_timed(cfg, net, dev, info.rank, args.steps, args.warmup, stream)
    elapsed, kernel_s = r["elapsed"], r["kernel_s"]
    base_b, base_s = r["base"]
    base_n = base_s.shape[0]
    value = B * args.steps * info.world / elapsed

    # ---- end to end through the host-buffer call ----
    # Inputs and outputs live in page-locked host memory (a serving loop
    # keeps such pools); every step copies its batch in and its results out.
    e2e_steps = max(3, min(args.steps, 200))
    nb = e2e_steps + 2
    host_b = torch.empty((nb, B, s.board_bytes), dtype=torch.int8, pin_memory=True).numpy()
    host_s = torch.empty((nb, B), dtype=torch.int8, pin_memory=True).numpy()
    for k in range(nb):
        host_b[k] = base_b[(k * B) % base_n:(k * B) % base_n + B]
        host_s[k] = base_s[(k * B) % base_n:(k * B) % base_n + B]
    out_pi = torch.empty((B, s.actions), dtype=torch.float32, pin_memory=True).numpy()
    out_v = torch.empty((B,), dtype=torch.float32, pin_memory=True).numpy()
    for k in range(2):
        net.predict_host(host_b[k], host_s[k], out=(out_pi, out_v))
    gzd.barrier()
    t0 = time.perf_counter()
    for k in range(e2e_steps):
        net.predict_host(host_b[k + 2], host_s[k + 2], out=(out_pi, out_v))
    e2e_el = gzd.max_over_ranks(time.perf_counter() - t0, device=f"cuda:{dev}")
    e2e = {"value": B * e2e_steps * info.world / e2e_el, "unit": "leaf evals/s",
           "h2d_bytes_per_step": B * (s.board_bytes + 1), "d2h_bytes_per_step": B * (s.actions + 1) * 4,
           "steps": e2e_steps,
           "call": ("gz_net_predict_host (page-locked host buffers, synchronise per step; Connect4: the forward "
                    "kernel reads the boards and writes pi and v through the buffers' mapped addresses; chess: "
                    "H2D, forward and D2H in four overlapped pieces)")}

    # ---- batched search throughput (secondary metric) ----
    mcts = None
    if game == CONNECT4 and cfg["kind"] == GAT and args.mcts_moves > 0:
        mcts = mcts_bench(net, dev, game, trees=1024, sims=800, leaves=4, moves=args.mcts_moves,
                          seed=shard_seed(cfg["index"], info.rank))

    if comm is not None:
        gz.nccl_comm_destroy(comm)
    kernel_name = net.kernel_name
    net.close()
    if info.rank == 0:
        line = {
            "metric": metric_name(cfg),
            "value": value, "unit": "leaf evals/s", "n_gpus": info.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": kernel_name.rsplit("_", 1)[-1].replace("fp", "f"),
            "data": "synthetic",
            "config": config_block(cfg, info.world),
            "e2e": e2e,
            "roofline": roofline(cfg, kernel_name, kernel_s),
            "clocks": r["clocks"],
            "gpu_launches": args.steps,
        }
        if mcts:
            line["mcts"] = mcts
        if info.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg)
        if info.world == 1 and args.config == "c1" and not args.no_other_configs:
            line["configs"] = {name: other_config(name, dev, stream, not args.no_cpu_baseline)
                               for name in ("c0", "c2", "c3")}
            line["train"] = train_bench(dev, stream)
        print(json.dumps(line), flush=True)
    gzd.barrier()
    if multi:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c1")
    ap.add_argument("--mcts-moves", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        reference_arm(args, cfg)
    else:
        ours(args, cfg)


if __name__ == "__main__":
    main()
