#!/usr/bin/env python
"""Leaf evaluations per second for GraphZero's Connect4 GAT (batch 4096 per
GPU), plus batched-search simulations per second, on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1|c0|c2|c3] [--mcts-moves M]

One step = one forward pass over one batch of positions.  Multi-GPU runs
are launched with torchrun (one process per GPU); every rank evaluates its
own shard of positions with the network replicated (weak scaling), the
weights reach every GPU through one NCCL broadcast before timing, and the
reported time is the maximum over ranks.  Prints ONE JSON line on rank 0.

--impl reference times the CPU restatement of the same math (the reference's
own network code does not build) on the host cores with all threads.
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

import graphzero_b200 as gz  # noqa: E402
from graphzero_b200 import dist as gzd  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAK_TFLOPS = 1590.0

CONFIGS = {
    "c0": dict(index=0, game=gz.TICTACTOE, kind=gz.GAT, batch=256, precision=gz.PREC_FP32, dtype="f32",
               workload="TicTacToe GAT forward, 4 layers 8x32 heads, fp32, batch 256 per GPU"),
    "c1": dict(index=1, game=gz.CONNECT4, kind=gz.GAT, batch=4096, precision=gz.PREC_AUTO, dtype="bf16",
               workload="Connect4 GAT leaf evaluation, 6 layers 8x32 heads, bf16 operands fp32 accumulate, "
                        "batch 4096 per GPU"),
    "c2": dict(index=2, game=gz.CONNECT4, kind=gz.RESNET, batch=4096, precision=gz.PREC_AUTO, dtype="bf16",
               workload="Connect4 ResNet leaf evaluation, 3x3 stem + 10 residual blocks of 128 channels, "
                        "bf16 operands fp32 accumulate, batch 4096 per GPU"),
    "c3": dict(index=3, game=gz.CHESS, kind=gz.GAT, batch=8192, precision=gz.PREC_AUTO, dtype="bf16",
               workload="Chess GAT leaf evaluation, 64 nodes x 18 features, queen+knight graph (1856 edges), "
                        "8 layers 8x32 heads, 4672-way policy, bf16 operands fp32 accumulate, batch 8192 per GPU"),
}


def metric_name(cfg: dict) -> str:
    net = {gz.TICTACTOE: "TicTacToe", gz.CONNECT4: "Connect4", gz.CHESS: "Chess"}[cfg["game"]]
    kind = "GAT" if cfg["kind"] == gz.GAT else "ResNet"
    return f"leaf evals/sec ({net} {kind}, b={cfg['batch']})"


def resnet_gemm_flops() -> float:
    """Algorithmic FLOPs per position of the ResNet tower (implicit-GEMM
    convolutions + heads)."""
    conv = 2.0 * 42 * 128 * 128 * 9
    f = 20 * conv + 2.0 * 42 * 128 * 27       # blocks + stem
    f += 2.0 * 42 * 128 * 3                    # 1x1 head convolutions
    f += 2.0 * 84 * 7 + 2.0 * 42 * 128 + 2.0 * 128
    return f


def gat_gemm_flops(game: int) -> float:
    """Algorithmic GEMM FLOPs per position: projections + head GEMMs."""
    s = gz.game_shape(game)
    f = 2.0 * s.nodes * (s.features * 256 + (s.layers - 1) * 256 * 256)
    f += 2.0 * 256 * 64 + 2.0 * 64  # value head
    if game == gz.CONNECT4:
        f += 2.0 * 7 * 256
    else:
        f += 2.0 * s.nodes * 256 * s.policy_per_node
    return f


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


def cpu_baseline(cfg: dict, w: np.ndarray, seconds: float = 10.0) -> dict:
    """The oracle (C++ restatement of the same math, AVX2 build) on all host
    cores over a bounded sample of the same workload."""
    import oracle

    threads = oracle.cpu_threads()
    game = cfg["game"]
    chunk = 32 * threads
    done, t0, i = 0, time.perf_counter(), 0
    while True:
        boards, side = gz.synth_positions(game, chunk, seed=gzd.shard_seed(cfg["index"], 0) + 77, first=i * chunk)
        if cfg["kind"] == gz.GAT:
            oracle.gat_forward(game, w, boards, side, threads=threads, native=True)
        else:
            oracle.resnet_forward(w, boards, side, threads=threads, native=True)
        done += chunk
        i += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 1 << 16:
            break
    return {"value": done / el, "unit": "leaf evals/s", "cores": threads, "kind": "port",
            "sample": f"{done} positions of the same workload in {el:.1f} s (oracle/oracle.cpp, "
                      f"-O3 -march=x86-64-v3, {threads} threads)"}


def reference_arm(args, cfg: dict) -> None:
    info = gzd.rank_info()
    if info.rank != 0:
        return
    import oracle

    threads = oracle.cpu_threads()
    game = cfg["game"]
    w = gz.synth_weights(game, cfg["kind"], seed=gzd.shard_seed(cfg["index"], 0))
    fwd = (lambda b, s: oracle.gat_forward(game, w, b, s, threads=threads, native=True)) if cfg["kind"] == gz.GAT \
        else (lambda b, s: oracle.resnet_forward(w, b, s, threads=threads, native=True))
    # size one step so the whole run stays within a couple of minutes
    probe_n = 4 * threads
    b, s = gz.synth_positions(game, probe_n, seed=1)
    t0 = time.perf_counter()
    fwd(b, s)
    rate = probe_n / (time.perf_counter() - t0)
    per_step = int(max(threads, min(cfg["batch"], rate * min(2.0, 100.0 / max(1, args.steps + args.warmup)))))
    boards, side = gz.synth_positions(game, per_step * (args.steps + args.warmup),
                                      seed=gzd.shard_seed(cfg["index"], 0))
    for k in range(args.warmup):
        sl = slice(k * per_step, (k + 1) * per_step)
        fwd(boards[sl], side[sl])
    t0 = time.perf_counter()
    for k in range(args.warmup, args.warmup + args.steps):
        sl = slice(k * per_step, (k + 1) * per_step)
        fwd(boards[sl], side[sl])
    el = time.perf_counter() - t0
    value = per_step * args.steps / el
    line = {
        "impl": "reference", "metric": metric_name(cfg), "value": value, "unit": "leaf evals/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["workload"], "batch_per_gpu": cfg["batch"],
                   "sample_per_step": per_step},
        "cpu_baseline": {"value": value, "unit": "leaf evals/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} positions per step of the same workload; the reference's own "
                                   f"network code does not build, so its CPU restatement (oracle/oracle.cpp) runs"},
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
           "config": f"{trees} games/GPU x {sims} sims/move, leaf batch {trees * leaves}, c_puct 1.5, "
                     f"virtual loss 3, Dirichlet(1.0, 0.25), {moves} timed moves",
           "gpu_launches_per_move": 3 * waves + 2}

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


def ours(args, cfg: dict) -> None:
    import torch

    info = gzd.rank_info()
    dev = info.local_rank
    torch.cuda.set_device(dev)
    multi = gzd.init_process_group("nccl", info)
    game, B = cfg["game"], cfg["batch"]
    s = gz.game_shape(game)
    stream = torch.cuda.current_stream()

    # ---- network, weights from rank 0 over NCCL ----
    net = gz.Net(game, cfg["kind"], device=dev, precision=cfg["precision"], max_batch=B)
    w = gz.synth_weights(game, cfg["kind"], seed=gzd.shard_seed(cfg["index"], 0))
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

    # ---- inputs: a pool of distinct batches larger than L2, resident in HBM ----
    seed = gzd.shard_seed(cfg["index"], info.rank)
    base_n = 16384 if game == gz.CHESS else 65536  # chess playouts are slow to generate
    base_b, base_s = gz.synth_positions(game, base_n, seed=seed)
    n_batches = max(8, math.ceil(1.05 * L2_BYTES / (B * s.board_bytes)))
    g = torch.Generator(device="cpu").manual_seed(seed)
    idx = torch.randint(0, base_n, (n_batches * B,), generator=g).to(f"cuda:{dev}")
    pool_b = torch.from_numpy(base_b).to(f"cuda:{dev}")[idx].contiguous()
    pool_s = torch.from_numpy(base_s).to(f"cuda:{dev}")[idx].contiguous()
    pi = torch.empty((B, s.actions), device=f"cuda:{dev}")
    v = torch.empty(B, device=f"cuda:{dev}")

    def step(k):
        j = k % n_batches
        net.predict_batch(pool_b[j * B].data_ptr(), pool_s[j * B].data_ptr(), B, pi, v, stream)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()

    # ---- timed region (device time, max over ranks) ----
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gzd.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev) as clocks:
        t_begin.record(stream)
        for k in range(args.steps):
            starts[k].record(stream)
            step(args.warmup + k)
            ends[k].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    gzd.barrier()
    elapsed = t_begin.elapsed_time(t_end) / 1e3
    kernel_s = statistics.mean(a.elapsed_time(b) for a, b in zip(starts, ends)) / 1e3
    elapsed = gzd.max_over_ranks(elapsed, device=f"cuda:{dev}")
    kernel_s = gzd.max_over_ranks(kernel_s, device=f"cuda:{dev}")
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
           "call": "gz_net_predict_host (page-locked host buffers: H2D, forward, D2H, synchronise per step)"}

    # ---- batched search throughput (secondary metric) ----
    mcts = None
    if game == gz.CONNECT4 and cfg["kind"] == gz.GAT and args.mcts_moves > 0:
        mcts = mcts_bench(net, dev, game, trees=1024, sims=800, leaves=4, moves=args.mcts_moves,
                          seed=seed)

    if comm is not None:
        gz.nccl_comm_destroy(comm)
    if info.rank == 0:
        flops = (gat_gemm_flops(game) if cfg["kind"] == gz.GAT else resnet_gemm_flops()) * B
        peak, peak_src = measured_peak()
        achieved = flops / kernel_s / 1e12
        kernel_name = net.kernel_name
        traffic = ncu_traffic(kernel_name, f"batch{B}")
        line = {
            "metric": metric_name(cfg),
            "value": value, "unit": "leaf evals/s", "n_gpus": info.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": kernel_name.rsplit("_", 1)[-1].replace("fp", "f"),
            "data": "synthetic",
            "config": {"workload": cfg["workload"], "batch_per_gpu": B, "global_batch": B * info.world,
                       "positions": "uniform random legal playouts (seeded per rank)",
                       "weights": "Glorot-uniform from seed, bf16-representable",
                       "l2": f"inputs larger than L2: {n_batches} distinct batches "
                             f"({n_batches * B * s.board_bytes / 2**20:.0f} MiB of boards) cycled",
                       "parallelism": f"dp{info.world} (independent shards, one NCCL weight broadcast)"},
            "e2e": e2e,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": kernel_name, "kernel_ms": kernel_s * 1e3,
                         "flops_per_launch": flops, "peak_source": peak_src},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps,
        }
        if mcts:
            line["mcts"] = mcts
        if info.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, w)
        print(json.dumps(line), flush=True)
    gzd.barrier()
    net.close()
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
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        reference_arm(args, cfg)
    else:
        ours(args, cfg)


if __name__ == "__main__":
    main()
