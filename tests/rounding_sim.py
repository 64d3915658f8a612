"""CPU rounding simulation of the tensor-core GAT kernels (test infrastructure).

The Connect4 and chess tensor-core kernels compute the GAT forward of the
oracle with their operands rounded at fixed points.  This module repeats the
forward in float64 with exactly those roundings and nothing else, so the
error it shows against the oracle is the error the operand formats allow --
the floor any kernel with these operand types reaches.  The GPU tests take
their tolerances from it (max over the same inputs, times a margin).

Rounding points, per layer l (activations carried times log2(e) from the
first ELU on, so the softmax works in base 2):
  X_l        the projection's A operand: bf16 or fp16, stochastically
             rounded ("sr") or rounded to nearest ("rn"); layer 0's one-hot
             features are exact
  W_l        the B operand: stochastically rounded in the operand format
             by a hash of each weight's index in the blob (`round_weights`,
             the pack kernels' rule, bit for bit); `wround="rn"` models the
             earlier kernels, which rounded weights to nearest
  W_l a      attention-score weights as a high part plus the rounding of the
             remainder (two MMA columns) -- fp32-level accurate
  Wh         the gather's B operand: fp16, rounded to nearest
  e_ij       softmax numerators exp2(lrelu(s_i + t_j) - max): fp16, rounded
             to nearest; z sums these fp16 values
  X_last     the last layer's activations, the pooling input: fp16 rounded
             to nearest (`last="fp16"`) or stochastically (`"fp16sr"`), or
             kept in fp32 (`"fp32"`)
Sums (MMA accumulators, pooling, heads) are exact here; fp32 accumulation
adds errors far below the operand roundings.

Reference semantics: networks/gat/gat.cu:836-870 (layer), 916-948 (heads),
the standard GAT the reference's kernels never completed.
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634
LN2 = 0.6931471805599453


def round_bf16(x: np.ndarray, mode: str, rng: np.random.Generator | None = None) -> np.ndarray:
    """bf16 rounding of float32 values: "rn" (nearest even) or "sr"
    (stochastic: random 16 bits added below the kept mantissa, then
    truncated -- what cvt.rs does)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    if mode == "rn":
        u = u + 0x7FFF + ((u >> 16) & 1)
    else:
        u = u + rng.integers(0, 1 << 16, size=u.shape, dtype=np.uint64)
    return (u & 0xFFFF0000).astype(np.uint32).view(np.float32).astype(np.float64)


def round_fp16(x: np.ndarray, mode: str, rng: np.random.Generator | None = None) -> np.ndarray:
    """fp16 rounding of float32 values, "rn" or "sr" (the two neighbours
    chosen with probability proportional to closeness)."""
    x32 = np.asarray(x, dtype=np.float32)
    h = x32.astype(np.float16)
    if mode == "rn":
        return h.astype(np.float64)
    xd = x32.astype(np.float64)
    hd = h.astype(np.float64)
    d = xd - hd
    other = np.nextafter(h, np.where(d > 0, np.float16(np.inf), np.float16(-np.inf)).astype(np.float16))
    od = other.astype(np.float64)
    gap = np.abs(od - hd)
    with np.errstate(invalid="ignore", divide="ignore"):
        p = np.where(gap > 0, np.abs(d) / gap, 0.0)
    take = rng.random(size=xd.shape) < p
    return np.where(take & (d != 0), od, hd)


def mix32(i: np.ndarray) -> np.ndarray:
    """The "lowbias32" integer hash (Chris Wellons), on uint32 arrays."""
    x = np.asarray(i, dtype=np.uint32).copy()
    x ^= x >> np.uint32(16)
    x *= np.uint32(0x7FEB352D)
    x ^= x >> np.uint32(15)
    x *= np.uint32(0x846CA68B)
    x ^= x >> np.uint32(16)
    return x


def _bits16(x32: np.ndarray, fmt: str) -> np.ndarray:
    if fmt == "fp16":
        return x32.astype(np.float16).view(np.uint16)
    u = x32.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def _value16(b: np.ndarray, fmt: str) -> np.ndarray:
    if fmt == "fp16":
        return b.view(np.float16).astype(np.float64)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32).astype(np.float64)


def round_weights(x: np.ndarray, fmt: str, index: np.ndarray) -> np.ndarray:
    """The pack kernels' weight rounding (graphzero_b200/csrc/gz_round.h):
    n = x to nearest in `fmt`; where n != x the other neighbour o replaces it
    when |x - n| 2^32 > mix32(index) |o - n|, i.e. with probability
    |x - n| / |o - n|.  `index` is each weight's offset in the blob."""
    if fmt == "exact":
        return np.asarray(x, dtype=np.float64)
    x32 = np.ascontiguousarray(x, dtype=np.float32)
    nb = _bits16(x32, fmt)
    n = _value16(nb, fmt)
    xd = x32.astype(np.float64)
    up = xd > n
    zero = (nb & 0x7FFF) == 0
    away = up != ((nb & 0x8000) != 0)
    ob = np.where(zero, np.where(up, 0x0001, 0x8001),
                  np.where(away, nb.astype(np.int32) + 1, nb.astype(np.int32) - 1)).astype(np.uint16)
    o = _value16(ob, fmt)
    with np.errstate(invalid="ignore"):
        take = (np.abs(xd - n) * 4294967296.0 > mix32(np.broadcast_to(index, x32.shape)).astype(np.float64) * np.abs(o - n))
    keep = (n == xd) | ~np.isfinite(n)
    return np.where(keep | ~take, n, o)


def round_op(x: np.ndarray, fmt: str, mode: str, rng=None) -> np.ndarray:
    if fmt == "exact":
        return np.asarray(x, dtype=np.float64)
    if fmt == "bf16":
        return round_bf16(x, mode, rng)
    return round_fp16(x, mode, rng)


def _views(game: int, shape, w: np.ndarray, offsets: dict | None = None) -> dict:
    """Named float64 views of a GAT weight blob; `offsets`, when given, gets
    each tensor's blob index array (same shape)."""
    o, p = {}, 0
    P = shape.policy_per_node
    specs = [(k, sh) for l in range(shape.layers)
             for k, sh in ((f"W{l}", (shape.features if l == 0 else 256, 256)), (f"b{l}", (256,)), (f"a{l}", (8, 2, 32)))]
    specs += [("w_pi", (256, P)), ("b_pi", (P,)), ("W_v1", (256, 64)), ("b_v1", (64,)), ("w_v2", (64,)), ("b_v2", (1,))]
    for k, sh in specs:
        m = int(np.prod(sh))
        o[k] = w[p:p + m].reshape(sh).astype(np.float64)
        if offsets is not None:
            offsets[k] = (p + np.arange(m, dtype=np.int64)).reshape(sh)
        p += m
    return o


def gat_forward_rounded(game: int, shape, features: np.ndarray, rowptr: np.ndarray, col: np.ndarray,
                        w: np.ndarray, op: str = "bf16", act: str = "sr", gather: str = "fp16",
                        last: str = "fp16", seed: int = 0, wround: str = "sr") -> tuple[np.ndarray, np.ndarray]:
    """The GAT forward with the tensor-core kernels' roundings.

    features: [B][N][F] one-hot node features (exact).  op: operand format of
    the projection ("bf16", "fp16" or "exact"); act: "sr" or "rn" for the
    activations written as the next projection's operand; gather: format of
    the softmax numerators and Wh in the gather ("fp16" or "exact"); last:
    "fp16" or "fp32" pooling input; wround: the weights' rounding, "sr" (the
    pack kernels' hashed stochastic rounding) or "rn".  Returns (pi [B][A],
    v [B])."""
    rng = np.random.default_rng(seed)
    idx = {}
    o = _views(game, shape, w, idx)

    def wr(k):
        if wround == "rn" or op == "exact":
            return round_op(o[k].astype(np.float32), op, "rn")
        return round_weights(o[k].astype(np.float32), op, idx[k])

    B, N, _ = features.shape
    deg = np.diff(rowptr)
    src = np.repeat(np.arange(N), deg)
    dst = col.astype(np.int64)
    adj = np.zeros((N, N), bool)
    adj[src, dst] = True
    X = features.astype(np.float64)
    g_round = (lambda x: round_fp16(x, "rn")) if gather == "fp16" else (lambda x: np.asarray(x, np.float64))
    for l in range(shape.layers):
        Wl = o[f"W{l}"]
        Wr = wr(f"W{l}")
        Wa = np.einsum("khf,hvf->khv", Wl.reshape(-1, 8, 32), o[f"a{l}"])  # [K][8][2]
        if l == 0:
            Wa = Wa * LOG2E
        Wa32 = Wa.astype(np.float32)
        hi = round_op(Wa32, op, "rn")
        lo = round_op((Wa32.astype(np.float64) - hi).astype(np.float32), op, "rn")
        Xr = X if l == 0 else round_op(X.astype(np.float32), op, act, rng)
        Wh = Xr @ Wr                                        # [B][N][256]
        S = np.einsum("bnk,khv->bnhv", Xr, hi + lo)         # [B][N][8][2]
        x = S[:, :, None, :, 0] + S[:, None, :, :, 1]       # [B][i][j][8]: s_i + t_j
        lg = np.where(adj[None, :, :, None], np.maximum(x, 0.2 * x), -np.inf)
        e = g_round(np.exp2(lg - lg.max(2, keepdims=True)))  # 0 off the graph
        z = e.sum(2)                                        # [B][i][8]
        Whg = g_round(Wh.astype(np.float32)).reshape(B, N, 8, 32)
        out = np.einsum("bijh,bjhd->bihd", e, Whg)
        y = out / z[..., None] * (LOG2E if l == 0 else 1.0) + o[f"b{l}"].reshape(8, 32) * LOG2E
        y = y.reshape(B, N, 256)
        X = np.maximum((np.exp2(-np.abs(y)) - 1.0) * LOG2E, y)   # ELU(y) log2(e)
    if shape.nodes == 64:
        # chess: the policy is an MMA on the last activations as the
        # projection operand (format `op`, mode `act`, or exact with
        # `last="fp32"`) and W_pi rounded like the W_l; the value head pools
        # the fp32 activations
        Xp = X if last == "fp32" else round_op(X.astype(np.float32), op, act, rng)
        Wp = wr("w_pi") if last != "fp32" else o["w_pi"]
        lgp = (Xp * LN2 @ Wp + o["b_pi"]).reshape(B, -1)
        Xv = X
    else:
        if last in ("fp16", "fp16sr"):
            X = round_fp16(X.astype(np.float32), "rn" if last == "fp16" else "sr", rng)
        Xv = X
    Xv = Xv * LN2                                           # back to natural units
    gmean = Xv.mean(1)
    zv = np.maximum(gmean @ o["W_v1"] + o["b_v1"], 0.0)
    v = np.tanh(zv @ o["w_v2"] + o["b_v2"][0])
    if shape.nodes == 42:
        lgp = (Xv.reshape(B, 6, 7, 256).mean(1) @ o["w_pi"])[..., 0] + o["b_pi"][0]
    elif shape.nodes == 9:
        lgp = (Xv @ o["w_pi"])[..., 0] + o["b_pi"][0]
    lgp = lgp - lgp.max(1, keepdims=True)
    pe = np.exp(lgp)
    return pe / pe.sum(1, keepdims=True), v


def resnet_forward_rounded(w: np.ndarray, boards: np.ndarray, side: np.ndarray, op: str = "fp16",
                           resid: str = "op", wround: str = "sr") -> tuple[np.ndarray, np.ndarray]:
    """The Connect4 ResNet tower with the tensor-core kernel's roundings:
    every convolution's input activations rounded to nearest in `op`
    ("bf16", "fp16", "exact") and its weights by the pack kernel's hashed
    stochastic rounding (`wround="sr"`) or to nearest ("rn"); BN folded in fp32 (exact here); the
    residual read back from the rounded block input (`resid="op"`) or kept
    exact (`"exact"`); heads from the last convolution's exact output.
    Reference semantics: networks/resnet/resnet.cu:506-667."""
    import torch
    from helpers import res_blob_views

    o = res_blob_views()

    def t(k):
        p, sh = o[k]
        return torch.tensor(w[p:p + int(np.prod(sh))].reshape(sh), dtype=torch.float64)

    def rnd(x: torch.Tensor) -> torch.Tensor:
        if op == "exact":
            return x
        return torch.tensor(round_op(x.numpy().astype(np.float32), op, "rn"))

    b = torch.tensor(boards.astype(np.int64)).view(-1, 6, 7)
    sd = torch.tensor(side.astype(np.int64)).view(-1, 1, 1)
    x = torch.stack([(b == sd), (b == -sd), (sd == 1).expand_as(b)], 1).double()

    def rnd_w(k):
        if op == "exact" or wround == "rn":
            return rnd(t(k))
        p, sh = o[k]
        m = int(np.prod(sh))
        return torch.tensor(round_weights(w[p:p + m], op, p + np.arange(m, dtype=np.int64)).reshape(sh))

    def conv_bn(x, kw, kb):
        wt = rnd_w(kw).permute(0, 3, 1, 2)
        y = torch.nn.functional.conv2d(rnd(x), wt, padding=1)
        g, be, mu, var = t(kb)
        sc = g / torch.sqrt(var + 1e-5)
        return y * sc.view(1, -1, 1, 1) + (be - mu * sc).view(1, -1, 1, 1)

    a = torch.relu(conv_bn(x, "stem_w", "stem_bn"))
    for k in range(10):
        hmid = torch.relu(conv_bn(a, f"c1_{k}", f"bn1_{k}"))
        res = a if resid == "exact" else rnd(a)
        a = torch.relu(conv_bn(hmid, f"c2_{k}", f"bn2_{k}") + res)

    def bn(x, k):
        g, be, mu, var = t(k)
        sh = (1, -1, 1, 1)
        return (x - mu.view(sh)) / torch.sqrt(var.view(sh) + 1e-5) * g.view(sh) + be.view(sh)

    pf = bn(torch.einsum("oc,bchw->bohw", t("pol_w"), a), "pol_bn").reshape(-1, 84)
    pi = torch.softmax(pf @ t("pol_fc") + t("pol_fc_b"), -1)
    vf = bn(torch.einsum("oc,bchw->bohw", t("val_w"), a), "val_bn").reshape(-1, 42)
    hv = torch.relu(vf @ t("val_fc1") + t("val_fc1_b"))
    v = torch.tanh(hv @ t("val_fc2") + t("val_fc2_b"))
    return pi.numpy(), v.numpy()


def simulated_error(game: int, w: np.ndarray, boards: np.ndarray, side: np.ndarray, ref_pi: np.ndarray,
                    ref_v: np.ndarray, seeds=(0, 1, 2), **mode) -> float:
    """Max-abs difference of the rounded forward from (ref_pi, ref_v), the
    worst over `seeds` of the stochastic rounding."""
    import graphzero_b200 as gz
    from helpers import torch_features

    shape = gz.game_shape(game)
    rp, col = gz.game_graph(game)
    f = torch_features(game, boards, side).numpy()
    worst = 0.0
    for s in seeds:
        pi, v = gat_forward_rounded(game, shape, f, rp, col, w, seed=s, **mode)
        worst = max(worst, float(np.abs(pi - ref_pi).max()), float(np.abs(v - ref_v).max()))
    return worst


# Operand modes.  "bf16" / "fp16": the tensor-core kernels as built (bf16
# activations stochastically rounded, fp16 rounded to nearest; Connect4 pools
# the last layer in fp32); "*-fp16pool": the earlier Connect4 kernels, which
# pooled fp16-rounded last-layer activations and rounded fp16 stochastically.
MODES = {
    "connect4": {"bf16": dict(op="bf16", act="sr", last="fp32"), "fp16": dict(op="fp16", act="rn", last="fp32"),
                 "bf16-fp16pool": dict(op="bf16", act="sr", last="fp16"),
                 "fp16-sr-fp16pool": dict(op="fp16", act="sr", last="fp16")},
    "chess": {"bf16": dict(op="bf16", act="sr"), "fp16": dict(op="fp16", act="rn"),
              "fp16-sr": dict(op="fp16", act="sr")},
    "resnet": {"bf16": dict(op="bf16"), "fp16": dict(op="fp16"), "fp16-exact-residual": dict(op="fp16", resid="exact")},
}

# The GPU tests' inputs: weight seed, position seed base, batch sizes
# (tests/test_gat_gpu.py, tests/test_resnet_gpu.py).
TEST_INPUTS = {"connect4": (17, 200, (1, 2, 3, 4, 7, 300, 1000)), "chess": (23, 300, (1, 2, 3, 65, 300)),
               "resnet": (31, 40, (1, 2, 3, 5, 64, 301))}


def main() -> None:
    """Simulated max-abs error per mode on the GPU tests' inputs; writes
    tests/golden/rounding_bounds.json, which the GPU tests take their
    tolerances from.  Usage: python tests/rounding_sim.py [connect4|chess|resnet ...]"""
    import json
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent
    for p in (here, here.parent, here.parent / "oracle"):
        sys.path.insert(0, str(p))
    import graphzero_b200 as gz
    import oracle
    from helpers import sharpen

    out_path = here / "golden" / "rounding_bounds.json"
    table = json.loads(out_path.read_text()) if out_path.exists() else {}
    games = {"connect4": gz.CONNECT4, "chess": gz.CHESS}
    for label in sys.argv[1:] or ["connect4", "chess", "resnet"]:
        wseed, pseed, sizes = TEST_INPUTS[label]
        for sharp in ((False, True) if label != "resnet" else (False,)):
            key = f"{label}{'-sharp' if sharp else ''}"
            row = {}
            for name, mode in MODES[label].items():
                worst = 0.0
                for n in sizes:
                    if label == "resnet":
                        w = gz.synth_weights(gz.CONNECT4, gz.RESNET, seed=wseed)
                        boards, side = gz.synth_positions(gz.CONNECT4, n, seed=pseed + n)
                        opi, ov = oracle.resnet_forward(w, boards, side)
                        pi, v = resnet_forward_rounded(w, boards, side, **mode)
                        worst = max(worst, float(np.abs(pi - opi).max()), float(np.abs(v - ov).max()))
                        continue
                    game = games[label]
                    w = gz.synth_weights(game, seed=wseed, bias_scale=0.4 if sharp else 0.0)
                    if sharp:
                        w = sharpen(game, w)
                    boards, side = gz.synth_positions(game, n, seed=pseed + n)
                    opi, ov = oracle.gat_forward(game, w, boards, side)
                    worst = max(worst, simulated_error(game, w, boards, side, opi, ov, **mode))
                row[name] = float(f"{worst:.3e}")
            table[key] = row
            print(key, row, flush=True)
            out_path.write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
