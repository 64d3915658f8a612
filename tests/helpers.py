"""Test helpers: an independent torch fp32/fp64 restatement of the GAT and
ResNet forwards (used to cross-check the oracle), weight-blob views, and
weight "sharpening" so policy parity is not trivially satisfied."""
from __future__ import annotations

import numpy as np
import torch

import graphzero_b200 as gz


def gat_blob_views(game: int) -> dict:
    """name -> (offset, shape) in the documented GAT blob layout."""
    s = gz.game_shape(game)
    o, p = {}, 0
    for l in range(s.layers):
        fin = s.features if l == 0 else 256
        for k, sh in ((f"W{l}", (fin, 256)), (f"b{l}", (256,)), (f"a{l}", (8, 2, 32))):
            o[k] = (p, sh)
            p += int(np.prod(sh))
    P = s.policy_per_node
    for k, sh in (("w_pi", (256, P)), ("b_pi", (P,)), ("W_v1", (256, 64)), ("b_v1", (64,)), ("w_v2", (64,)),
                  ("b_v2", (1,))):
        o[k] = (p, sh)
        p += int(np.prod(sh))
    assert p == gz.weight_count(game)
    return o


def sharpen(game: int, w: np.ndarray, policy_gain: float = 30.0, value_gain: float = 4.0) -> np.ndarray:
    """Scale the policy and value heads so outputs spread far from uniform."""
    w = w.copy()
    o = gat_blob_views(game)
    p, sh = o["w_pi"]
    w[p:p + int(np.prod(sh))] *= policy_gain
    p, sh = o["W_v1"]
    w[p:p + int(np.prod(sh))] *= value_gain
    return w


def _t(w, o, k, dt):
    p, sh = o[k]
    return torch.tensor(w[p:p + int(np.prod(sh))].reshape(sh), dtype=dt)


def torch_features(game: int, boards: np.ndarray, side: np.ndarray) -> torch.Tensor:
    b = torch.tensor(boards.astype(np.int64))
    sd = torch.tensor(side.astype(np.int64)).view(-1, 1)
    if game != gz.CHESS:
        f = torch.stack([(b == 0), (b == sd), (b == -sd), (sd == 1).expand_as(b)], -1)
        return f.double()
    sq = b[:, :64]
    f = torch.zeros(b.shape[0], 64, 18, dtype=torch.float64)
    for k in range(6):
        f[..., k] = (sq == k + 1).double()
        f[..., 6 + k] = (sq == -(k + 1)).double()
    f[..., 12] = (sd == 1).double().expand(-1, 64)
    castle = (b[:, 64] & 0xFF).view(-1, 1)
    for k in range(4):
        f[..., 13 + k] = ((castle >> k) & 1).double().expand(-1, 64)
    f[..., 17] = (torch.arange(64).view(1, 64) == b[:, 65].view(-1, 1)).double()
    return f


def torch_gat(game: int, w: np.ndarray, boards: np.ndarray, side: np.ndarray,
              dtype=torch.float64) -> tuple[np.ndarray, np.ndarray]:
    """Vectorised restatement of the GAT forward (edge-list form)."""
    s = gz.game_shape(game)
    o = gat_blob_views(game)
    rp, col = gz.game_graph(game)
    B, N = len(side), s.nodes
    X = torch_features(game, boards, side).to(dtype)
    src = torch.repeat_interleave(torch.arange(N), torch.tensor(np.diff(rp).astype(np.int64)))
    dst = torch.tensor(col.astype(np.int64))
    for l in range(s.layers):
        Wh = X @ _t(w, o, f"W{l}", dtype)
        Whh = Wh.view(B, N, 8, 32)
        a = _t(w, o, f"a{l}", dtype)
        ss = (Whh * a[:, 0]).sum(-1)
        sn = (Whh * a[:, 1]).sum(-1)
        e = torch.nn.functional.leaky_relu(ss[:, src] + sn[:, dst], 0.2)
        m = torch.full((B, N, 8), -torch.inf, dtype=dtype).scatter_reduce(
            1, src.view(1, -1, 1).expand(B, -1, 8), e, "amax")
        p = torch.exp(e - m[:, src])
        z = torch.zeros(B, N, 8, dtype=dtype).index_add(1, src, p)
        al = p / z[:, src]
        out = torch.zeros(B, N, 8, 32, dtype=dtype).index_add(1, src, al.unsqueeze(-1) * Whh[:, dst])
        X = torch.nn.functional.elu(out.view(B, N, 256) + _t(w, o, f"b{l}", dtype))
    g = X.mean(1)
    z = torch.relu(g @ _t(w, o, "W_v1", dtype) + _t(w, o, "b_v1", dtype))
    v = torch.tanh(z @ _t(w, o, "w_v2", dtype) + _t(w, o, "b_v2", dtype))
    if game == gz.TICTACTOE:
        lg = (X @ _t(w, o, "w_pi", dtype)).squeeze(-1) + _t(w, o, "b_pi", dtype)
    elif game == gz.CONNECT4:
        lg = (X.view(B, 6, 7, 256).mean(1) @ _t(w, o, "w_pi", dtype)).squeeze(-1) + _t(w, o, "b_pi", dtype)
    else:
        lg = (X @ _t(w, o, "w_pi", dtype) + _t(w, o, "b_pi", dtype)).reshape(B, -1)
    return torch.softmax(lg, -1).numpy(), v.numpy()


def res_blob_views() -> dict:
    o, p = {}, 0
    C = 128
    items = [("stem_w", (C, 3, 3, 3)), ("stem_bn", (4, C))]
    for k in range(10):
        items += [(f"c1_{k}", (C, 3, 3, C)), (f"bn1_{k}", (4, C)), (f"c2_{k}", (C, 3, 3, C)), (f"bn2_{k}", (4, C))]
    items += [("pol_w", (2, C)), ("pol_bn", (4, 2)), ("pol_fc", (84, 7)), ("pol_fc_b", (7,)), ("val_w", (1, C)),
              ("val_bn", (4, 1)), ("val_fc1", (42, 128)), ("val_fc1_b", (128,)), ("val_fc2", (128,)),
              ("val_fc2_b", (1,))]
    for k, sh in items:
        o[k] = (p, sh)
        p += int(np.prod(sh))
    assert p == gz.weight_count(gz.CONNECT4, gz.RESNET)
    return o


def torch_resnet(w: np.ndarray, boards: np.ndarray, side: np.ndarray, dtype=torch.float64):
    o = res_blob_views()
    b = torch.tensor(boards.astype(np.int64)).view(-1, 6, 7)
    sd = torch.tensor(side.astype(np.int64)).view(-1, 1, 1)
    x = torch.stack([(b == sd), (b == -sd), (sd == 1).expand_as(b)], 1).to(dtype)  # NCHW

    def conv(x, k):  # weights [Cout][ky][kx][Cin] -> [Cout][Cin][ky][kx]
        return torch.nn.functional.conv2d(x, _t(w, o, k, dtype).permute(0, 3, 1, 2), padding=1)

    def bn(x, k):
        g, be, mu, var = _t(w, o, k, dtype)
        sh = (1, -1, 1, 1)
        return (x - mu.view(sh)) / torch.sqrt(var.view(sh) + 1e-5) * g.view(sh) + be.view(sh)

    a = torch.relu(bn(conv(x, "stem_w"), "stem_bn"))
    for k in range(10):
        t = torch.relu(bn(conv(a, f"c1_{k}"), f"bn1_{k}"))
        a = torch.relu(bn(conv(t, f"c2_{k}"), f"bn2_{k}") + a)
    pf = bn(torch.einsum("oc,bchw->bohw", _t(w, o, "pol_w", dtype), a), "pol_bn").reshape(-1, 84)
    pi = torch.softmax(pf @ _t(w, o, "pol_fc", dtype) + _t(w, o, "pol_fc_b", dtype), -1)
    vf = bn(torch.einsum("oc,bchw->bohw", _t(w, o, "val_w", dtype), a), "val_bn").reshape(-1, 42)
    h = torch.relu(vf @ _t(w, o, "val_fc1", dtype) + _t(w, o, "val_fc1_b", dtype))
    v = torch.tanh(h @ _t(w, o, "val_fc2", dtype) + _t(w, o, "val_fc2_b", dtype))
    return pi.numpy(), v.numpy()


def chess_boards(n: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Random chess-like records (piece placement, castling, en passant) for
    exercising the chess encoder and network math; not necessarily legal."""
    rng = np.random.default_rng(seed)
    b = np.zeros((n, 66), np.int8)
    for i in range(n):
        sq = rng.choice(64, size=rng.integers(2, 33), replace=False)
        b[i, sq] = rng.choice([-6, -5, -4, -3, -2, -1, 1, 2, 3, 4, 5, 6], size=sq.size)
        b[i, 64] = rng.integers(0, 16)
        b[i, 65] = rng.choice([-1, int(rng.integers(16, 24)), int(rng.integers(40, 48))])
    side = rng.choice([-1, 1], size=n).astype(np.int8)
    return b, side


def torch_gat_loss(game: int, w: np.ndarray, boards: np.ndarray, side: np.ndarray, pi: np.ndarray, v: np.ndarray,
                   dtype=torch.float64) -> tuple[float, float, np.ndarray]:
    """Training loss of the GAT (mean policy cross-entropy, mean squared value
    error) and its gradient with respect to the flat weight blob, by torch
    autograd on an independent restatement of the forward."""
    s = gz.game_shape(game)
    o = gat_blob_views(game)
    rp, col = gz.game_graph(game)
    B, N = len(side), s.nodes
    flat = torch.tensor(w.astype(np.float64), dtype=dtype, requires_grad=True)

    def t(k):
        p, sh = o[k]
        return flat[p:p + int(np.prod(sh))].view(sh)

    X = torch_features(game, boards, side).to(dtype)
    src = torch.repeat_interleave(torch.arange(N), torch.tensor(np.diff(rp).astype(np.int64)))
    dst = torch.tensor(col.astype(np.int64))
    for l in range(s.layers):
        Wh = X @ t(f"W{l}")
        Whh = Wh.view(B, N, 8, 32)
        a = t(f"a{l}")
        ss = (Whh * a[:, 0]).sum(-1)
        sn = (Whh * a[:, 1]).sum(-1)
        e = torch.nn.functional.leaky_relu(ss[:, src] + sn[:, dst], 0.2)
        m = torch.full((B, N, 8), -torch.inf, dtype=dtype).scatter_reduce(
            1, src.view(1, -1, 1).expand(B, -1, 8), e, "amax").detach()
        p = torch.exp(e - m[:, src])
        z = torch.zeros(B, N, 8, dtype=dtype).index_add(1, src, p)
        al = p / z[:, src]
        out = torch.zeros(B, N, 8, 32, dtype=dtype).index_add(1, src, al.unsqueeze(-1) * Whh[:, dst])
        X = torch.nn.functional.elu(out.reshape(B, N, 256) + t(f"b{l}"))
    g = X.mean(1)
    hv = torch.relu(g @ t("W_v1") + t("b_v1"))
    val = torch.tanh(hv @ t("w_v2") + t("b_v2"))
    if game == gz.TICTACTOE:
        lg = (X @ t("w_pi")).squeeze(-1) + t("b_pi")
    elif game == gz.CONNECT4:
        lg = (X.view(B, 6, 7, 256).mean(1) @ t("w_pi")).squeeze(-1) + t("b_pi")
    else:
        lg = (X @ t("w_pi") + t("b_pi")).reshape(B, -1)
    tp = torch.tensor(pi, dtype=dtype)
    lp = -(tp * torch.log_softmax(lg, -1)).sum(-1).mean()
    lv = ((torch.tensor(v, dtype=dtype) - val) ** 2).mean()
    (lp + lv).backward()
    return float(lp.detach()), float(lv.detach()), flat.grad.numpy()


def resnet_frozen_mask() -> np.ndarray:
    """True at the ResNet's BN means and variances (fixed statistics)."""
    o = res_blob_views()
    mask = np.zeros(gz.weight_count(gz.CONNECT4, gz.RESNET), bool)
    for k, (p, sh) in o.items():
        if k.endswith("bn") or k.startswith("bn"):
            c = sh[1]
            mask[p + 2 * c:p + 4 * c] = True
    return mask


def torch_resnet_loss(w: np.ndarray, boards: np.ndarray, side: np.ndarray, pi: np.ndarray, v: np.ndarray,
                      dtype=torch.float64) -> tuple[float, float, np.ndarray]:
    """Training loss of the Connect4 ResNet (BN in inference form with its
    stored statistics held fixed) and its gradient with respect to the flat
    weight blob, by torch autograd on an independent restatement."""
    o = res_blob_views()
    flat = torch.tensor(w.astype(np.float64), dtype=dtype, requires_grad=True)
    frozen = torch.tensor(resnet_frozen_mask())
    src = torch.where(frozen, flat.detach(), flat)

    def t(k):
        p, sh = o[k]
        return src[p:p + int(np.prod(sh))].view(sh)

    b = torch.tensor(boards.astype(np.int64)).view(-1, 6, 7)
    sd = torch.tensor(side.astype(np.int64)).view(-1, 1, 1)
    x = torch.stack([(b == sd), (b == -sd), (sd == 1).expand_as(b)], 1).to(dtype)

    def conv(x, k):
        return torch.nn.functional.conv2d(x, t(k).permute(0, 3, 1, 2), padding=1)

    def bn(x, k):
        g, be, mu, var = t(k)
        sh = (1, -1, 1, 1)
        return (x - mu.view(sh)) / torch.sqrt(var.view(sh) + 1e-5) * g.view(sh) + be.view(sh)

    a = torch.relu(bn(conv(x, "stem_w"), "stem_bn"))
    for k in range(10):
        h = torch.relu(bn(conv(a, f"c1_{k}"), f"bn1_{k}"))
        a = torch.relu(bn(conv(h, f"c2_{k}"), f"bn2_{k}") + a)
    pf = bn(torch.einsum("oc,bchw->bohw", t("pol_w"), a), "pol_bn").reshape(-1, 84)
    lg = pf @ t("pol_fc") + t("pol_fc_b")
    vf = bn(torch.einsum("oc,bchw->bohw", t("val_w"), a), "val_bn").reshape(-1, 42)
    hv = torch.relu(vf @ t("val_fc1") + t("val_fc1_b"))
    val = torch.tanh(hv @ t("val_fc2") + t("val_fc2_b"))
    tp = torch.tensor(pi, dtype=dtype)
    lp = -(tp * torch.log_softmax(lg, -1)).sum(-1).mean()
    lv = ((torch.tensor(v, dtype=dtype) - val) ** 2).mean()
    (lp + lv).backward()
    return float(lp.detach()), float(lv.detach()), flat.grad.numpy()
