"""ctypes wrapper of the CPU oracle (oracle/oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, as the checker and the timed CPU baseline.  The
graphzero_b200 package never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
LIB_NATIVE = HERE / "_build" / "liboracle_native.so"
REF_RULES = HERE / "_ref" / "libref_rules.so"

_vp, _i8p, _f32p, _i32p = C.c_void_p, C.POINTER(C.c_int8), C.POINTER(C.c_float), C.POINTER(C.c_int32)


def build() -> None:
    r = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")


def _cpu_has_avx2() -> bool:
    try:
        return " avx2 " in (" " + Path("/proc/cpuinfo").read_text().replace("\n", " ") + " ")
    except OSError:
        return False


def _load(path: Path):
    if not path.exists():
        build()
    lib = C.CDLL(str(path))
    sigs = {
        "orc_shape": (C.c_int, [C.c_int, _i32p]),
        "orc_graph": (C.c_int, [C.c_int, _i32p, _i32p]),
        "orc_features": (None, [C.c_int, _i8p, C.c_int, _f32p]),
        "orc_gat_weight_count": (C.c_size_t, [C.c_int]),
        "orc_res_weight_count": (C.c_size_t, []),
        "orc_gat_forward": (C.c_int, [C.c_int, _f32p, _i8p, _i8p, C.c_int, _f32p, _f32p, C.c_int, C.c_int]),
        "orc_resnet_forward": (C.c_int, [_f32p, _i8p, _i8p, C.c_int, _f32p, _f32p, C.c_int, C.c_int]),
        "orc_synth_gat_weights": (C.c_int, [C.c_int, C.c_uint64, C.c_float, C.c_int, _f32p]),
        "orc_synth_res_weights": (C.c_int, [C.c_uint64, C.c_int, _f32p]),
        "orc_synth_positions": (C.c_int, [C.c_int, C.c_uint64, C.c_uint64, C.c_int, _i8p, _i8p]),
        "orc_apply": (C.c_int, [C.c_int, _i8p, C.c_int, C.c_int]),
        "orc_legal": (C.c_int, [C.c_int, _i8p, C.c_int]),
        "orc_has_won": (C.c_int, [C.c_int, _i8p, C.c_int]),
        "orc_outcome": (C.c_int, [C.c_int, _i8p, C.c_int]),
        "orc_mcts_create": (_vp, [C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int]),
        "orc_mcts_destroy": (None, [_vp]),
        "orc_mcts_set_roots": (None, [_vp, _i8p, _i8p]),
        "orc_mcts_select": (C.c_int, [_vp, _i8p, _i8p, _i8p]),
        "orc_mcts_backup": (C.c_int, [_vp, _f32p, _f32p]),
        "orc_mcts_root_stats": (None, [_vp, _i32p, _f32p]),
        "orc_mcts_tree_sizes": (None, [_vp, _i32p, _i32p]),
        "orc_mcts_play": (None, [_vp, _i32p, C.c_int, _i8p]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    return lib


_lib = None
_lib_native = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load(LIB)
    return _lib


def lib_native():
    """Speed build (AVX2/FMA) for the CPU baseline; the checker build if the
    host CPU lacks AVX2."""
    global _lib_native
    if _lib_native is None:
        _lib_native = _load(LIB_NATIVE) if _cpu_has_avx2() else lib()
    return _lib_native


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def shape(game: int) -> dict:
    out = np.zeros(9, np.int32)
    if lib().orc_shape(game, _p(out, C.c_int32)) != 0:
        raise ValueError(game)
    keys = ("nodes", "rows", "cols", "actions", "features", "layers", "policy_per_node", "board_bytes", "nnz")
    return dict(zip(keys, map(int, out)))


def graph(game: int) -> tuple[np.ndarray, np.ndarray]:
    s = shape(game)
    rp = np.zeros(s["nodes"] + 1, np.int32)
    col = np.zeros(s["nnz"], np.int32)
    lib().orc_graph(game, _p(rp, C.c_int32), _p(col, C.c_int32))
    return rp, col


def features(game: int, board: np.ndarray, side: int) -> np.ndarray:
    s = shape(game)
    b = np.ascontiguousarray(board, np.int8)
    out = np.zeros((s["nodes"], s["features"]), np.float32)
    lib().orc_features(game, _p(b, C.c_int8), int(side), _p(out, C.c_float))
    return out


def gat_forward(game: int, w: np.ndarray, boards: np.ndarray, side: np.ndarray, threads: int = 0,
                f64: bool = False, native: bool = False) -> tuple[np.ndarray, np.ndarray]:
    s = shape(game)
    w = np.ascontiguousarray(w, np.float32)
    assert w.size == lib().orc_gat_weight_count(game)
    boards = np.ascontiguousarray(boards, np.int8)
    side = np.ascontiguousarray(side, np.int8)
    n = side.shape[0]
    pi = np.zeros((n, s["actions"]), np.float32)
    v = np.zeros(n, np.float32)
    L = lib_native() if native else lib()
    rc = L.orc_gat_forward(game, _p(w, C.c_float), _p(boards, C.c_int8), _p(side, C.c_int8), n,
                           _p(pi, C.c_float), _p(v, C.c_float), threads, int(f64))
    assert rc == 0
    return pi, v


def resnet_forward(w: np.ndarray, boards: np.ndarray, side: np.ndarray, threads: int = 0, f64: bool = False,
                   native: bool = False) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, np.float32)
    assert w.size == lib().orc_res_weight_count()
    boards = np.ascontiguousarray(boards, np.int8)
    side = np.ascontiguousarray(side, np.int8)
    n = side.shape[0]
    pi = np.zeros((n, 7), np.float32)
    v = np.zeros(n, np.float32)
    L = lib_native() if native else lib()
    rc = L.orc_resnet_forward(_p(w, C.c_float), _p(boards, C.c_int8), _p(side, C.c_int8), n,
                              _p(pi, C.c_float), _p(v, C.c_float), threads, int(f64))
    assert rc == 0
    return pi, v


def synth_gat_weights(game: int, seed: int, bias_scale: float = 0.0, bf16_exact: bool = True) -> np.ndarray:
    """Seeded GAT weight blob (the same streams as the product's generator)."""
    w = np.zeros(lib().orc_gat_weight_count(game), np.float32)
    assert lib().orc_synth_gat_weights(game, seed, bias_scale, int(bf16_exact), _p(w, C.c_float)) == 0
    return w


def synth_res_weights(seed: int, bf16_exact: bool = True) -> np.ndarray:
    """Seeded Connect4 ResNet weight blob."""
    w = np.zeros(lib().orc_res_weight_count(), np.float32)
    assert lib().orc_synth_res_weights(seed, int(bf16_exact), _p(w, C.c_float)) == 0
    return w


def synth_positions(game: int, n: int, seed: int, first: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Random legal TicTacToe / Connect4 positions (the product generator's
    streams)."""
    s = shape(game)
    b = np.zeros((n, s["board_bytes"]), np.int8)
    sd = np.zeros(n, np.int8)
    assert lib().orc_synth_positions(game, seed, first, n, _p(b, C.c_int8), _p(sd, C.c_int8)) == 0
    return b, sd


def apply(game: int, board: np.ndarray, action: int, player: int) -> int:
    assert board.dtype == np.int8 and board.flags["C_CONTIGUOUS"]
    return lib().orc_apply(game, _p(board, C.c_int8), action, player)


def legal(game: int, board: np.ndarray, action: int) -> bool:
    b = np.ascontiguousarray(board, np.int8)
    return bool(lib().orc_legal(game, _p(b, C.c_int8), action))


def has_won(game: int, board: np.ndarray, player: int) -> bool:
    b = np.ascontiguousarray(board, np.int8)
    return bool(lib().orc_has_won(game, _p(b, C.c_int8), player))


def outcome(game: int, board: np.ndarray, moved: int) -> int:
    b = np.ascontiguousarray(board, np.int8)
    return lib().orc_outcome(game, _p(b, C.c_int8), moved)


class Mcts:
    """Sequential CPU run of the batched PUCT wave algorithm."""

    def __init__(self, game: int, trees: int, leaves: int = 4, c_puct: float = 1.5, virtual_loss: int = 3,
                 node_capacity: int = 4096):
        self.game, self.trees, self.leaves = game, trees, leaves
        self.s = shape(game)
        self._h = lib().orc_mcts_create(game, trees, leaves, c_puct, virtual_loss, node_capacity)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_mcts_destroy(self._h)
            self._h = None

    def set_roots(self, boards: np.ndarray, side: np.ndarray) -> None:
        b = np.ascontiguousarray(boards, np.int8)
        s = np.ascontiguousarray(side, np.int8)
        lib().orc_mcts_set_roots(self._h, _p(b, C.c_int8), _p(s, C.c_int8))

    def select(self) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        L = self.trees * self.leaves
        b = np.zeros((L, self.s["nodes"]), np.int8)
        sd = np.zeros(L, np.int8)
        t = np.zeros(L, np.int8)
        rc = lib().orc_mcts_select(self._h, _p(b, C.c_int8), _p(sd, C.c_int8), _p(t, C.c_int8))
        if rc != 0:
            raise RuntimeError(f"oracle select failed: {rc}")
        return b, sd, t

    def backup(self, pi: np.ndarray, v: np.ndarray) -> None:
        p = np.ascontiguousarray(pi, np.float32)
        vv = np.ascontiguousarray(v, np.float32)
        rc = lib().orc_mcts_backup(self._h, _p(p, C.c_float), _p(vv, C.c_float))
        if rc != 0:
            raise RuntimeError(f"oracle backup failed: {rc}")

    def root_stats(self) -> tuple[np.ndarray, np.ndarray]:
        A = self.s["actions"]
        vis = np.zeros((self.trees, A), np.int32)
        w = np.zeros((self.trees, A), np.float32)
        lib().orc_mcts_root_stats(self._h, _p(vis, C.c_int32), _p(w, C.c_float))
        return vis, w

    def tree_sizes(self) -> tuple[np.ndarray, np.ndarray]:
        n = np.zeros(self.trees, np.int32)
        e = np.zeros(self.trees, np.int32)
        lib().orc_mcts_tree_sizes(self._h, _p(n, C.c_int32), _p(e, C.c_int32))
        return n, e

    def play(self, actions: np.ndarray, reserve: int) -> np.ndarray:
        a = np.ascontiguousarray(actions, np.int32)
        done = np.zeros(self.trees, np.int8)
        lib().orc_mcts_play(self._h, _p(a, C.c_int32), reserve, _p(done, C.c_int8))
        return done


def ref_rules():
    """The reference's own rule functions (oracle/_ref), or None if not built."""
    if not REF_RULES.exists():
        return None
    L = C.CDLL(str(REF_RULES))
    L.ref_next_state.argtypes = [C.c_int, _i32p, C.c_int, C.c_int, _i32p, _i32p]
    L.ref_valid_moves.argtypes = [C.c_int, _i32p, C.c_int, C.POINTER(C.c_uint8)]
    L.ref_game_ended.argtypes = [C.c_int, _i32p, C.c_int]
    L.ref_game_ended.restype = C.c_int
    L.ref_canonical.argtypes = [C.c_int, _i32p, C.c_int, _i32p]
    return L


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
