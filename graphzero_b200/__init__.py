"""graphzero_b200: B200 leaf evaluation and batched PUCT search for GraphZero.

Python mirror of the C ABI in include/graphzero_b200.h.  The compute path is
the CUDA library libgraphzero_b200.so built in this directory (see
graphzero_b200.build); importing this package fails loudly when it is
missing — there is no CPU or eager fallback.

The interface follows the reference's model interface INeuralNet
(networks/neural_network.h:16-27: init / predict / save / load / destroy /
broadcast_weights) and its factory create_neural_net(type, game)
(networks/neural_network.c:6-13), with batched device-pointer calls added.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libgraphzero_b200.so"

TICTACTOE, CONNECT4, CHESS = 0, 1, 2
GAT, RESNET = 0, 1
PREC_AUTO, PREC_FP32, PREC_BF16, PREC_FP16 = 0, 1, 2, 3
GAME_NAMES = {"tictactoe": TICTACTOE, "connect4": CONNECT4, "chess": CHESS}

OK, ERR_INVALID_ARG, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_IO, ERR_CAPACITY, ERR_UNSUPPORTED = range(8)


class GZError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is missing: run `python graphzero_b200/build.py` (nvcc, sm_100a)")
_lib = C.CDLL(str(LIB_PATH))

_vp, _i8p, _f32p, _i32p = C.c_void_p, C.POINTER(C.c_int8), C.POINTER(C.c_float), C.POINTER(C.c_int32)


class NetConfig(C.Structure):
    _fields_ = [("game", C.c_int), ("kind", C.c_int), ("precision", C.c_int), ("max_batch", C.c_int)]


class MctsConfig(C.Structure):
    _fields_ = [("game", C.c_int), ("trees", C.c_int), ("leaves_per_tree", C.c_int), ("c_puct", C.c_float),
                ("virtual_loss", C.c_int), ("node_capacity", C.c_int), ("dirichlet_alpha", C.c_float),
                ("dirichlet_eps", C.c_float), ("seed", C.c_uint64)]


class TrainConfig(C.Structure):
    """gz_train_config: Adam hyper-parameters, batch size, passes, order seed."""
    _fields_ = [("learning_rate", C.c_float), ("weight_decay", C.c_float), ("beta1", C.c_float),
                ("beta2", C.c_float), ("eps", C.c_float), ("batch_size", C.c_int), ("epochs", C.c_int),
                ("seed", C.c_uint64)]


class TrainStats(C.Structure):
    _fields_ = [("policy_loss", C.c_float), ("value_loss", C.c_float), ("steps", C.c_int64)]


# name -> (restype, argtypes)
_SIGS = {
    "gz_status_string": (C.c_char_p, [C.c_int]),
    "gz_last_error": (C.c_char_p, []),
    "gz_version": (C.c_char_p, []),
    "gz_game_shape": (C.c_int, [C.c_int, _i32p]),
    "gz_game_graph": (C.c_int, [C.c_int, _i32p, _i32p]),
    "gz_game_next_state": (C.c_int, [C.c_int, _i8p, C.c_int, C.c_int, _i8p, C.POINTER(C.c_int)]),
    "gz_game_valid_moves": (C.c_int, [C.c_int, _i8p, C.POINTER(C.c_uint8)]),
    "gz_game_ended": (C.c_int, [C.c_int, _i8p, C.c_int, C.POINTER(C.c_int)]),
    "gz_weight_count": (C.c_size_t, [C.c_int, C.c_int]),
    "gz_synth_weights": (C.c_int, [C.c_int, C.c_int, C.c_uint64, C.c_float, C.c_int, _f32p, C.c_size_t]),
    "gz_synth_positions": (C.c_int, [C.c_int, C.c_uint64, C.c_uint64, C.c_int, _i8p, _i8p]),
    "gz_chess_legal_count": (C.c_int, [_i8p, C.c_int, C.POINTER(C.c_int)]),
    "gz_chess_perft": (C.c_int, [_i8p, C.c_int, C.c_int, C.POINTER(C.c_uint64)]),
    "gz_chess_legal_actions": (C.c_int, [_i8p, C.c_int, C.POINTER(C.c_int16), C.POINTER(C.c_int)]),
    "gz_chess_valid_moves": (C.c_int, [_i8p, C.c_int, C.POINTER(C.c_uint8)]),
    "gz_chess_next_state": (C.c_int, [_i8p, C.c_int, C.c_int, _i8p, C.POINTER(C.c_int)]),
    "gz_chess_ended": (C.c_int, [_i8p, C.c_int, C.POINTER(C.c_int)]),
    "gz_synth_positions_device": (C.c_int, [C.c_int, C.c_uint64, C.c_uint64, C.c_int, _vp, _vp, _vp]),
    "gz_chess_legal_actions_device": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp, _vp]),
    "gz_net_create": (C.c_int, [C.POINTER(NetConfig), C.c_int, C.POINTER(_vp)]),
    "gz_net_destroy": (C.c_int, [_vp]),
    "gz_net_weight_count": (C.c_size_t, [_vp]),
    "gz_net_kernel_name": (C.c_char_p, [_vp]),
    "gz_net_load_weights": (C.c_int, [_vp, _f32p, C.c_size_t]),
    "gz_net_save_weights": (C.c_int, [_vp, _f32p, C.c_size_t]),
    "gz_net_predict_batch": (C.c_int, [_vp, _vp, _vp, C.c_int, _vp, _vp, _vp]),
    "gz_net_check": (C.c_int, [_vp]),
    "gz_net_predict_host": (C.c_int, [_vp, _vp, _vp, C.c_int, _vp, _vp]),  # raw addresses: the per-step call
    "gz_net_predict": (C.c_int, [_vp, _f32p, _f32p, _f32p]),
    "gz_net_broadcast": (C.c_int, [_vp, _vp, C.c_int, _vp]),
    "gz_net_save_checkpoint": (C.c_int, [_vp, C.c_char_p]),
    "gz_net_load_checkpoint": (C.c_int, [_vp, C.c_char_p]),
    "gz_create_connect4_game": (_vp, []),
    "gz_create_tictactoe_game": (_vp, []),
    "gz_game_free": (None, [_vp]),
    "gz_create_neural_net": (_vp, [C.c_char_p, _vp, C.c_int]),
    "gz_shim_net": (_vp, [_vp]),
    "gz_shim_make_ineuralnet": (_vp, [_vp]),
    "gz_nccl_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
    "gz_nccl_comm_init": (C.c_int, [C.POINTER(C.c_uint8), C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    "gz_nccl_comm_destroy": (C.c_int, [_vp]),
    "gz_mcts_create": (C.c_int, [C.POINTER(MctsConfig), C.c_int, C.POINTER(_vp)]),
    "gz_mcts_destroy": (C.c_int, [_vp]),
    "gz_mcts_reset_roots": (C.c_int, [_vp, _vp, _vp, _vp]),
    "gz_mcts_select": (C.c_int, [_vp, _vp]),
    "gz_mcts_leaf_buffers": (C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp)]),
    "gz_mcts_copy_leaves": (C.c_int, [_vp, _i8p, _i8p, _i8p, _vp]),
    "gz_mcts_backup": (C.c_int, [_vp, _vp, _vp, _vp]),
    "gz_mcts_step": (C.c_int, [_vp, _vp, _vp]),
    "gz_mcts_run": (C.c_int, [_vp, _vp, C.c_int, _vp]),
    "gz_mcts_root_stats": (C.c_int, [_vp, _i32p, _f32p, _vp]),
    "gz_mcts_tree_sizes": (C.c_int, [_vp, _i32p, _i32p, _vp]),
    "gz_mcts_choose": (C.c_int, [_vp, C.c_int, _vp, _vp]),
    "gz_mcts_play": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp]),
    "gz_mcts_check": (C.c_int, [_vp]),
    "gz_selfplay_create": (C.c_int, [_vp, C.c_int, C.POINTER(_vp)]),
    "gz_selfplay_destroy": (C.c_int, [_vp]),
    "gz_selfplay_run": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, _vp]),
    "gz_selfplay_take": (C.c_int, [_vp, _vp, C.c_int64, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "gz_arena_play": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, _i32p, _i32p, _i32p, _vp]),
    "gz_train_examples_save": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(_vp), _i32p]),
    "gz_train_examples_load": (C.c_int, [C.c_char_p, _vp, C.c_int64, _i32p, C.c_int, C.POINTER(C.c_int),
                                         C.POINTER(C.c_int64)]),
    "gz_selftest_wait_timeout": (C.c_int, [C.c_int, C.c_int]),
    "gz_train_config_default": (None, [C.POINTER(TrainConfig)]),
    "gz_net_loss_grad": (C.c_int, [_vp, _vp, _vp, _vp, _vp, C.c_int, _vp, _f32p, _vp]),
    "gz_net_train_step": (C.c_int, [_vp, _vp, _vp, _vp, _vp, C.c_int, C.POINTER(TrainConfig), _vp, C.c_int, _f32p,
                                    _vp]),
    "gz_net_train": (C.c_int, [_vp, _vp, C.c_int64, C.POINTER(TrainConfig), _vp, C.c_int, C.c_int,
                               C.POINTER(TrainStats)]),
    "gz_train_batch_indices": (C.c_int, [C.c_int64, C.POINTER(TrainConfig), C.c_int, C.c_int64, C.c_int, C.c_int,
                                         C.POINTER(C.c_int64)]),
    "gz_train_bucket_range": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "gz_gat_c4_predict_noalloc": (C.c_int, [C.c_int, _f32p, C.c_size_t, _i8p, _i8p, C.c_int, _f32p, _f32p]),
    "gz_gat_c4_noalloc_scratch_bytes": (C.c_size_t, []),
    "gz_gat_c4_noalloc_max_batch": (C.c_int, []),
}
for _name, (_res, _args) in _SIGS.items():
    _f = getattr(_lib, _name)
    _f.restype, _f.argtypes = _res, _args

EXPORTED_SYMBOLS = tuple(_SIGS)


def _check(status: int) -> None:
    if status != OK:
        raise GZError(status, _lib.gz_last_error().decode(errors="replace"))


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(C.POINTER(t))


def _dev(x) -> int:
    """Raw device address of a torch tensor (or an int address)."""
    if x is None:
        return None
    return x if isinstance(x, int) else x.data_ptr()


def _stream(s) -> int | None:
    if s is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:  # noqa: BLE001
            return None
    return s if isinstance(s, int) else s.cuda_stream


def gat_c4_noalloc_max_batch() -> int:
    return _lib.gz_gat_c4_noalloc_max_batch()


def gat_c4_noalloc_scratch_bytes() -> int:
    return _lib.gz_gat_c4_noalloc_scratch_bytes()


def gat_c4_predict_noalloc(weights: np.ndarray, boards: np.ndarray, side: np.ndarray,
                           device: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Connect4 GAT evaluation that allocates no device memory (host buffers
    in and out, staging in a fixed device array; n <= 4096 per call)."""
    w = np.ascontiguousarray(weights, np.float32)
    b = np.ascontiguousarray(boards, np.int8)
    s = np.ascontiguousarray(side, np.int8)
    n = s.shape[0]
    pi = np.empty((n, 7), np.float32)
    v = np.empty(n, np.float32)
    _check(_lib.gz_gat_c4_predict_noalloc(device, _ptr(w, C.c_float), w.size, _ptr(b, C.c_int8), _ptr(s, C.c_int8), n,
                                          _ptr(pi, C.c_float), _ptr(v, C.c_float)))
    return pi, v


def selftest_wait_timeout(device: int = 0, limit_us: int = 20000) -> int:
    """Status of a kernel whose bounded wait on a never-arriving barrier runs
    out (GZ_ERR_TIMEOUT expected; the context stays usable)."""
    return int(_lib.gz_selftest_wait_timeout(device, limit_us))


def version() -> str:
    return _lib.gz_version().decode()


class GameShape:
    __slots__ = ("nodes", "rows", "cols", "actions", "features", "layers", "policy_per_node", "board_bytes", "nnz")

    def __init__(self, v):
        for k, x in zip(self.__slots__, v):
            setattr(self, k, int(x))


def game_shape(game: int) -> GameShape:
    out = np.zeros(9, np.int32)
    _check(_lib.gz_game_shape(game, _ptr(out, C.c_int32)))
    return GameShape(out)


def game_graph(game: int) -> tuple[np.ndarray, np.ndarray]:
    s = game_shape(game)
    rp = np.zeros(s.nodes + 1, np.int32)
    col = np.zeros(s.nnz, np.int32)
    _check(_lib.gz_game_graph(game, _ptr(rp, C.c_int32), _ptr(col, C.c_int32)))
    return rp, col


def next_state(game: int, board: np.ndarray, player: int, action: int) -> tuple[np.ndarray, int]:
    b = np.ascontiguousarray(board, np.int8)
    out = np.zeros_like(b)
    np_ = C.c_int()
    _check(_lib.gz_game_next_state(game, _ptr(b, C.c_int8), player, action, _ptr(out, C.c_int8), C.byref(np_)))
    return out, np_.value


def valid_moves(game: int, board: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(board, np.int8)
    out = np.zeros(game_shape(game).actions, np.uint8)
    _check(_lib.gz_game_valid_moves(game, _ptr(b, C.c_int8), _ptr(out, C.c_uint8)))
    return out.astype(bool)


def game_ended(game: int, board: np.ndarray, player: int) -> int:
    b = np.ascontiguousarray(board, np.int8)
    r = C.c_int()
    _check(_lib.gz_game_ended(game, _ptr(b, C.c_int8), player, C.byref(r)))
    return r.value


def weight_count(game: int, kind: int = GAT) -> int:
    return int(_lib.gz_weight_count(game, kind))


def synth_weights(game: int, kind: int = GAT, seed: int = 0x6A5A, bias_scale: float = 0.0,
                  bf16_exact: bool = True) -> np.ndarray:
    n = weight_count(game, kind)
    if n == 0:
        raise GZError(ERR_INVALID_ARG, f"no weight layout for game {game} kind {kind}")
    w = np.empty(n, np.float32)
    _check(_lib.gz_synth_weights(game, kind, seed, bias_scale, int(bf16_exact), _ptr(w, C.c_float), n))
    return w


def chess_legal_count(board: np.ndarray, side: int) -> int:
    b = np.ascontiguousarray(board, np.int8)
    r = C.c_int()
    _check(_lib.gz_chess_legal_count(_ptr(b, C.c_int8), side, C.byref(r)))
    return r.value


def chess_perft(board: np.ndarray, side: int, depth: int) -> int:
    b = np.ascontiguousarray(board, np.int8)
    r = C.c_uint64()
    _check(_lib.gz_chess_perft(_ptr(b, C.c_int8), side, depth, C.byref(r)))
    return r.value


CHESS_ACTIONS = 64 * 73


def chess_legal_actions(board: np.ndarray, side: int) -> np.ndarray:
    """Action indices (from * 73 + t) of the legal moves, in generation order."""
    b = np.ascontiguousarray(board, np.int8)
    out = np.empty(256, np.int16)
    r = C.c_int()
    _check(_lib.gz_chess_legal_actions(_ptr(b, C.c_int8), side, _ptr(out, C.c_int16), C.byref(r)))
    return out[:r.value].copy()


def chess_valid_moves(board: np.ndarray, side: int) -> np.ndarray:
    b = np.ascontiguousarray(board, np.int8)
    v = np.zeros(CHESS_ACTIONS, np.uint8)
    _check(_lib.gz_chess_valid_moves(_ptr(b, C.c_int8), side, _ptr(v, C.c_uint8)))
    return v


def chess_next_state(board: np.ndarray, side: int, action: int) -> tuple[np.ndarray, int]:
    b = np.ascontiguousarray(board, np.int8)
    nb = np.empty(66, np.int8)
    ns = C.c_int()
    _check(_lib.gz_chess_next_state(_ptr(b, C.c_int8), side, action, _ptr(nb, C.c_int8), C.byref(ns)))
    return nb, ns.value


def chess_ended(board: np.ndarray, side: int) -> int:
    """0 while the side to move has a legal move, -1 checkmated, 2 stalemate."""
    b = np.ascontiguousarray(board, np.int8)
    r = C.c_int()
    _check(_lib.gz_chess_ended(_ptr(b, C.c_int8), side, C.byref(r)))
    return r.value


def synth_positions_device(game: int, n: int, seed: int = 0x6A5A, first: int = 0, device: int = 0, stream=None):
    """synth_positions made on the GPU: (boards, side) as torch int8 tensors on
    cuda:device, byte for byte what synth_positions returns."""
    import torch
    s = game_shape(game)
    boards = torch.empty((n, s.board_bytes), dtype=torch.int8, device=f"cuda:{device}")
    side = torch.empty(n, dtype=torch.int8, device=boards.device)
    with torch.cuda.device(boards.device):
        _check(_lib.gz_synth_positions_device(game, seed, first, n, _dev(boards), _dev(side), _stream(stream)))
    return boards, side


def chess_legal_actions_device(boards, side, stream=None):
    """Legal action lists of chess positions on the GPU (torch int8 tensors
    [n][66] and [n]): (actions int16 [n][256], -1 padded; counts int32 [n])."""
    import torch
    n = boards.shape[0]
    actions = torch.empty((n, 256), dtype=torch.int16, device=boards.device)
    counts = torch.empty(n, dtype=torch.int32, device=boards.device)
    with torch.cuda.device(boards.device):
        _check(_lib.gz_chess_legal_actions_device(_dev(boards.contiguous()), _dev(side.contiguous()), n, _dev(actions),
                                                  _dev(counts), _stream(stream)))
    return actions, counts


def synth_positions(game: int, n: int, seed: int = 0x6A5A, first: int = 0) -> tuple[np.ndarray, np.ndarray]:
    s = game_shape(game)
    boards = np.zeros((n, s.board_bytes), np.int8)
    side = np.zeros(n, np.int8)
    _check(_lib.gz_synth_positions(game, seed, first, n, _ptr(boards, C.c_int8), _ptr(side, C.c_int8)))
    return boards, side


class Net:
    """A network on one device: the INeuralNet replacement."""

    def __init__(self, game: int, kind: int = GAT, device: int = 0, precision: int = PREC_AUTO,
                 max_batch: int = 4096):
        cfg = NetConfig(game, kind, precision, max_batch)
        h = _vp()
        _check(_lib.gz_net_create(C.byref(cfg), device, C.byref(h)))
        self._h = h
        self.game, self.kind, self.device, self.max_batch = game, kind, device, max_batch
        self.shape = game_shape(game)

    @property
    def handle(self) -> int:
        return self._h.value

    def close(self) -> None:
        if self._h:
            _lib.gz_net_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def weight_count(self) -> int:
        return int(_lib.gz_net_weight_count(self._h))

    @property
    def kernel_name(self) -> str:
        return _lib.gz_net_kernel_name(self._h).decode()

    def load_weights(self, blob: np.ndarray) -> None:
        blob = np.ascontiguousarray(blob, np.float32)
        _check(_lib.gz_net_load_weights(self._h, _ptr(blob, C.c_float), blob.size))

    def save_weights(self) -> np.ndarray:
        out = np.empty(self.weight_count(), np.float32)
        _check(_lib.gz_net_save_weights(self._h, _ptr(out, C.c_float), out.size))
        return out

    def predict_batch(self, d_boards, d_side, n: int, d_pi, d_v, stream=None) -> None:
        """Device-pointer batch evaluation (torch tensors or raw addresses)."""
        _check(_lib.gz_net_predict_batch(self._h, _dev(d_boards), _dev(d_side), n, _dev(d_pi), _dev(d_v),
                                         _stream(stream)))

    def check(self) -> None:
        """Raise if a bounded wait inside a forward kernel gave up."""
        _check(_lib.gz_net_check(self._h))

    def predict_host(self, boards: np.ndarray, side: np.ndarray,
                     out: tuple[np.ndarray, np.ndarray] | None = None) -> tuple[np.ndarray, np.ndarray]:
        """Host buffers in, host buffers out (synchronous).  `out` = (pi, v)
        reuses caller arrays (float32, C-contiguous, [n][actions] and [n]);
        page-locked arrays (see `pinned_empty`) are transferred directly."""
        boards = np.ascontiguousarray(boards, np.int8)
        side = np.ascontiguousarray(side, np.int8)
        n = side.shape[0]
        if out is None:
            pi = np.empty((n, self.shape.actions), np.float32)
            v = np.empty(n, np.float32)
        else:
            pi, v = out
            if (pi.dtype != np.float32 or v.dtype != np.float32 or not pi.flags.c_contiguous
                    or not v.flags.c_contiguous or pi.size < n * self.shape.actions or v.size < n):
                raise ValueError("out must be float32 C-contiguous arrays of at least [n][actions] and [n]")
        _check(_lib.gz_net_predict_host(self._h, boards.ctypes.data, side.ctypes.data, n, pi.ctypes.data,
                                        v.ctypes.data))
        return pi, v

    def predict(self, canonical_board: np.ndarray) -> tuple[np.ndarray, float]:
        """INeuralNet::predict: one canonical float board (own stones +1)."""
        b = np.ascontiguousarray(canonical_board, np.float32).reshape(-1)
        pi = np.empty(self.shape.actions, np.float32)
        v = np.empty(1, np.float32)
        _check(_lib.gz_net_predict(self._h, _ptr(b, C.c_float), _ptr(pi, C.c_float), _ptr(v, C.c_float)))
        return pi, float(v[0])

    def save_checkpoint(self, path: str) -> None:
        _check(_lib.gz_net_save_checkpoint(self._h, os.fsencode(path)))

    def load_checkpoint(self, path: str) -> None:
        _check(_lib.gz_net_load_checkpoint(self._h, os.fsencode(path)))

    def broadcast(self, comm: int, root: int = 0, stream=None) -> None:
        _check(_lib.gz_net_broadcast(self._h, comm, root, _stream(stream)))

    def loss_grad(self, d_boards, d_side, d_pi, d_v, n: int, d_grad=None, stream=None) -> tuple[float, float]:
        """Loss terms (policy cross-entropy, value squared error; batch means)
        of one batch of device buffers; the gradient (weight layout) into
        d_grad when given.  No update."""
        loss = np.zeros(2, np.float32)
        _check(_lib.gz_net_loss_grad(self._h, _dev(d_boards), _dev(d_side), _dev(d_pi), _dev(d_v), n,
                                     _dev(d_grad) if d_grad is not None else None, _ptr(loss, C.c_float),
                                     _stream(stream)))
        return float(loss[0]), float(loss[1])

    def train_step(self, d_boards, d_side, d_pi, d_v, n: int, cfg: TrainConfig | None = None, comm: int | None = None,
                   world: int = 1, stream=None) -> tuple[float, float]:
        """One Adam step on one batch of device buffers (gradients averaged
        over the ranks of `comm`); returns this batch's loss terms."""
        cfg = cfg or train_config()
        loss = np.zeros(2, np.float32)
        _check(_lib.gz_net_train_step(self._h, _dev(d_boards), _dev(d_side), _dev(d_pi), _dev(d_v), n, C.byref(cfg),
                                      comm, world, _ptr(loss, C.c_float), _stream(stream)))
        return float(loss[0]), float(loss[1])

    def train(self, examples: np.ndarray, cfg: TrainConfig | None = None, comm: int | None = None, rank: int = 0,
              world: int = 1) -> TrainStats:
        """INeuralNet::train over EXAMPLE_DTYPE records (canonical boards)."""
        ex = np.ascontiguousarray(examples, dtype=EXAMPLE_DTYPE)
        cfg = cfg or train_config()
        st = TrainStats()
        _check(_lib.gz_net_train(self._h, ex.ctypes.data if ex.size else None, ex.size, C.byref(cfg), comm, rank,
                                 world, C.byref(st)))
        return st


def train_config(**kw) -> TrainConfig:
    """The reference's training defaults (gz_train_config_default), with
    fields overridden by keyword."""
    c = TrainConfig()
    _lib.gz_train_config_default(C.byref(c))
    for k, val in kw.items():
        setattr(c, k, val)
    return c


def train_batch_indices(n: int, cfg: TrainConfig, epoch: int, step: int, rank: int = 0, world: int = 1) -> np.ndarray:
    """Example indices of one rank's batch (gz_net_train's order)."""
    out = np.zeros(cfg.batch_size, np.int64)
    _check(_lib.gz_train_batch_indices(n, C.byref(cfg), epoch, step, rank, world, _ptr(out, C.c_int64)))
    return out


def train_bucket_range(game: int, k: int) -> tuple[int, int]:
    """(offset, length) in floats of gradient bucket k (layers, then the heads)."""
    off, cnt = C.c_size_t(), C.c_size_t()
    _check(_lib.gz_train_bucket_range(game, k, C.byref(off), C.byref(cnt)))
    return off.value, cnt.value


def create_neural_net(net_type: str, game: int | str, device: int = 0, **kw) -> Net:
    """Factory mirroring create_neural_net (networks/neural_network.c:6-13)."""
    g = GAME_NAMES[game] if isinstance(game, str) else game
    kinds = {"gat": GAT, "resnet": RESNET}
    if net_type not in kinds:
        raise GZError(ERR_INVALID_ARG, f"unknown network type {net_type!r}")
    return Net(g, kinds[net_type], device=device, **kw)


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _check(_lib.gz_nccl_unique_id(buf))
    return bytes(buf)


def nccl_comm_init(uid: bytes, world: int, rank: int, device: int) -> int:
    buf = (C.c_uint8 * 128).from_buffer_copy(uid)
    comm = _vp()
    _check(_lib.gz_nccl_comm_init(buf, world, rank, device, C.byref(comm)))
    return comm.value


def nccl_comm_destroy(comm: int) -> None:
    _check(_lib.gz_nccl_comm_destroy(comm))


class Mcts:
    """Batched PUCT search over `trees` concurrent games on one device."""

    def __init__(self, game: int, trees: int, leaves_per_tree: int = 4, c_puct: float = 1.5, virtual_loss: int = 3,
                 node_capacity: int = 4096, dirichlet_alpha: float = 1.0, dirichlet_eps: float = 0.0,
                 seed: int = 0x6A5A, device: int = 0):
        cfg = MctsConfig(game, trees, leaves_per_tree, c_puct, virtual_loss, node_capacity, dirichlet_alpha,
                         dirichlet_eps, seed)
        h = _vp()
        _check(_lib.gz_mcts_create(C.byref(cfg), device, C.byref(h)))
        self._h = h
        self.game, self.trees, self.leaves, self.device = game, trees, leaves_per_tree, device
        self.shape = game_shape(game)

    def close(self) -> None:
        if self._h:
            _lib.gz_mcts_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def reset_roots(self, d_boards, d_side, stream=None) -> None:
        _check(_lib.gz_mcts_reset_roots(self._h, _dev(d_boards), _dev(d_side), _stream(stream)))

    def select(self, stream=None) -> None:
        _check(_lib.gz_mcts_select(self._h, _stream(stream)))

    def leaf_buffers(self) -> tuple[int, int, int]:
        b, s, t = _vp(), _vp(), _vp()
        _check(_lib.gz_mcts_leaf_buffers(self._h, C.byref(b), C.byref(s), C.byref(t)))
        return b.value, s.value, t.value

    def copy_leaves(self, stream=None) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        L = self.trees * self.leaves
        b = np.zeros((L, self.shape.board_bytes), np.int8)
        s = np.zeros(L, np.int8)
        t = np.zeros(L, np.int8)
        _check(_lib.gz_mcts_copy_leaves(self._h, _ptr(b, C.c_int8), _ptr(s, C.c_int8), _ptr(t, C.c_int8),
                                        _stream(stream)))
        return b, s, t

    def backup(self, d_pi, d_v, stream=None) -> None:
        _check(_lib.gz_mcts_backup(self._h, _dev(d_pi), _dev(d_v), _stream(stream)))

    def step(self, net: Net, stream=None) -> None:
        _check(_lib.gz_mcts_step(self._h, net._h, _stream(stream)))

    def run(self, net: Net, sims: int, stream=None) -> None:
        _check(_lib.gz_mcts_run(self._h, net._h, sims, _stream(stream)))

    def root_stats(self, stream=None) -> tuple[np.ndarray, np.ndarray]:
        visits = np.zeros((self.trees, self.shape.actions), np.int32)
        wsum = np.zeros((self.trees, self.shape.actions), np.float32)
        _check(_lib.gz_mcts_root_stats(self._h, _ptr(visits, C.c_int32), _ptr(wsum, C.c_float), _stream(stream)))
        return visits, wsum

    def tree_sizes(self, stream=None) -> tuple[np.ndarray, np.ndarray]:
        nodes = np.zeros(self.trees, np.int32)
        edges = np.zeros(self.trees, np.int32)
        _check(_lib.gz_mcts_tree_sizes(self._h, _ptr(nodes, C.c_int32), _ptr(edges, C.c_int32), _stream(stream)))
        return nodes, edges

    def choose(self, temp_moves: int, d_actions, stream=None) -> None:
        _check(_lib.gz_mcts_choose(self._h, temp_moves, _dev(d_actions), _stream(stream)))

    def play(self, d_actions, reserve: int, d_done=None, stream=None) -> None:
        _check(_lib.gz_mcts_play(self._h, _dev(d_actions), reserve, _dev(d_done), _stream(stream)))

    def check(self) -> None:
        _check(_lib.gz_mcts_check(self._h))


# TrainingExample of self_play/self_play.cuh:56-60 (gz_train_example): 516 bytes
EXAMPLE_DTYPE = np.dtype([("board", "<i4", 64), ("pi", "<f4", 64), ("v", "<f4")])
assert EXAMPLE_DTYPE.itemsize == 516


class SelfPlay:
    """Self-play episodes on every tree of a search handle (gz_selfplay_*)."""

    def __init__(self, mcts: Mcts, max_examples: int):
        h = _vp()
        _check(_lib.gz_selfplay_create(mcts._h, max_examples, C.byref(h)))
        self._h, self.mcts = h, mcts  # keeps the search handle alive

    def close(self) -> None:
        if self._h:
            _lib.gz_selfplay_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def run(self, net: Net, n_games: int, sims: int, temp_moves: int = 15, stream=None) -> None:
        _check(_lib.gz_selfplay_run(self._h, net._h, n_games, sims, temp_moves, _stream(stream)))

    def take(self) -> tuple[np.ndarray, int]:
        """The buffered examples (EXAMPLE_DTYPE records, in the order the games
        ended) and the number of games they come from; empties the buffer."""
        n, g = C.c_int64(), C.c_int64()
        # with no room the call only reports the counts (or, with nothing
        # buffered, succeeds and resets them)
        if _lib.gz_selfplay_take(self._h, None, 0, C.byref(n), C.byref(g)) == 0:
            return np.zeros(0, EXAMPLE_DTYPE), int(g.value)
        out = np.zeros(n.value, EXAMPLE_DTYPE)
        _check(_lib.gz_selfplay_take(self._h, out.ctypes.data, out.size, C.byref(n), C.byref(g)))
        return out, int(g.value)


def arena_play(mcts: Mcts, net_a: Net, net_b: Net, n_games: int, sims: int, stream=None) -> tuple[int, int, int]:
    """(games won by net_a, games won by net_b, draws); see gz_arena_play."""
    r = np.zeros(3, np.int32)
    _check(_lib.gz_arena_play(mcts._h, net_a._h, net_b._h, n_games, sims, _ptr(r[0:], C.c_int32),
                              _ptr(r[1:], C.c_int32), _ptr(r[2:], C.c_int32), _stream(stream)))
    return int(r[0]), int(r[1]), int(r[2])


def save_train_examples(path, iterations: list) -> None:
    """The reference's train_examples_*.bin layout (self_play.cu:510-534)."""
    arrs = [np.ascontiguousarray(a, dtype=EXAMPLE_DTYPE) for a in iterations]
    ptrs = (_vp * max(1, len(arrs)))(*[a.ctypes.data for a in arrs])
    counts = np.array([a.size for a in arrs] or [0], np.int32)
    _check(_lib.gz_train_examples_save(str(path).encode(), len(arrs), ptrs, _ptr(counts, C.c_int32)))


def load_train_examples(path) -> list:
    """Reads such a file back: one EXAMPLE_DTYPE array per iteration."""
    n_it, total = C.c_int(), C.c_int64()
    _check(_lib.gz_train_examples_load(str(path).encode(), None, 0, None, 0, C.byref(n_it), C.byref(total)))
    out = np.zeros(total.value, EXAMPLE_DTYPE)
    counts = np.zeros(max(1, n_it.value), np.int32)
    _check(_lib.gz_train_examples_load(str(path).encode(), out.ctypes.data, out.size, _ptr(counts, C.c_int32),
                                       n_it.value, C.byref(n_it), C.byref(total)))
    offs = np.concatenate([[0], np.cumsum(counts[:n_it.value])])
    return [out[offs[i]:offs[i + 1]] for i in range(n_it.value)]


# ---- reference-layout shim (include/graphzero_b200_compat.h) ----
_fn = C.CFUNCTYPE
_ip, _fp = C.POINTER(C.c_int), C.POINTER(C.c_float)


class IGame(C.Structure):
    pass


IGame._fields_ = [
    ("init", _fn(None, C.POINTER(IGame))),
    ("get_init_board", _fn(None, C.POINTER(IGame), _ip)),
    ("get_board_size", _fn(None, C.POINTER(IGame), _ip, _ip)),
    ("get_action_size", _fn(C.c_int, C.POINTER(IGame))),
    ("get_next_state", _fn(None, C.POINTER(IGame), _ip, C.c_int, C.c_int, _ip, _ip)),
    ("get_valid_moves", _fn(None, C.POINTER(IGame), _ip, C.c_int, C.POINTER(C.c_bool))),
    ("get_game_ended", _fn(C.c_int, C.POINTER(IGame), _ip, C.c_int)),
    ("get_canonical_form", _fn(None, C.POINTER(IGame), _ip, C.c_int, _ip)),
    ("evaluate", _fn(C.c_float, C.POINTER(IGame), _ip, C.c_int)),
    ("get_symmetries", _fn(None, C.POINTER(IGame), _ip, _fp, C.POINTER(C.c_int * 64), C.POINTER(C.c_float * 64), _ip)),
    ("string_representation", _fn(None, C.POINTER(IGame), _ip, C.c_char_p, C.c_int)),
    ("display", _fn(None, C.POINTER(IGame), _ip)),
]


class INeuralNet(C.Structure):
    pass


INeuralNet._fields_ = [
    ("impl", _vp),
    ("init", _fn(None, C.POINTER(INeuralNet), C.POINTER(IGame))),
    ("train", _fn(None, C.POINTER(INeuralNet), _vp, C.c_int)),
    ("predict", _fn(None, C.POINTER(INeuralNet), _fp, _fp, _fp)),
    ("save_checkpoint", _fn(None, C.POINTER(INeuralNet), C.c_char_p, C.c_char_p)),
    ("load_checkpoint", _fn(None, C.POINTER(INeuralNet), C.c_char_p, C.c_char_p)),
    ("destroy", _fn(None, C.POINTER(INeuralNet))),
    ("train_distributed", _fn(None, C.POINTER(INeuralNet), _fp, _fp, _fp, C.c_int, C.c_int, C.c_int, _vp, _vp)),
    ("broadcast_weights", _fn(None, C.POINTER(INeuralNet), C.c_int, C.c_int, _vp, _vp)),
]


def create_igame(name: str):
    """IGame vtable of `name` ('connect4' or 'tictactoe'); free with free_igame."""
    h = {"connect4": _lib.gz_create_connect4_game, "tictactoe": _lib.gz_create_tictactoe_game}[name]()
    if not h:
        raise GZError(ERR_INVALID_ARG, f"cannot create game {name}")
    return C.cast(h, C.POINTER(IGame))


def free_igame(g) -> None:
    _lib.gz_game_free(C.cast(g, _vp))


def create_ineuralnet(net_type: str, game, device: int = 0):
    """INeuralNet vtable (create_neural_net, networks/neural_network.c:6-13)."""
    h = _lib.gz_create_neural_net(net_type.encode(), C.cast(game, _vp), device)
    if not h:
        raise GZError(ERR_CUDA, _lib.gz_last_error().decode(errors="replace"))
    return C.cast(h, C.POINTER(INeuralNet))


def loaded_library_path() -> str:
    return os.fspath(LIB_PATH)
