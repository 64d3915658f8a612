"""The C ABI without a GPU: every declared symbol is exported, argument
errors come back as status codes with messages, and no call exits."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import graphzero_b200 as gz
import oracle

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"^\s*[\w\s\*]+?\b(gz_\w+)\s*\(", text, flags=re.M))
    return sorted(names)


def test_header_symbols_exported():
    names = declared_functions()
    assert len(names) >= 30
    lib = C.CDLL(str(gz.LIB_PATH))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python mirror binds every one of them
    assert set(names) <= set(gz.EXPORTED_SYMBOLS)


def test_weight_counts_match_oracle():
    for g in (gz.TICTACTOE, gz.CONNECT4, gz.CHESS):
        assert gz.weight_count(g, gz.GAT) == oracle.lib().orc_gat_weight_count(g)
    assert gz.weight_count(gz.CONNECT4, gz.RESNET) == oracle.lib().orc_res_weight_count()
    assert gz.weight_count(gz.TICTACTOE, gz.RESNET) == 0


def test_synth_weights_deterministic_and_bf16_exact():
    a = gz.synth_weights(gz.CONNECT4, seed=3, bias_scale=0.1)
    b = gz.synth_weights(gz.CONNECT4, seed=3, bias_scale=0.1)
    assert (a == b).all()
    bits = a.view(np.uint32)
    assert (bits & 0xFFFF == 0).all()
    c = gz.synth_weights(gz.CONNECT4, seed=3, bf16_exact=False)
    assert (c.view(np.uint32) & 0xFFFF != 0).any()
    # Glorot bound of the first layer: sqrt(6 / (4 + 256))
    assert np.abs(c[:4 * 256]).max() <= np.sqrt(6 / 260) + 1e-6


def test_invalid_arguments_are_reported():
    with pytest.raises(gz.GZError) as e:
        gz.game_shape(7)
    assert e.value.status == gz.ERR_INVALID_ARG and "bad game" in str(e.value)
    with pytest.raises(gz.GZError):
        gz.synth_weights(gz.TICTACTOE, gz.RESNET)
    b, s = gz.synth_positions(gz.CHESS, 2)
    with pytest.raises(gz.GZError) as e:
        gz.chess_perft(b[0], int(s[0]), 7)
    assert e.value.status == gz.ERR_INVALID_ARG
    with pytest.raises(gz.GZError) as e:
        gz.chess_legal_count(b[0], 0)
    assert e.value.status == gz.ERR_INVALID_ARG
    lib = C.CDLL(str(gz.LIB_PATH))
    assert gz._lib.gz_net_predict_batch(None, None, None, 4, None, None, None) == gz.ERR_INVALID_ARG
    assert gz._lib.gz_mcts_select(None, None) == gz.ERR_INVALID_ARG
    assert lib.gz_status_string(6) is not None


def test_create_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(gz.GZError) as e:
        gz.Net(gz.CONNECT4)
    assert e.value.status in (gz.ERR_CUDA, gz.ERR_INVALID_ARG)
    with pytest.raises(gz.GZError):
        gz.Mcts(gz.CONNECT4, trees=4)


def test_mcts_config_validation():
    cfg = gz.MctsConfig(7, 4, 4, 1.5, 3, 64, 1.0, 0.0, 1)  # no such game
    h = C.c_void_p()
    assert gz._lib.gz_mcts_create(C.byref(cfg), 0, C.byref(h)) == gz.ERR_INVALID_ARG
    cfg = gz.MctsConfig(gz.CONNECT4, 0, 4, 1.5, 3, 64, 1.0, 0.0, 1)
    assert gz._lib.gz_mcts_create(C.byref(cfg), 0, C.byref(h)) == gz.ERR_INVALID_ARG
