"""The allocation-free Connect4 entry point (gz_gat_c4_predict_noalloc).

Some callers cannot allocate device memory: a plugin inside a host
application that owns the CUDA context and fixes the device-memory budget,
or a latency-critical loop that cannot pay for a synchronising cudaMalloc.
This entry point stages everything in one static device array instead.

It runs the same tensor-core kernel, in the same operand format, as a gz_net
made with PREC_AUTO, so the outputs agree to 1e-6 max-abs (in practice bit
for bit), and like that net it stays within the spec's 1e-3 of the CPU
oracle.  Two calls in a row, with different weights, positions and batch
sizes, check that the second call finds nothing stale from the first in the
shared device array, and the device's free memory is the same before and
after a call.  This file is collected last so that it runs both alone in a
fresh process and after every other GPU test.
"""
import numpy as np
import pytest
import torch

import graphzero_b200 as gz
import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-6         # against the gz_net path: the same kernel and format
ORACLE_TOL = 1e-3  # against the CPU oracle: the spec's bound


def reference_call(w, boards, side):
    net = gz.Net(gz.CONNECT4, precision=gz.PREC_AUTO, max_batch=4096)
    net.load_weights(w)
    return net.predict_host(boards, side)


def test_noalloc_matches_predict_host_twice(cuda):
    assert gz.gat_c4_noalloc_max_batch() == 4096
    calls = [(11, 4096), (12, 1000)]  # (seed, batch): the second call is smaller than the first
    for k, (seed, n) in enumerate(calls):
        w = gz.synth_weights(gz.CONNECT4, seed=seed, bias_scale=0.4)
        boards, side = gz.synth_positions(gz.CONNECT4, n, seed=200 + seed)
        torch.cuda.synchronize()
        free_before, _ = torch.cuda.mem_get_info(0)
        pi, v = gz.gat_c4_predict_noalloc(w, boards, side)
        free_after, _ = torch.cuda.mem_get_info(0)
        if k > 0:  # the first call may still load the library's kernels (lazy module loading)
            assert free_after == free_before, (free_before, free_after)
        rpi, rv = reference_call(w, boards, side)
        assert pi.shape == (n, 7) and v.shape == (n,)
        assert np.isfinite(pi).all() and np.isfinite(v).all()
        assert np.abs(pi - rpi).max() <= TOL
        assert np.abs(v - rv).max() <= TOL
        opi, ov = oracle.gat_forward(gz.CONNECT4, w, boards, side)
        assert np.abs(pi - opi).max() < ORACLE_TOL and np.abs(v - ov).max() < ORACLE_TOL


def test_noalloc_rejects_oversize_and_bad_blob(cuda):
    w = gz.synth_weights(gz.CONNECT4, seed=3)
    boards, side = gz.synth_positions(gz.CONNECT4, 4097, seed=5)
    with pytest.raises(gz.GZError, match="at most 4096"):
        gz.gat_c4_predict_noalloc(w, boards, side)
    with pytest.raises(gz.GZError, match="GAT blob"):
        gz.gat_c4_predict_noalloc(w[:-1], boards[:8], side[:8])
    # the scratch still works after the rejected calls
    pi, v = gz.gat_c4_predict_noalloc(w, boards[:64], side[:64])
    rpi, rv = reference_call(w, boards[:64], side[:64])
    assert np.abs(pi - rpi).max() <= TOL and np.abs(v - rv).max() <= TOL
