"""Multi-GPU paths over NCCL (one spawned process per GPU): the V-head sharded
layer against the unsharded layer, and the pipeline stage handoff between
GPUs.  Skipped on a box with fewer than two GPUs."""
import multiprocessing as mp
import socket

import pytest
import torch

import _nccl_workers as W

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(target, *args, world=2, timeout=300):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args) for r in range(world)]
    for p in procs:
        p.start()
    codes = []
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            codes.append("hung")
        else:
            codes.append(p.exitcode)
    return codes


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("D", [128, 64])     # tensor-core and fp32 prefill kernels
def test_tp2_head_sharded_layer_nccl(D):
    _need(2)
    assert _run(W.tp_layer_worker, D) == [0, 0]


@pytest.mark.parametrize("mode", ["packed", "presum"])
def test_pipeline_handoff_nccl(mode):
    _need(2)
    assert _run(W.nccl_handoff_worker, mode) == [0, 0]


@pytest.mark.parametrize("D", [128, 64])
def test_tp4_head_sharded_layer_nccl(D):
    """Four TP ranks: one k-head and two v-heads each."""
    _need(4)
    assert _run(W.tp_layer_worker, D, world=4) == [0, 0, 0, 0]


@pytest.mark.parametrize("mode", ["packed", "presum"])
def test_pipeline_handoff_nccl_4_stages(mode):
    _need(4)
    assert _run(W.nccl_handoff_worker, mode, world=4) == [0, 0, 0, 0]


@pytest.mark.parametrize("D", [128, 64])
def test_tp8_head_sharded_layer_nccl(D):
    """Eight TP ranks: one k-head and two v-heads each (16 v-heads total)."""
    _need(8)
    assert _run(W.tp_layer_worker, D, 8, 16, world=8) == [0] * 8


@pytest.mark.parametrize("mode", ["packed", "presum"])
def test_pipeline_handoff_nccl_8_stages(mode):
    _need(8)
    assert _run(W.nccl_handoff_worker, mode, world=8) == [0] * 8
