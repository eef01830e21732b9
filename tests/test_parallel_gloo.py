"""Multi-process (world_size 2 and 3, gloo, CPU) tests of the pipeline stage handoff,
the row-parallel all-reduce, V-head sharding, and failure detection on the
host (a peer that disappears makes the receiver error out, never hang)."""
import multiprocessing as mp
import socket

import pytest

import _gloo_workers as W


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(target, *args, world=2, timeout=120, expect=0):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    codes = []
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            codes.append("hung")
        else:
            codes.append(p.exitcode)
    return codes


@pytest.mark.parametrize("mode", ["packed", "presum"])
def test_pipeline_handoff(mode):
    assert _run(W.handoff_worker, mode) == [0, 0]


def test_pipeline_handoff_three_stages_boundary_groups():
    """A middle stage receives and sends on different two-rank groups."""
    assert _run(W.handoff_chain_worker, world=3) == [0, 0, 0]


def test_handoff_peer_death_is_detected():
    codes = _run(W.handoff_peer_dies_worker, timeout=60)
    assert codes == [0, 0], codes


def test_row_parallel_all_reduce():
    assert _run(W.row_parallel_worker) == [0, 0]


def test_head_sharded_layer_matches_single_process():
    assert _run(W.head_sharded_layer_worker, timeout=300) == [0, 0]
