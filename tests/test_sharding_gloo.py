"""Token sharding + parameter-gradient all-reduce across 2 gloo ranks on CPU.

Each rank runs the CPU oracle's backward on its own token shard (standing in
for the GPU kernel, whose per-shard results the GPU tests already pin) and
all-reduces the summed gradients; the result must equal the full-batch
gradient. A second test kills one rank before the collective and checks that
the survivor gets an error from the process-group timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from attnres_b200.sharding import allreduce_param_grads, token_shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_token_shard_covers_rows_exactly():
    for n in (0, 1, 7, 16384, 16385):
        for world in (1, 2, 3, 8):
            spans = [token_shard(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        token_shard(10, 2, 2)


def _inputs():
    rng = np.random.default_rng(5)
    S, N, D, R, H = 5, 37, 64, 16, 2
    return (rng.standard_normal((S, N, D)).astype(np.float32), rng.standard_normal((S, N, R)).astype(np.float32),
            rng.standard_normal((N, D)).astype(np.float32), rng.standard_normal((H, R // H)).astype(np.float32),
            np.full(H, 0.3, np.float32), rng.standard_normal((N, H, R // H)).astype(np.float32),
            rng.standard_normal(S).astype(np.float32), H)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from oracle import oracle

    v, k, g, q, gate, qd, bias, H = _inputs()
    a, b = token_shard(v.shape[1], rank, world)
    res = oracle.lrid_backward(v[:, a:b], k[:, a:b], H, 0.5, True, g[a:b], query=q, gate=gate,
                               query_dynamic=qd[a:b], logit_bias=bias)
    grads = [torch.tensor(res["dq"]), torch.tensor(res["dgate"]), torch.tensor(res["dbias"])]
    allreduce_param_grads(grads)
    out[rank] = [x.numpy().copy() for x in grads]
    dist.destroy_process_group()


def test_sharded_parameter_grads_equal_full_batch():
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
    from oracle import oracle

    v, k, g, q, gate, qd, bias, H = _inputs()
    full = oracle.lrid_backward(v, k, H, 0.5, True, g, query=q, gate=gate, query_dynamic=qd, logit_bias=bias)
    for rank in range(world):
        dq, dgate, dbias = out[rank]
        np.testing.assert_allclose(dq, full["dq"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(dgate, full["dgate"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(dbias, full["dbias"], rtol=1e-5, atol=1e-5)


def _dying_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    try:
        allreduce_param_grads([torch.ones(4)])
        out[rank] = "no error"
    except Exception as e:  # gloo reports the lost peer or the timeout
        out[rank] = "error: " + type(e).__name__


def test_lost_rank_surfaces_as_an_error_not_a_hang():
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert all(not p.is_alive() for p in procs)
    assert str(out.get(0, "")).startswith("error"), out.get(0)
