"""CPU (gloo, world size 2 and 3) test of the ring-attention algorithm used by
aex_ring_attention: contiguous sequence shards, K/V passed to rank r+1 each hop,
partial results merged by their log2-sum-exp, against the full-sequence oracle.
Mirrors the hop/peer schedule and the merge formula of
aestrix_b200/csrc/ring_attention.cpp and ring_kernels.cu on numpy arrays."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial(q, k, v, scale):
    """Normalized partial attention and per-row log2-sum-exp ([S, H] each row/head)."""
    sc = np.einsum("shd,thd->hst", q, k).astype(np.float64) * scale
    m = sc.max(-1, keepdims=True)
    p = np.exp(sc - m)
    l = p.sum(-1, keepdims=True)
    o = np.einsum("hst,thd->shd", p / l, v)
    lse2 = (m[..., 0] + np.log(l[..., 0])) / np.log(2.0)  # [H, S]
    return o, lse2


def _merge(o_acc, lse_acc, o_h, lse_h):
    mx = np.maximum(lse_acc, lse_h)
    wa, wh = np.exp2(lse_acc - mx), np.exp2(lse_h - mx)
    lse = mx + np.log2(wa + wh)
    o = (o_acc * wa.T[..., None] + o_h * wh.T[..., None]) / (wa + wh).T[..., None]
    return o, lse


def _worker(rank, world, port, S, H, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((S, H, 128)).astype(np.float32) for _ in range(3))
    Sp = S // world
    sl = slice(rank * Sp, (rank + 1) * Sp)
    ql, kv = q[sl], np.stack([k[sl], v[sl]])
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    o_acc = lse_acc = None
    for hop in range(world):
        src = (rank - hop) % world  # owner of the shard in hand
        if hop + 1 < world:  # ring exchange: send to rank+1, receive from rank-1
            recv = torch.empty(kv.shape, dtype=torch.float32)
            reqs = [dist.isend(torch.from_numpy(kv), nxt), dist.irecv(recv, prv)]
        o_h, lse_h = _partial(ql, kv[0], kv[1], 1 / np.sqrt(128))
        assert np.array_equal(kv[0], k[src * Sp:(src + 1) * Sp])
        o_acc, lse_acc = (o_h, lse_h) if hop == 0 else _merge(o_acc, lse_acc, o_h, lse_h)
        if hop + 1 < world:
            for r in reqs:
                r.wait()
            kv = recv.numpy()
    ref = O.sdpa(q[None], k[None], v[None], 1 / np.sqrt(128))[0]
    result[rank] = float(np.abs(o_acc - ref[sl]).max())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ring_schedule_and_merge_gloo(world):
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), 96 * world, 2, result), nprocs=world, join=True,
                       start_method="spawn")
    assert len(result) == world
    assert max(result.values()) < 1e-5, dict(result)
