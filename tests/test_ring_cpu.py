"""CPU (gloo, world size 2 to 4) tests of the exchange schedules of
aex_ring_attention against the full-sequence oracle, on contiguous sequence
shards:
* overlap (the default for more than one rank): the plan comes from the
  library itself (aex_sp_plan, the host logic ring_attention.cpp runs on the
  GPU path), and each rank executes its steps in order with gloo point-to-point
  transfers and numpy attention partials, merged with the formula of
  merge_splits_kernel;
* the ring (K/V passed to rank r+1 each hop, partial results merged by their
  log2-sum-exp; the hop/peer schedule and merge formula of
  aestrix_b200/csrc/ring_attention.cpp and ring_kernels.cu);
* the all-gather (every rank's K/V written token-major into slot r of one
  buffer, gathered in place, then one attention over all keys).
Also the schedule choice of aex_sp_schedule (host logic, no GPU)."""
import subprocess
import sys
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


def _gather_worker(rank, world, port, S, H, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(4)
    q, k, v = (rng.standard_normal((S, H, 128)).astype(np.float32) for _ in range(3))
    Sp = S // world
    sl = slice(rank * Sp, (rank + 1) * Sp)
    # K_all / V_all [world * Sp][H][128]; this rank fills its slot, the gather fills the rest.
    k_all = torch.zeros(world * Sp, H, 128)
    v_all = torch.zeros(world * Sp, H, 128)
    k_all[sl] = torch.from_numpy(k[sl])
    v_all[sl] = torch.from_numpy(v[sl])
    for buf in (k_all, v_all):  # in place: rank r's input is its own slot of the output
        parts = list(buf.view(world, Sp, H, 128).unbind(0))
        dist.all_gather(parts, parts[rank].clone())
    assert np.array_equal(k_all.numpy(), k) and np.array_equal(v_all.numpy(), v)
    o, _ = _partial(q[sl], k_all.numpy(), v_all.numpy(), 1 / np.sqrt(128))
    ref = O.sdpa(q[None], k[None], v[None], 1 / np.sqrt(128))[0]
    result[rank] = float(np.abs(o - ref[sl]).max())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_schedule_gloo(world):
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_gather_worker, args=(world, _free_port(), 96 * world, 2, result), nprocs=world, join=True,
                       start_method="spawn")
    assert len(result) == world
    assert max(result.values()) < 1e-5, dict(result)


def _overlap_worker(rank, world, port, S, H, result):
    from aestrix_b200 import _lib

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(5)
    q, k, v = (rng.standard_normal((S, H, 128)).astype(np.float32) for _ in range(3))
    Sp = S // world
    sl = slice(rank * Sp, (rank + 1) * Sp)
    slots = {rank: np.stack([k[sl], v[sl]])}  # K/V slot r: rank r's shard, as in K_all / V_all
    landed = {}  # exchange index -> slot it filled
    parts = {}
    out = None
    for op in _lib.sp_plan(world, rank):
        if op.kind == _lib.AEX_SP_OP_EXCHANGE:
            recv = torch.empty((2, Sp, H, 128), dtype=torch.float32)
            reqs = [dist.isend(torch.from_numpy(slots[rank]), op.send_to), dist.irecv(recv, op.recv_from)]
            for r in reqs:
                r.wait()
            assert op.recv_from not in slots
            slots[op.recv_from] = recv.numpy()
            landed[op.part] = op.recv_from
        elif op.kind == _lib.AEX_SP_OP_ATTEND:
            if op.wait_exchange >= 0:  # reads exactly the shard that exchange delivered
                assert landed[op.wait_exchange] == op.slot
            else:
                assert op.slot == rank
            kv = slots[op.slot]
            assert np.array_equal(kv[0], k[op.slot * Sp:(op.slot + 1) * Sp])
            assert op.part not in parts
            parts[op.part] = _partial(q[sl], kv[0], kv[1], 1 / np.sqrt(128))
        else:  # merge_splits_kernel: sum_r 2^(lse_r - max) o_r / sum_r 2^(lse_r - max)
            assert sorted(parts) == list(range(op.part)) and op.part == world
            lse = np.stack([parts[r][1] for r in range(op.part)])  # [P, H, S]
            w = np.exp2(lse - lse.max(0, keepdims=True))
            out = sum(w[r].T[..., None] * parts[r][0] for r in range(op.part)) / w.sum(0).T[..., None]
    assert sorted(slots) == list(range(world))
    ref = O.sdpa(q[None], k[None], v[None], 1 / np.sqrt(128))[0]
    result[rank] = float(np.abs(out - ref[sl]).max())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_overlap_plan_gloo(world):
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_overlap_worker, args=(world, _free_port(), 64 * world, 2, result), nprocs=world, join=True,
                       start_method="spawn")
    assert len(result) == world
    assert max(result.values()) < 1e-5, dict(result)


def test_overlap_plan_shape():
    """Every rank's plan: the local shard's attention first, P - 1 exchanges whose pairs match across ranks
    (rank r sends to r + h exactly when rank r + h receives from r in the same exchange h), one attention per
    shard on alternating streams, one merge of all P partials; bad arguments give -1."""
    from aestrix_b200 import _lib

    for world in (1, 2, 5, 8, 16):
        plans = [_lib.sp_plan(world, r) for r in range(world)]
        for r, plan in enumerate(plans):
            kinds = [op.kind for op in plan]
            assert kinds == [1] + [0] * (world - 1) + [1] * (world - 1) + [2]
            assert plan[0].slot == r and plan[0].wait_exchange == -1 and plan[0].part == 0
            for op in plan[1:world]:
                h = op.part
                peer = plans[op.send_to][h]
                assert peer.kind == 0 and peer.recv_from == r
            attends = plan[world:2 * world - 1]
            assert sorted(op.slot for op in plan if op.kind == 1) == list(range(world))
            assert [op.stream for op in attends] == [h & 1 for h in range(1, world)]
            assert plan[-1].part == world
    L = _lib.lib()
    assert L.aex_sp_plan(17, 0, None, 0) == -1
    assert L.aex_sp_plan(4, 4, None, 0) == -1
    assert L.aex_sp_plan(4, 1, (_lib.aex_sp_op * 2)(), 2) == -1  # too few entries


_SCHEDULE_PROBE = (
    "import sys; sys.path.insert(0, sys.argv[1]); from aestrix_b200 import _lib; L = _lib.lib(); "
    "print(L.aex_sp_schedule(8, 2112, 24), L.aex_sp_schedule(2, 8448, 24), L.aex_sp_schedule(8, 1 << 20, 24), "
    "L.aex_sp_schedule(1, 2112, 24), L.aex_sp_schedule(0, 2112, 24), L.aex_sp_schedule(2, 0, 24))")


@pytest.mark.parametrize("env,want", [(None, "1 2 0 1 -1 -1"), ("ring", "0 0 0 0 -1 -1"), ("gather", "1 1 1 1 -1 -1"),
                                      ("overlap", "2 2 2 2 -1 -1")])
def test_sp_schedule_choice(env, want):
    """While the gathered K/V (2 * world * seq * heads * 256 bytes) fit in 8 GiB: overlap at two ranks,
    all-gather at one or more than two; ring beyond; AEX_SP_SCHEDULE overrides. Each case in a fresh process:
    the override is read once."""
    e = {k: v for k, v in os.environ.items() if k != "AEX_SP_SCHEDULE"}
    if env:
        e["AEX_SP_SCHEDULE"] = env
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", _SCHEDULE_PROBE, root], env=e, capture_output=True, text=True,
                         timeout=120, check=True).stdout.split()
    assert " ".join(out) == want


@pytest.mark.parametrize("k", [2, 3, 4])
def test_key_range_merge(k):
    """The gather schedule's split attention: k contiguous key ranges, each a normalized partial with its
    log2-sum-exp, combined as sum_r 2^(lse_r - max) o_r / sum_r 2^(lse_r - max) (merge_splits_kernel in
    aestrix_b200/csrc/ring_kernels.cu), equals attention over all keys."""
    rng = np.random.default_rng(11 + k)
    S, T, H = 40, 128 * 3 * k + 37, 2  # 3k + 1 key blocks, the last one ragged
    q, kk, v = (rng.standard_normal((n, H, 128)).astype(np.float32) for n in (S, T, T))
    blocks = (T + 127) // 128
    per = -(-blocks // k)  # whole 128-key blocks per range, every range non-empty
    assert (k - 1) * per < blocks
    rng_keys = [slice(r * per * 128, min(T, (r + 1) * per * 128)) for r in range(k)]
    parts = [_partial(q, kk[sl], v[sl], 1 / np.sqrt(128)) for sl in rng_keys]
    lse = np.stack([p[1] for p in parts])  # [k, H, S]
    w = np.exp2(lse - lse.max(0, keepdims=True))
    out = sum(w[r].T[..., None] * parts[r][0] for r in range(k)) / w.sum(0).T[..., None]
    ref = _partial(q, kk, v, 1 / np.sqrt(128))[0]
    assert float(np.abs(out - ref).max()) < 1e-5


@pytest.mark.parametrize("world,seq,heads,sms,want", [
    (8, 2112, 24, 148, 2),   # 216 CTAs = 1.46 waves -> 432 = 2.92
    (4, 4224, 24, 148, 1),   # 408 CTAs = 2.76 waves: a split fills no better
    (2, 8448, 24, 148, 2),   # 792 CTAs = 5.35 waves -> 1584 = 10.7
    (1, 384, 2, 148, 1),     # 3 key blocks: no range of at least 8 blocks
    (0, 2112, 24, 148, -1),  # bad arguments
    (8, 2112, 24, 0, -1),
])
def test_sp_key_ranges(world, seq, heads, sms, want):
    """Key ranges of the gather schedule's attention: the smallest split (<= 4) whose wave fill beats no split
    by more than 5 points, ranges of at least 8 key blocks."""
    from aestrix_b200 import _lib
    assert _lib.lib().aex_sp_key_ranges(world, seq, heads, sms) == want


@pytest.mark.parametrize("world", [2, 3])
def test_ring_schedule_and_merge_gloo(world):
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), 96 * world, 2, result), nprocs=world, join=True,
                       start_method="spawn")
    assert len(result) == world
    assert max(result.values()) < 1e-5, dict(result)
