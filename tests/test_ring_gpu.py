"""aex_ring_attention on 2 GPUs (one process per GPU, NCCL over NVLink) against
the full-sequence oracle: fused QK-RMSNorm + RoPE + SDPA of the joint sequence
split into contiguous shards, under the three exchange schedules (ring of
point-to-point hops; one all-gather; pairwise exchanges overlapped with
per-shard attention); the 2-rank cases skip on a box with fewer than 2 GPUs. On one GPU, a 1-rank communicator runs the all-gather
schedule's attention split into key ranges.
Tolerance: relative L2 <= 1e-2, max-abs <= 2e-2 (as the single-GPU attention)."""
import ctypes as C
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, l_txt, grid, heads, out_dir, schedule):
    os.environ["AEX_SP_SCHEDULE"] = schedule  # read at the first sequence-parallel call
    import torch.distributed as dist

    from aestrix_b200 import _lib, attention
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(rank)
    ctx = _lib.Context(rank)
    L = _lib.lib()
    uid = (C.c_char * 128)()
    if rank == 0:
        ctx.check(L.aex_comm_unique_id(uid))
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (C.c_char * 128).from_buffer_copy(obj[0])
    comm = C.c_void_p()
    ctx.check(L.aex_comm_create(ctx.handle, world, rank, uid, 60000, C.byref(comm)))
    S = l_txt + grid * grid
    Sp = S // world
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(1, S, heads, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    wq = (1 + 0.1 * torch.randn(128, generator=g)).float()
    wk = (1 + 0.1 * torch.randn(128, generator=g)).float()
    ids = np.concatenate([O.text_ids(l_txt), O.grid_ids(grid, grid)], 0)
    cos, sin = O.rope_freqs(ids, 2000.0)
    sl = slice(rank * Sp, (rank + 1) * Sp)
    dev = torch.device("cuda", rank)
    ql, kl, vl = (t[:, sl].contiguous().to(dev) for t in (q, k, v))
    cl, sn = torch.from_numpy(cos[sl]).to(dev), torch.from_numpy(sin[sl]).to(dev)
    out = torch.empty_like(ql)
    a = attention.make_args(ql, kl, vl, out, "bshd", wq.to(dev), wk.to(dev), 1e-5, cl, sn)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(2):  # twice: the second call reuses the ring buffers
        ctx.check(L.aex_ring_attention(ctx.handle, comm, C.byref(a), stream))
    ctx.sync(stream, timeout_ms=60000)
    got = out.float().cpu().numpy()
    rows = np.r_[0:32, Sp - 32:Sp]
    ref = O.joint_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), wq.numpy(), wk.numpy(), 1e-5,
                            cos, sin, q_begin=rank * Sp, q_end=(rank + 1) * Sp)[:, sl]
    d = got[:, rows] - ref[:, rows]
    rel = float(np.linalg.norm(d) / np.linalg.norm(ref[:, rows]))
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array([rel, float(np.abs(d).max()), ctx.device_status()]))
    L.aex_comm_destroy(comm)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("schedule", ["ring", "gather", "overlap"])
@pytest.mark.parametrize("l_txt,grid,heads", [(64, 24, 4), (512, 128, 2)])
def test_ring_attention_two_gpus(tmp_path, l_txt, grid, heads, schedule):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _free_port(), l_txt, grid, heads, str(tmp_path), schedule), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        rel, mx, status = np.load(tmp_path / f"rank{r}.npy")
        assert status == 0
        assert rel <= 1e-2 and mx <= 2e-2, f"rank {r}: rel-L2 {rel:.3e} max-abs {mx:.3e}"


def test_single_rank_gather_with_key_ranges():
    """One GPU, a 1-rank communicator: the gather schedule's attention over a 2,112-row shard with 24 heads
    (216 CTAs, under 1.5 waves of 148 SMs) runs as two key ranges merged by log-sum-exp (aex_sp_schedule says
    gather; the split is chosen from the SM count). Against the oracle on 64 rows, same tolerance."""
    from aestrix_b200 import _lib, attention
    from oracle import oracle as O

    L = _lib.lib()
    ctx = _lib.Context(0)
    dev = torch.device("cuda", 0)
    uid = (C.c_char * 128)()
    ctx.check(L.aex_comm_unique_id(uid))
    comm = C.c_void_p()
    ctx.check(L.aex_comm_create(ctx.handle, 1, 0, uid, 60000, C.byref(comm)))
    try:
        S, H = 2112, 24
        assert L.aex_sp_schedule(1, S, H) == 1
        g = torch.Generator().manual_seed(9)
        q, k, v = (torch.randn(1, S, H, 128, generator=g).to(torch.bfloat16) for _ in range(3))
        wq = (1 + 0.1 * torch.randn(128, generator=g)).float()
        wk = (1 + 0.1 * torch.randn(128, generator=g)).float()
        ang = (torch.rand(S, 64, generator=g) * 6.2831853).double()
        cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
        qd, kd, vd = (t.to(dev) for t in (q, k, v))
        out = torch.empty_like(qd)
        a = attention.make_args(qd, kd, vd, out, "bshd", wq.to(dev), wk.to(dev), 1e-5, cos.to(dev), sin.to(dev))
        stream = torch.cuda.current_stream(dev).cuda_stream
        for _ in range(2):
            ctx.check(L.aex_ring_attention(ctx.handle, comm, C.byref(a), stream))
        ctx.sync(stream, timeout_ms=60000)
        assert ctx.device_status() == 0
        args = (q.float().numpy(), k.float().numpy(), v.float().numpy(), wq.numpy(), wk.numpy(), 1e-5,
                cos.numpy(), sin.numpy())
        ref = np.concatenate([O.joint_attention(*args, q_begin=0, q_end=32)[:, :32],
                              O.joint_attention(*args, q_begin=S - 32, q_end=S)[:, S - 32:]], 1)
        got = out.float().cpu().numpy()[:, np.r_[0:32, S - 32:S]]
        d = got - ref
        rel = float(np.linalg.norm(d) / np.linalg.norm(ref))
        assert rel <= 1e-2 and float(np.abs(d).max()) <= 2e-2, f"rel-L2 {rel:.3e} max-abs {np.abs(d).max():.3e}"
    finally:
        L.aex_comm_destroy(comm)


def test_sequence_parallel_call_rejects_bad_args():
    """aex_ring_attention applies the same argument checks as aex_joint_attention before any launch: a NULL or
    misaligned tensor comes back as AEX_ERR_INVALID_ARG with a message, not as a device fault."""
    from aestrix_b200 import _lib, attention

    L = _lib.lib()
    ctx = _lib.Context(0)
    dev = torch.device("cuda", 0)
    uid = (C.c_char * 128)()
    ctx.check(L.aex_comm_unique_id(uid))
    comm = C.c_void_p()
    ctx.check(L.aex_comm_create(ctx.handle, 1, 0, uid, 60000, C.byref(comm)))
    try:
        q, k, v = (torch.randn(1, 256, 2, 128, device=dev).to(torch.bfloat16) for _ in range(3))
        out = torch.empty_like(q)
        a = attention.make_args(q, k, v, out, "bshd")
        a.q.data = None
        rc = L.aex_ring_attention(ctx.handle, comm, C.byref(a), None)
        assert rc == _lib.AEX_ERR_INVALID_ARG
        assert b"q.data" in L.aex_last_error_string(ctx.handle)
        a = attention.make_args(q, k, v, out, "bshd")
        a.k.data = k.data_ptr() + 2  # not 16-byte aligned
        rc = L.aex_ring_attention(ctx.handle, comm, C.byref(a), None)
        assert rc == _lib.AEX_ERR_INVALID_ARG
        assert ctx.device_status() == 0
    finally:
        L.aex_comm_destroy(comm)
