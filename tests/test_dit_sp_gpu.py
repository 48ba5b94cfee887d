"""Sequence-parallel DiT (aex_dit_set_sequence_parallel) on 2 GPUs against the
one-GPU engine on the whole sequence: the small config (hidden 256 = 2 heads,
1 double + 2 single blocks, 32 text + 8x8 image tokens) split into two equal
contiguous shards (rank 0: the 32 text rows + 16 image rows; rank 1: 48 image
rows), joint attention over NCCL under the three exchange schedules (ring; one
all-gather; pairwise exchanges overlapped with per-shard attention), 3-step
denoise. Tolerance: relative L2 <= 2e-2 on each rank's
latents (bf16 activations; the ring merges per-hop bf16 partial outputs by
log-sum-exp). Skips with fewer than 2 GPUs."""
import ctypes as C
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L_TXT, GRID, STEPS = 32, 8, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg(l_txt, l_img):
    from aestrix_b200 import dit
    return dit.DitConfig(hidden=256, heads=2, n_double=1, n_single=2, mlp_hidden=768, in_channels=128,
                         text_dim=384, timestep_dim=256, l_txt=l_txt, l_img=l_img)


def _engine(cfg, ctx, dev, lin, norms, cos, sin, embeds):
    from aestrix_b200 import dit
    eng = dit.DitEngine(cfg, ctx=ctx, device=dev.index)
    eng.load(lin, norms)
    eng.set_rope(cos.contiguous(), sin.contiguous())
    eng.project_context(embeds)
    return eng


def _worker(rank, world, port, out_dir, schedule):
    os.environ["AEX_SP_SCHEDULE"] = schedule  # read at the first sequence-parallel call
    import torch.distributed as dist

    from aestrix_b200 import _lib, attention, dit

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=180))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    ctx = _lib.Context(rank)
    L = _lib.lib()
    J, l_img = L_TXT + GRID * GRID, GRID * GRID
    full = _cfg(L_TXT, l_img)
    lin, norms = dit.random_weights(full, seed=2024, device=dev)  # the same values on every GPU
    ids = torch.cat([attention.text_ids(L_TXT, dev), attention.grid_ids(GRID, GRID, 0.0, dev)]).contiguous()
    cos, sin = attention.rope_tables(ids, 2000.0, ctx=ctx)
    g = torch.Generator().manual_seed(7)
    embeds = torch.randn(L_TXT, full.text_dim, generator=g).to(torch.bfloat16).to(dev)
    lat = torch.randn(l_img, full.in_channels, generator=g).to(dev)
    # sequence shard of this rank (contiguous joint rows; text first)
    Jp = J // world
    r0, r1 = rank * Jp, (rank + 1) * Jp
    lt = max(0, min(L_TXT, r1) - r0)
    li = Jp - lt
    img0 = r0 + lt - L_TXT  # first image row of the shard
    uid = (C.c_char * 128)()
    if rank == 0:
        ctx.check(L.aex_comm_unique_id(uid))
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (C.c_char * 128).from_buffer_copy(obj[0])
    comm = C.c_void_p()
    ctx.check(L.aex_comm_create(ctx.handle, world, rank, uid, 60000, C.byref(comm)))
    eng = _engine(_cfg(lt, li), ctx, dev, lin, norms, cos[r0:r1], sin[r0:r1], embeds)
    eng.set_sequence_parallel(comm, L_TXT, l_img)
    x = lat[img0:img0 + li].clone()
    eng.denoise(x, steps=STEPS)
    ref_eng = _engine(full, ctx, dev, lin, norms, cos, sin, embeds)
    xr = ref_eng.denoise(lat.clone(), steps=STEPS)[img0:img0 + li]
    torch.cuda.synchronize()
    rel = float((x - xr).norm() / xr.norm())
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array([rel, float(torch.isfinite(x).all()),
                                                                   ctx.device_status(), li]))
    eng.close()
    ref_eng.close()
    L.aex_comm_destroy(comm)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("schedule", ["ring", "gather", "overlap"])
def test_dit_sequence_parallel_two_gpus(tmp_path, schedule):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), schedule), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        rel, finite, status, li = np.load(tmp_path / f"rank{r}.npy")
        assert finite == 1 and status == 0 and li > 0
        assert rel <= 2e-2, f"rank {r}: latents rel-L2 {rel:.3e}"
