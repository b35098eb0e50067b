"""Ulysses sequence parallelism on 2 GPUs: wx_dit_block_forward_sp over NCCL
against the single-GPU block on the same inputs (dense, SOL and top-k
attention; refresh and PAB reuse). Skipped on boxes with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, sparse_name, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from tests._util import cosine, f32, max_rel_err, to_np_bf16, to_torch_bf16
        from tests.test_gpu_block import gpu_block, make_block
        from wuxianhuabu_b200 import h3
        hidden, heads, ffn, rot, eps, g = 256, 2, 512, 96, 1e-6, 40
        S = 512
        w, mods, h, cos, sin, rowmap = make_block(9, hidden, heads, ffn, 0, S, rot)
        sparse = {"dense": None, "sol": dict(tau=0.4), "topk": dict(block=128, topk_ratio=0.25, tail=False)}[sparse_name]
        spec = None if sparse is None else h3.H3SolAttnConfig(**sparse).spec(g)
        blk = gpu_block(w, hidden, heads, ffn, 0, rot, eps)
        md = [to_torch_bf16(m, dev) for m in mods]
        rm = torch.from_numpy(rowmap.view(np.int32)).to(dev)
        c, s = to_torch_bf16(cos, dev), to_torch_bf16(sin, dev)
        # single-GPU reference on this device (before the communicator exists)
        ref = to_torch_bf16(h, dev)
        slot_ref = torch.empty((S, hidden), dtype=torch.bfloat16, device=dev)
        blk.block_forward(0, ref, md, rm, c, s, spec, pab_slot=slot_ref, refresh=True)
        ref2 = ref.clone()
        blk.block_forward(0, ref2, md, rm, c, s, spec, pab_slot=slot_ref, refresh=False)
        torch.cuda.synchronize()

        def bcast(obj):
            box = [obj]
            dist.broadcast_object_list(box, src=0)
            return box[0]
        h3.init_sequence_parallel(world, rank, bcast)
        rows = S // world
        r0 = rank * rows
        hl = to_torch_bf16(h, dev)[r0:r0 + rows].contiguous()
        slot = torch.empty((rows, hidden), dtype=torch.bfloat16, device=dev)
        blk2 = gpu_block(w, hidden, heads, ffn, 0, rot, eps)
        blk2.block_forward(0, hl, md, rm[r0:r0 + rows].contiguous(), c[r0:r0 + rows].contiguous(),
                           s[r0:r0 + rows].contiguous(), spec, pab_slot=slot, refresh=True, S_total=S)
        hl2 = hl.clone()
        blk2.block_forward(0, hl2, md, rm[r0:r0 + rows].contiguous(), c[r0:r0 + rows].contiguous(),
                           s[r0:r0 + rows].contiguous(), spec, pab_slot=slot, refresh=False, S_total=S)
        torch.cuda.synchronize()
        h3.context(rank).check_device()
        got, want = f32(to_np_bf16(hl)), f32(to_np_bf16(ref[r0:r0 + rows]))
        got2, want2 = f32(to_np_bf16(hl2)), f32(to_np_bf16(ref2[r0:r0 + rows]))
        out_q.put((rank, max_rel_err(got, want), cosine(got, want), max_rel_err(got2, want2), cosine(got2, want2)))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("sparse_name", ["dense", "sol", "topk"])
def test_ulysses_block_matches_single_gpu(sparse_name):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, sparse_name, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in procs] == [0, 0]
    res = []
    while not q.empty():
        res.append(q.get())
    assert len(res) == 2
    for rank, e1, c1, e2, c2 in res:
        # same kernels on the same rows: only the attention split differs
        assert e1 <= 2e-2 and c1 >= 0.999, (rank, e1, c1)
        assert e2 <= 2e-2 and c2 >= 0.999, (rank, e2, c2)
