"""Ulysses sequence parallelism on 2, 4 and 8 GPUs: wx_dit_block_forward_sp against the
single-GPU block on the same inputs (dense, SOL and top-k attention, and a dense block with
LoRA adapters on its four linears; refresh, refresh, PAB reuse in sequence), with the exchange
over NVLink peer memory (default: the q|k|v projection's epilogue stores into the owners'
buffers) and over NCCL all-to-alls (WX_SP_P2P=0). S = 1000 rows, so that rank boundaries fall
inside 128-row query tiles; heads = max(4, P). Each world size is skipped on boxes with fewer
GPUs."""
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


def _maybe_lora(blk, sparse_name, hidden, heads, ffn):
    """("lora" case) one adapter on each of the four linears, the same on every rank"""
    if sparse_name != "lora":
        return blk
    from tests.test_gpu_lora import _adapters, _refs
    from wuxianhuabu_b200 import h3
    inner = heads * 128
    dims = [(hidden, 3 * inner), (inner, hidden), (hidden, ffn), (ffn, hidden)]
    for i, (lin, (k, n)) in enumerate(zip(blk.blocks[0].linears(), dims)):
        lin.set_lora(_refs(_adapters(60 + i, k, n, [16], [0.9])))
    return h3.H3DiTBlocks(blk.cfg, blk.blocks)


def _worker(rank, world, port, sparse_name, p2p, out_q, fused="1"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["WX_SP_P2P"] = p2p
    os.environ["WX_QKV_ROPE_FUSED"] = fused
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
        hidden, heads, ffn, rot, eps, g = 256, max(4, world), 512, 96, 1e-6, 40
        S = 1000  # 1000 / P rows per rank: rank boundaries fall inside 128-row query tiles
        w, mods, h, cos, sin, rowmap = make_block(9, hidden, heads, ffn, 0, S, rot)
        sparse = {"dense": None, "lora": None, "sol": dict(tau=0.4),
                  "topk": dict(block=128, topk_ratio=0.25, tail=False)}[sparse_name]
        spec = None if sparse is None else h3.H3SolAttnConfig(**sparse).spec(g)
        blk = _maybe_lora(gpu_block(w, hidden, heads, ffn, 0, rot, eps), sparse_name, hidden, heads, ffn)
        md = [to_torch_bf16(m, dev) for m in mods]
        rm = torch.from_numpy(rowmap.view(np.int32)).to(dev)
        c, s = to_torch_bf16(cos, dev), to_torch_bf16(sin, dev)
        schedule = [True, True, False]  # refresh, refresh, PAB reuse
        # single-GPU reference on this device (before the communicator exists)
        ref = to_torch_bf16(h, dev)
        slot_ref = torch.empty((S, hidden), dtype=torch.bfloat16, device=dev)
        refs = []
        for refresh in schedule:
            blk.block_forward(0, ref, md, rm, c, s, spec, pab_slot=slot_ref, refresh=refresh)
            refs.append(ref.clone())
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
        blk2 = _maybe_lora(gpu_block(w, hidden, heads, ffn, 0, rot, eps), sparse_name, hidden, heads, ffn)
        res = []
        for refresh, want in zip(schedule, refs):
            blk2.block_forward(0, hl, md, rm[r0:r0 + rows].contiguous(), c[r0:r0 + rows].contiguous(),
                               s[r0:r0 + rows].contiguous(), spec, pab_slot=slot, refresh=refresh, S_total=S)
            torch.cuda.synchronize()
            got, wnt = f32(to_np_bf16(hl)), f32(to_np_bf16(want[r0:r0 + rows]))
            res += [max_rel_err(got, wnt), cosine(got, wnt)]
        h3.context(rank).check_device()
        path = h3.context(rank).sp_exchange()
        out_q.put((rank, path, *res))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("p2p", ["1", "0"])
@pytest.mark.parametrize("sparse_name", ["dense", "sol", "topk", "lora"])
def test_ulysses_block_matches_single_gpu(sparse_name, p2p, world):
    _run_group(sparse_name, p2p, world, "1")


@pytest.mark.parametrize("sparse_name", ["dense", "sol"])
def test_ulysses_peer_exchange_with_the_separate_norm_rope_kernel(sparse_name):
    """WX_QKV_ROPE_FUSED=0: the q|k|v stores into the owners' buffers come from
    qk_norm_rope_vec_kernel<RopePeerDst> after the projection instead of its epilogue."""
    _run_group(sparse_name, "1", 2, "0")


def _run_group(sparse_name, p2p, world, fused):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, sparse_name, p2p, q, fused)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in procs] == [0] * world
    res = []
    while not q.empty():
        res.append(q.get())
    assert len(res) == world
    for rank, path, *errs in res:
        # the exchange path asked for was taken (1 peer memory, 0 all-to-alls)
        assert path == int(p2p), (rank, path)
        # same kernels on the same rows: only the attention split differs
        for i in range(0, len(errs), 2):
            assert errs[i] <= 2e-2 and errs[i + 1] >= 0.999, (rank, i // 2, errs[i], errs[i + 1])
