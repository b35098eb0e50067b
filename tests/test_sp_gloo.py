"""Ulysses sequence parallelism on CPU ranks (gloo, world size 2).

* The partition of wx_sp_make_plan and the data layout of the two all-to-alls
  (include/wx_api.h, wx_sp_plan) are exercised with torch tensors: after the
  first exchange each rank must hold the packed q|k|v of its heads for the
  whole sequence, after the second its own rows of every head — exactly what
  the CUDA pack/unpack kernels of wx_sp.cu produce on the GPU.
* Failure detection happens on the host: a rank that dies before the exchange
  makes the other rank's collective end with an error after a short timeout.
"""
import datetime
import os
import socket

import pytest

pytestmark = pytest.mark.timeout(180) if hasattr(pytest.mark, "timeout") else []


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layout_worker(rank, world, port, S, H, hd, out_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from wuxianhuabu_b200 import h3
        plan = h3.sp_plan(S, H, hd, world, rank)
        P, rows, Hl = plan.P, plan.rows, plan.heads
        full = torch.arange(S * 3 * H * hd, dtype=torch.float64).reshape(S, 3 * H * hd)
        local = full[plan.row0:plan.row0 + rows]
        # pack: send[r][row][part][c] = local[row, part*H*hd + r*Hl*hd + c]
        send = local.reshape(rows, 3, P, Hl * hd).permute(2, 0, 1, 3).contiguous()
        assert send.numel() == P * plan.qkv_chunk
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv.view(-1), send.view(-1))
        got = recv.reshape(S, 3 * Hl * hd)
        want = full.reshape(S, 3, H, hd)[:, :, plan.head0:plan.head0 + Hl, :].reshape(S, 3 * Hl * hd)
        ok_fwd = torch.equal(got, want)
        # attention output of this rank's heads (any function of the full sequence)
        attf = got.reshape(S, 3, Hl * hd)[:, 0, :] * 2 + 1
        ret = torch.empty((P, rows, Hl * hd), dtype=attf.dtype)
        dist.all_to_all_single(ret.view(-1), attf.contiguous().view(-1))
        assert ret.numel() == P * plan.out_chunk
        # unpack: att[row][r*Hl*hd + c] = ret[r][row][c]
        att = ret.permute(1, 0, 2).reshape(rows, P * Hl * hd)
        q_full = full.reshape(S, 3, H * hd)[:, 0, :]
        ok_ret = torch.equal(att, (q_full * 2 + 1)[plan.row0:plan.row0 + rows])
        out_q.put((rank, ok_fwd, ok_ret, plan.row0, plan.head0))
    finally:
        dist.destroy_process_group()


def _failing_worker(rank, world, port, out_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # this rank dies between steps, before the exchange
    x = torch.zeros(8)
    y = torch.empty(8)
    try:
        dist.all_to_all_single(y, x)
        out_q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001 - any collective error is the detection
        out_q.put((rank, "error:" + type(e).__name__))


def _run(fn, world, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = []
    while not q.empty():
        res.append(q.get())
    return res, [p.exitcode for p in procs]


@pytest.mark.parametrize("S,H", [(96, 4), (126512 // 64 * 2, 24)])
def test_ulysses_layout_two_ranks(S, H):
    res, codes = _run(_layout_worker, 2, _free_port(), S, H, 128)
    assert codes == [0, 0], codes
    res = sorted(res)
    assert [r[0] for r in res] == [0, 1]
    for rank, ok_fwd, ok_ret, row0, head0 in res:
        assert ok_fwd and ok_ret, (rank, ok_fwd, ok_ret)
        assert row0 == rank * (S // 2) and head0 == rank * (H // 2)


def test_plan_rejects_uneven_partitions():
    from wuxianhuabu_b200 import _lib, h3
    with pytest.raises(_lib.WxError):
        h3.sp_plan(100, 24, 128, 8, 0)   # rows do not split evenly
    with pytest.raises(_lib.WxError):
        h3.sp_plan(128, 20, 128, 8, 0)   # heads do not split evenly
    p = h3.sp_plan(126512, 24, 128, 8, 7)
    assert (p.rows, p.row0, p.heads, p.head0) == (15814, 7 * 15814, 3, 21)
    assert p.qkv_chunk == 15814 * 3 * 3 * 128 and p.out_chunk == 15814 * 3 * 128


def test_dead_rank_is_detected_by_the_survivor():
    res, codes = _run(_failing_worker, 2, _free_port())
    assert codes[1] == 3
    assert res and res[0][0] == 0 and res[0][1].startswith("error:"), res
