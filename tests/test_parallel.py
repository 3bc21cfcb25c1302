"""Row sharding across ranks (host logic): gloo process groups on CPU with
world sizes 2 and 4. The conversion applied per shard is CPU PyTorch's own
(the kernels need a GPU); what is tested is the partition and the
replicated-output gather."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fp4_fp8_for_torch_mps.parallel import (PeerLeft, announce_leave, check_peers, gather_rows, shard_rows,
                                            sharded_rows_apply, sharded_scaled_mm)


@pytest.mark.parametrize("total,ws", [(0, 2), (1, 4), (7, 2), (16, 4), (1000, 8), (16384, 8)])
def test_shard_rows_partition(total, ws):
    blocks = [shard_rows(total, ws, r) for r in range(ws)]
    assert blocks[0][0] == 0 and blocks[-1][1] == total
    for (s0, e0), (s1, e1) in zip(blocks, blocks[1:]):
        assert e0 == s1
    sizes = [e - s for s, e in blocks]
    assert max(sizes) - min(sizes) <= 1


def test_single_process_is_identity():
    x = torch.randn(5, 3)
    assert torch.equal(sharded_rows_apply(x, lambda t: t * 2), x * 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, rows, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        _body(rank, ws, rows, q)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _body(rank, ws, rows, q):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(rows, 24, generator=g) * 50
    enc = sharded_rows_apply(x, lambda t: t.to(torch.float8_e4m3fn), gather=True)
    ok1 = torch.equal(enc.view(torch.uint8), x.to(torch.float8_e4m3fn).view(torch.uint8))
    local = sharded_rows_apply(x, lambda t: t.to(torch.float8_e5m2))
    s, e = shard_rows(rows, ws, rank)
    ok2 = torch.equal(local.view(torch.uint8), x[s:e].to(torch.float8_e5m2).view(torch.uint8))
    a = (torch.randn(rows, 32, generator=g) * 10).to(torch.float8_e4m3fn)
    b = (torch.randn(16, 32, generator=g) * 10).to(torch.float8_e4m3fn)
    sc = torch.tensor(0.5)
    full = sharded_scaled_mm(a, b.t(), sc, sc, gather=True, out_dtype=torch.float32)
    ok3 = torch.equal(full, torch._scaled_mm(a, b.t(), sc, sc, out_dtype=torch.float32))
    back = gather_rows(local, rows)
    ok4 = torch.equal(back.view(torch.uint8), x.to(torch.float8_e5m2).view(torch.uint8))
    q.put((rank, ok1, ok2, ok3, ok4))


@pytest.mark.parametrize("ws,rows", [(2, 37), (4, 64), (4, 3)])
def test_gloo_sharded_convert_and_gather(ws, rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, rows, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(len(r) == 5 and all(r[1:]) for r in res), res


def _failing_worker(rank, ws, port, q):
    """Rank 1 fails on the host before the gather (an exception in its
    conversion); the others must get an error from the collective, not wait
    for ever."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=10))
    x = torch.randn(8 * ws, 16)

    def convert(t):
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        return t.to(torch.float8_e4m3fn)
    try:
        sharded_rows_apply(x, convert, gather=True)
        q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001 - the test wants whatever the collective raised
        q.put((rank, "error", str(e)[:200]))
    q.close()
    q.join_thread()  # the message is in the pipe before the process ends
    os._exit(0)  # no destroy_process_group: the group is broken


@pytest.mark.parametrize("ws", [2, 3])
def test_gloo_rank_failure_surfaces_as_error(ws):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(ws))
    for p in procs:
        p.join(timeout=60)
    assert res[1][:2] == (1, "error") and "injected" in res[1][2], res
    for r in res:
        assert r[1] == "error", res  # no rank completes a gather that lost a member


def _leaving_worker(rank, ws, port, q):
    """Two steps of a sharded conversion + gather on every rank; then rank 1
    leaves between steps (announcing it in the store). The other ranks must
    detect that on the host before their third step and stop with PeerLeft,
    without entering a collective."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    store = dist.TCPStore("127.0.0.1", port + 1, ws, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", rank=rank, world_size=ws, store=dist.PrefixStore("pg", store),
                            timeout=datetime.timedelta(seconds=10))
    x = torch.randn(8 * ws, 16)
    steps = 0
    try:
        for step in range(4):
            check_peers(store, ws, rank)
            sharded_rows_apply(x, lambda t: t.to(torch.float8_e4m3fn), gather=True)
            steps += 1
            leaving = rank == 1 and step == 1
            if leaving:
                announce_leave(store, rank)  # before the barrier that closes its last step
            dist.barrier()  # the step is complete on every rank before the next check
            if leaving:
                q.put((rank, "left", steps))
                break
        else:
            q.put((rank, "completed", steps))
    except PeerLeft as e:
        q.put((rank, "peer_left", steps, str(e)))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("ws", [2, 3])
def test_gloo_rank_leaving_between_steps_is_detected(ws):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(ws))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == (1, "left", 2), res
    for r in res:
        if r[0] != 1:
            assert r[1] == "peer_left" and r[2] == 2 and "[1]" in r[3], res


def test_check_peers_single_store():
    store = dist.HashStore()
    check_peers(store, 3, 0)
    announce_leave(store, 2)
    with pytest.raises(PeerLeft):
        check_peers(store, 3, 0)
    check_peers(store, 3, 2)  # a rank does not report itself
