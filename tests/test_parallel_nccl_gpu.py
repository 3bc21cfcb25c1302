"""Multi-GPU failure detection over NCCL: ranks on two GPUs (one process per
GPU) run row-sharded FP4 decode steps through this package's kernel and
gather the rows with parallel.gather_rows (NCCL all_gather_into_tensor). After
its second step rank 1 leaves the job: it announces that in the store before
the barrier that closes the step, with none of its kernels or collectives in
flight. Rank 0 must find the record on the host before its third step and
stop with PeerLeft, without launching a kernel or entering a collective.

NVLS is off (NCCL_NVLS_ENABLE=0) and nothing here uses multicast memory, so a
rank that exits holds no NVLink multicast binding. Skipped with fewer than two
GPUs.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, q):
    import datetime

    import numpy as np
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from fp4_fp8_for_torch_mps import fp8_mps_native as nat
    from fp4_fp8_for_torch_mps.parallel import PeerLeft, announce_leave, check_peers, gather_rows, shard_rows
    from oracle import oracle as O

    store = dist.TCPStore("127.0.0.1", port, ws, rank == 0, timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("nccl", rank=rank, world_size=ws, store=dist.PrefixStore("pg", store),
                            timeout=datetime.timedelta(seconds=20), device_id=torch.device("cuda", rank))
    rows = 256
    x = torch.randint(0, 256, (rows, 512), dtype=torch.uint8, generator=torch.Generator().manual_seed(0))
    s, e = shard_rows(rows, ws, rank)
    xl = x[s:e].cuda()
    steps, ok = 0, True
    try:
        for step in range(4):
            check_peers(store, ws, rank)
            local = nat.fp4_decode(xl.view(torch.float4_e2m1fn_x2), torch.bfloat16, scale=torch.tensor([0.37]))
            full = gather_rows(local, rows)
            torch.cuda.synchronize()
            ref = O.fp4_decode(x.numpy(), 1, 0.37)
            ok = ok and bool(np.array_equal(full.cpu().view(torch.int16).numpy().view(np.uint16), ref))
            steps += 1
            leaving = rank == 1 and step == 1
            if leaving:
                announce_leave(store, rank)
            dist.barrier()
            torch.cuda.synchronize()
            if leaving:
                q.put((rank, "left", steps, ok))
                break
        else:
            q.put((rank, "completed", steps, ok))
    except PeerLeft as err:
        q.put((rank, "peer_left", steps, ok, str(err)))
    except Exception as err:  # noqa: BLE001 - reported to the parent instead of a hang
        q.put((rank, "error", steps, ok, repr(err)[:300]))
    q.close()
    q.join_thread()
    os._exit(0)  # the group lost a member: no collective teardown


def test_nccl_rank_leaving_between_steps_is_detected():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert res[1][:4] == (1, "left", 2, True), res
    assert res[0][:4] == (0, "peer_left", 2, True) and "[1]" in res[0][4], res
