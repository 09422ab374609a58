"""Multi-rank host logic on CPU (gloo, world size 2): the (b, h) / sequence
partition covers every unit exactly once, device timings reduce to the max
over ranks, and a rank that fails between steps is detected by the others
through a bounded process-group wait instead of a hang."""
import os
import socket
import traceback

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from lightserve_b200.sharding import max_over_ranks, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_partitions_units():
    for n in (0, 1, 7, 128, 131):
        for w in (1, 2, 3, 8):
            got = [shard_range(n, r, w) for r in range(w)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        if mode == "ok":
            units = list(range(*shard_range(128, rank, world)))
            gathered = [None] * world
            dist.all_gather_object(gathered, units)
            q.put((rank, sorted(sum(gathered, [])) == list(range(128)), max_over_ranks(float(rank + 1))))
        else:  # rank 1 fails before the step barrier; rank 0 must see an error, not hang
            if rank == 1:
                raise SystemExit(3)
            try:
                dist.barrier()
                q.put((rank, "no error", None))
            except Exception as e:  # noqa: BLE001 -- the detection being tested
                q.put((rank, "detected", type(e).__name__))
        dist.destroy_process_group()
    except SystemExit:
        raise
    except Exception:
        q.put((rank, "crash", traceback.format_exc()))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    for p in ps:
        if p.is_alive():
            p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda t: t[0]), [p.exitcode for p in ps]


def test_gloo_world2_partition_and_max():
    out, codes = _run("ok")
    assert codes == [0, 0], out
    assert [o[1] for o in out] == [True, True]
    assert [o[2] for o in out] == [2.0, 2.0]


def test_gloo_failed_rank_is_detected():
    out, codes = _run("fail")
    assert codes[1] == 3
    assert out and out[0][0] == 0 and out[0][1] == "detected", out
