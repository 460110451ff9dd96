"""Sharding of independent images / scenes over ranks and the optional depth gather
(CPU only: gloo process groups of world size 2 and 3 on 127.0.0.1)."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")

from da3cpplib_b200 import shard  # noqa: E402


def test_shard_range_partitions():
    for n in (0, 1, 7, 64, 65, 1000):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, _) in zip(spans, spans[1:]):
                assert b == c
            counts = [b - a for a, b in spans]
            assert max(counts) - min(counts) <= 1
            assert counts == shard.shard_counts(n, world)


def test_shard_range_bench_shapes():
    # C3: 64 images over 1/2/4/8 GPUs -> 64/N each; C4: 16 scenes of 8 views
    for world in (1, 2, 4, 8):
        assert shard.shard_counts(64, world) == [64 // world] * world
        assert shard.scene_views(16, 8, world, world - 1) == (8 * (16 - 16 // world), 128)


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard.shard_range(10, 2, 2)
    with pytest.raises(ValueError):
        shard.shard_range(10, 0, 0)
    with pytest.raises(ValueError):
        shard.shard_range(-1, 2, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gather_worker(rank, world, port, n_units, fail_rank, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        f, e = shard.shard_range(n_units, world, rank)
        # each unit's "depth map" is filled with its global index
        local = torch.arange(f, e, dtype=torch.float32)[:, None, None].expand(e - f, 3, 5).contiguous()
        if rank == fail_rank:
            local = local[:-1]  # a rank that holds the wrong number of units must raise
        out = shard.gather_to_rank0(local, n_units)
        if rank == 0:
            ok = out.shape == (n_units, 3, 5) and all(bool((out[i] == i).all()) for i in range(n_units))
            q.put(("ok" if ok else "bad", rank))
        else:
            q.put(("ok" if out is None else "bad", rank))
        dist.destroy_process_group()
    except ValueError as ex:
        q.put(("raised", rank, str(ex)))
    except Exception as ex:  # noqa: BLE001 - reported to the parent
        q.put(("error", rank, repr(ex)))


def _run(world, n_units, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, n_units, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    for _ in range(world):
        try:
            res.append(q.get(timeout=90))
        except Exception:  # noqa: BLE001
            break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    return res


@pytest.mark.parametrize("world,n_units", [(2, 64), (2, 7), (3, 10)])
def test_gather_to_rank0_gloo(world, n_units):
    res = _run(world, n_units)
    assert sorted(r[0] for r in res) == ["ok"] * world, res


def test_gather_rejects_wrong_local_count():
    """A rank whose slice does not match its shard raises before the collective; the
    other rank's collective then ends with the process group's timeout error instead
    of hanging (both outcomes are reported on the host)."""
    res = _run(2, 8, fail_rank=1)
    kinds = {r[1]: r[0] for r in res}
    assert kinds.get(1) == "raised"
    assert kinds.get(0) in ("error", None)
