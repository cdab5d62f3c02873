"""Host-side logic of the multi-GPU path, on CPU with gloo, world size 2.

The bench shards sequences across ranks with no token-path collective; the
only cross-rank traffic is timing barriers and max/sum reductions.  Here two
gloo ranks check that the shards tile the global set exactly once and that the
reductions behave as the bench assumes."""
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    sys.path[:0] = [str(ROOT / "verbum.cpp_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import vbdist
    g = vbdist.Group(backend="gloo", timeout_s=60)
    mine = list(vbdist.shard(130, g.rank, g.world))
    allidx = g.gather_ints([len(mine)])
    first = g.gather_ints([mine[0]])
    mx = g.reduce_max(1.5 + rank)
    sm = g.reduce_sum(10.0 * (rank + 1))
    g.barrier()
    seeds = [vbdist.sequence_seed(i) for i in mine]
    g.close()
    q.put((rank, mine, allidx, first, mx, sm, seeds))


def test_shard_partition_single_process():
    import vbdist
    for total in (1, 64, 130, 512):
        for world in (1, 2, 3, 8):
            got = [i for r in range(world) for i in vbdist.shard(total, r, world)]
            assert got == list(range(total))
    with pytest.raises(ValueError):
        vbdist.shard(10, 2, 2)


def test_two_rank_gloo_group():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, m0, c0, f0, mx0, sm0, s0), (r1, m1, c1, f1, mx1, sm1, s1) = out
    assert m0 + m1 == list(range(130))
    assert c0 == c1 == [65, 65]
    assert f0 == [0, 65]
    assert mx0 == mx1 == 2.5 and sm0 == sm1 == 30.0
    assert set(s0).isdisjoint(s1)
