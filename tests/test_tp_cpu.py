"""Host-side logic of the tensor-parallel engine, on CPU.

Shard plans (row ranges, stream byte ranges, arena layout) and the
multi-process plumbing the engine uses (handle exchange with
all_gather_object, a rank failing before it joins) run as 2 gloo ranks.
"""

import multiprocessing as mp
import os
import socket

import pytest

from turbopress_b200.tp import arena_layout, shard_rows, shard_stream_bytes


@pytest.mark.parametrize("n", [16, 17, 100, 1024, 2560, 9728, 151936])
@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_shard_rows_cover_exactly(n, world):
    tiles = -(-n // 16)
    if tiles < world:
        pytest.skip("fewer tiles than ranks")
    covered = []
    for r in range(world):
        r0, r1 = shard_rows(n, r, world)
        assert r0 % 16 == 0 and r0 < r1 <= n
        covered.extend(range(r0, r1))
    assert covered == list(range(n))


def test_shard_stream_bytes_tile_aligned():
    n, d, bits = 1000, 700, 3
    units_k = -(-d // 256)
    tile_bytes = units_k * 512 * bits
    total = -(-n // 16) * tile_bytes
    ends = []
    for r in range(4):
        r0, r1 = shard_rows(n, r, 4)
        b0, b1 = shard_stream_bytes(n, d, bits, r0, r1)
        assert b0 % tile_bytes == 0 and b1 % tile_bytes == 0
        ends.append((b0, b1))
    assert ends[0][0] == 0 and ends[-1][1] == total
    assert all(ends[i][1] == ends[i + 1][0] for i in range(3))


def test_arena_layout_aligned_disjoint():
    offs, total = arena_layout([4096, 1024, 1024, 2560], batch=3)
    assert all(o % 256 == 0 for o in offs)
    sizes = [3 * n * 4 for n in (4096, 1024, 1024, 2560)]
    for o, sz, nxt in zip(offs, sizes, offs[1:] + [total]):
        assert o + sz <= nxt
    assert total % 16 == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    handles = [bytes([rank]) * 64, bytes([rank + 10]) * 64, bytes([rank + 20]) * 64]
    got = [None] * world
    dist.all_gather_object(got, (rank, handles))
    # every rank sees every rank's handles, keyed by rank
    ok = sorted(r for r, _ in got) == list(range(world)) and all(h[0][0] == r for r, h in got)
    q.put((rank, ok, [shard_rows(2560, r, world) for r in range(world)]))
    dist.destroy_process_group()


def test_two_rank_handle_exchange_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_exchange, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res)
    assert res[0][2] == res[1][2]  # both ranks derive the same plan


def _late_joiner(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1:
        q.put((rank, "exited"))
        raise SystemExit(0)  # a rank that never joins
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        q.put((rank, "joined"))
    except Exception as e:  # rendezvous times out on the host: the failure is seen without any GPU
        q.put((rank, f"error:{type(e).__name__}"))


def test_rank_that_never_joins_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_late_joiner, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res[1] == "exited"
    assert res[0].startswith("error:")
