"""Chunk sharding + blob stitch across ranks, run as 2 gloo ranks on CPU.

The stitched result must equal the single-process result byte for byte, and
a rank that dies before the exchange must surface as an error on rank 0
(host-side failure, no GPU involved)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _codec(chunks):
    return [bytes(reversed(c)) + bytes([len(c) % 251]) for c in chunks]


def _worker(rank, world, port, items, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), KRUNCH_PG_TIMEOUT_S="20")
    from krunch_b200 import distributed as d
    try:
        d.init_from_env(backend="gloo")
        if mode == "die" and rank == 1:
            os._exit(3)  # leaves between steps, nothing in flight
        out = d.map_chunks(_codec, items)
        q.put((rank, "ok", out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "err", repr(e)))
    finally:
        try:
            d.shutdown()
        except Exception:
            pass


def _run(world, items, mode="ok"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, items, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    expect = world if mode == "ok" else 1
    for _ in range(expect):
        r, status, val = q.get(timeout=120)
        res[r] = (status, val)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("world,n", [(2, 7), (2, 1), (3, 10)])
def test_stitch_matches_single_process(world, n):
    items = [bytes([i]) * (i * 37 % 200 + 1) for i in range(n)]
    res = _run(world, items)
    assert res[0][0] == "ok", res[0]
    assert res[0][1] == _codec(items)
    for r in range(1, world):
        assert res[r] == ("ok", None)


def test_dead_rank_is_an_error_on_rank0():
    items = [b"x" * 10] * 4
    res = _run(2, items, mode="die")
    assert res[0][0] == "err"
