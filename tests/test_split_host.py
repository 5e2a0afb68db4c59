"""Sequence split, host side without a GPU: the handle exchange over
torch.distributed (gloo, two ranks) hands every rank all handles in rank
order, and a malformed handle is refused before any connect."""
import os
import socket

import pytest
import torch.multiprocessing as mp


class FakeModel:
    def __init__(self, rank, bad=False):
        self.rank, self.bad, self.connected = rank, bad, None

    def split_prepare(self, rank, world):
        assert rank == self.rank and world == 2
        n = 63 if self.bad else 64
        return bytes([rank + 1]) * n

    def split_connect(self, handles):
        self.connected = handles


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, bad_rank, q):
    import datetime
    import torch.distributed as dist
    import q35
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    m = FakeModel(rank, bad=(rank == bad_rank))
    try:
        q35.split_connect_dist(m)
        q.put((rank, "ok", m.connected))
    except q35.Q35Error as e:
        q.put((rank, "err", str(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bad_rank", [-1, 1])
def test_split_handle_exchange(bad_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, port, bad_rank, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    if bad_rank < 0:
        for rank, status, handles in res:
            assert status == "ok"
            assert handles == [b"\x01" * 64, b"\x02" * 64]
    else:
        # both ranks see the malformed handle and refuse to connect
        assert all(status == "err" and "malformed" in msg for _, status, msg in res)
