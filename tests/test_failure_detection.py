"""Host-side failure detection with CPU (gloo) ranks: no GPU is faulted, trapped or hung."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from granite_switch_b200.parallel.health import Heartbeat, PeerFailure

    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, timeout_s=1.5)
    t = torch.zeros(1)
    try:
        for step in range(20):
            if rank == 1 and step == 3:
                if mode == "leave":
                    hb.leave()
                    q.put((rank, "left"))
                    return  # exits between steps, nothing in flight
                if mode == "silent":
                    time.sleep(6)  # stops beating (e.g. stuck in host code)
                    q.put((rank, "woke"))
                    return
            hb.check()
            dist.all_reduce(t)
            hb.beat()
        q.put((rank, "finished"))
    except PeerFailure as e:
        q.put((rank, f"detected {e.ranks}"))
    except Exception as e:  # a collective that timed out is also a detection
        q.put((rank, f"collective error {type(e).__name__}"))


@pytest.mark.parametrize("mode", ["leave", "silent"])
def test_peer_failure_detected_before_hanging(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res[0].startswith("detected [1]") or res[0].startswith("collective error"), res
    assert time.time() - t0 < 40


def test_heartbeat_fresh_peers_pass():
    store = dist.HashStore()
    from granite_switch_b200.parallel.health import Heartbeat

    a = Heartbeat(store, 0, 2, timeout_s=5)
    b = Heartbeat(store, 1, 2, timeout_s=5)
    a.check()
    b.beat()
    a.check()
