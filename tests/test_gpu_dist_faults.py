"""A rank that leaves between steps, on two GPUs under NCCL.

Each rank runs the tiny step engine on its own GPU and meets the other at a
heartbeat (specdec.dist.PeerMonitor) before every step and at one NCCL
all-reduce after it.  Rank 1 raises after its third step, with no kernel or
collective of its own in flight; rank 0 learns of it from the store before
its next launch (RankLost, status SPECDEC_ETIMEOUT) and stops cleanly.  NVLS
is off; nothing waits on a collective that a peer has left.  Needs two GPUs
(skipped otherwise); the same logic runs as gloo ranks on CPU in
test_dist_faults.py."""
import os
import socket
import time

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _wait_key(store, key, limit):
    t0 = time.monotonic()
    while time.monotonic() - t0 < limit:
        try:
            if store.check([key]):
                return
        except Exception:
            return
        time.sleep(0.01)


def _worker(rank, world, port, q):
    import datetime

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import numpy as np
    import torch
    import torch.distributed as dist

    import specdec as S
    from specdec.dist import PeerMonitor, RankLost

    torch.cuda.set_device(rank)
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("nccl", store=store, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    out = {"rank": rank, "steps": [], "error": None, "raised": False}
    eng = S.Engine(S.MODEL_SHAPES["tiny"], batch=2, draft_len=3, max_ctx=256, temperature=1.0, seed=rank,
                   use_graph=True, device=rank)
    try:
        eng.init_weights(0)
        eng.seed_state(np.array([100, 60], np.int32), 5)
        mon = PeerMonitor(store, rank, world, timeout=20.0)
        t0 = time.monotonic()
        try:
            with mon.member():
                for step in range(5):
                    t0 = time.monotonic()
                    mon.begin_step(step)
                    acc, _ = eng.step_host()
                    t = torch.tensor([float(acc.sum() + 2)], device=f"cuda:{rank}")
                    dist.all_reduce(t)
                    torch.cuda.synchronize()
                    out["steps"].append(step)
                    if rank == 1 and step == 2:
                        raise ValueError("injected failure between steps")
        except RankLost as e:
            out["error"] = {"code": e.code, "peer": e.rank, "after": time.monotonic() - t0, "msg": str(e)[:200]}
        except ValueError:
            out["raised"] = True
        out["status"] = eng.info("status")
    finally:
        eng.close()
        q.put(out)
        q.close()
        q.join_thread()
        if rank == 0:
            _wait_key(store, "bye/1", 30.0)
        else:
            try:
                store.set("bye/1", "1")
            except Exception:
                pass
    os._exit(0)  # no collective is pending; the group is not torn down collectively


def test_rank_leaving_between_steps_on_two_gpus():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from specdec import ETIMEOUT

    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        deadline = time.monotonic() + 240
        while len(res) < 2 and time.monotonic() < deadline:
            try:
                o = q.get(timeout=5)
            except Exception:
                continue
            res[o["rank"]] = o
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    assert [p.exitcode for p in procs] == [0, 0]
    assert res[1]["raised"] and res[1]["steps"] == [0, 1, 2]
    assert res[0]["steps"] == [0, 1, 2]
    err = res[0]["error"]
    assert err["code"] == ETIMEOUT and err["peer"] == 1 and "left before step 3" in err["msg"]
    assert err["after"] < 10.0
    assert res[0]["status"] == 0 and res[1]["status"] == 0  # no device-side wait gave up
