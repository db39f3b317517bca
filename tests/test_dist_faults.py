"""Rank failures on the host, as gloo ranks on CPU: a rank that never joins a
collective, one that dies, one that raises between steps and one that stalls.

The surviving rank must learn of it within a bounded time, with status
SPECDEC_ETIMEOUT (specdec.dist.RankLost), instead of waiting for ever:
guarded collectives (TorchComm(timeout=...), step_throughput(timeout=...))
end a collective whose peer is missing, and the step heartbeat (PeerMonitor)
stops a rank before its next launch when a peer has left or fallen behind.
No GPU is involved: failures are made on the host (an exception, an exit, a
skipped call, a sleep)."""
import os
import socket
import time

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import datetime

    import torch.distributed as dist

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    return dist, store


def _wait_key(store, key, limit=60.0):
    t0 = time.monotonic()
    while time.monotonic() - t0 < limit:
        try:
            if store.check([key]):
                return
        except Exception:  # the store's host is gone
            return
        time.sleep(0.01)


def _worker(scenario, rank, world, port, q):
    import torch

    from specdec.dist import PeerMonitor, RankLost, TorchComm, step_throughput

    dist, store = _init(rank, world, port)
    out = {"rank": rank, "steps": [], "error": None}

    def lost(e, t0):
        out["error"] = {"type": type(e).__name__, "code": getattr(e, "code", None), "peer": getattr(e, "rank", None),
                        "after": time.monotonic() - t0, "msg": str(e)[:200]}

    try:
        if scenario == "never_joins":
            if rank == 0:
                comm = TorchComm(dist, timeout=1.5)
                t0 = time.monotonic()
                try:
                    comm.all_reduce_sum(torch.ones(4))
                except RankLost as e:
                    lost(e, t0)
                store.set("done/0", "1")
            else:
                _wait_key(store, "done/0")  # skips the collective
        elif scenario == "crash":
            dist.barrier()
            if rank == 1:
                os._exit(3)  # dies without a word between steps
            time.sleep(0.5)
            t0 = time.monotonic()
            try:
                step_throughput(dist, 10.0, 5, "cpu", timeout=20.0)
            except RankLost as e:
                lost(e, t0)
        elif scenario in ("raises", "stalls", "healthy"):
            mon = PeerMonitor(store, rank, world, timeout=20.0 if scenario == "raises" else 1.5)
            comm = TorchComm(dist, timeout=20.0)
            t0 = time.monotonic()
            try:
                with mon.member():
                    for step in range(5):
                        if scenario == "stalls" and rank == 1 and step == 2:
                            _wait_key(store, "done/0")  # stops publishing its steps
                            break
                        t0 = time.monotonic()
                        mon.begin_step(step)
                        s = comm.all_reduce_sum(torch.tensor([float(rank + 1)]))
                        out["steps"].append(float(s.item()))
                        if scenario == "raises" and rank == 1 and step == 2:
                            raise ValueError("injected failure between steps")
                    if scenario == "healthy":
                        out["throughput"] = step_throughput(dist, 100.0 + rank, 10, "cpu", timeout=20.0)
            except RankLost as e:
                lost(e, t0)
            except ValueError as e:
                out["raised"] = str(e)
            if rank == 0:
                store.set("done/0", "1")
    finally:
        q.put(out)
        q.close()
        q.join_thread()
        # rank 0 hosts the store: it leaves after every live peer said goodbye
        if rank == 0:
            for r in range(1, world):
                if not (scenario == "crash" and r == 1):
                    _wait_key(store, f"bye/{r}", 30.0)
        else:
            try:
                store.set(f"bye/{rank}", "1")
            except Exception:
                pass
    os._exit(0)  # no destroy_process_group: a peer may be gone or a collective abandoned


def _run(scenario, world):
    import torch.multiprocessing as mp

    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(scenario, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        deadline = time.monotonic() + 180
        expect = world - (1 if scenario == "crash" else 0)
        while len(res) < expect and time.monotonic() < deadline:
            try:
                o = q.get(timeout=5)
            except Exception:
                continue
            res[o["rank"]] = o
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    return res, [p.exitcode for p in procs]


def test_collective_a_rank_never_joins_times_out():
    from specdec import ETIMEOUT

    res, codes = _run("never_joins", 2)
    assert codes == [0, 0]
    err = res[0]["error"]
    assert err is not None and err["type"] == "RankLost" and err["code"] == ETIMEOUT
    assert 1.0 < err["after"] < 30.0


def test_collective_after_a_rank_died_fails_fast():
    from specdec import ETIMEOUT

    res, codes = _run("crash", 2)
    assert codes[1] == 3 and codes[0] == 0
    err = res[0]["error"]
    assert err is not None and err["type"] == "RankLost" and err["code"] == ETIMEOUT
    assert err["after"] < 30.0  # the closed connection (or at worst the 20 s limit), not the group's 60 s


def test_rank_raising_between_steps_stops_the_others_before_their_next_launch():
    res, codes = _run("raises", 2)
    assert codes == [0, 0]
    assert res[1]["raised"] == "injected failure between steps"
    assert res[1]["steps"] == [3.0, 3.0, 3.0] == res[0]["steps"]
    err = res[0]["error"]
    assert err["type"] == "RankLost" and err["peer"] == 1 and "left before step 3" in err["msg"]
    assert err["after"] < 10.0  # reported from the mark at once, not after the 20 s heartbeat limit


def test_stalled_rank_is_reported_when_the_heartbeat_runs_out():
    res, codes = _run("stalls", 2)
    assert codes == [0, 0]
    assert res[0]["steps"] == [3.0, 3.0]
    err = res[0]["error"]
    assert err["type"] == "RankLost" and err["peer"] == 1 and "did not reach step 2" in err["msg"]
    assert 1.0 < err["after"] < 30.0


def test_healthy_ranks_pass_the_guards():
    res, codes = _run("healthy", 3)
    assert codes == [0, 0, 0]
    for r in range(3):
        assert res[r]["error"] is None and "raised" not in res[r]
        assert res[r]["steps"] == [6.0] * 5
        assert res[r]["throughput"] == {"ms_max": 102.0, "tokens": 30.0, "value": pytest.approx(30.0 / 0.102)}


def test_monitor_rejects_bad_rank():
    from specdec.dist import PeerMonitor

    with pytest.raises(ValueError):
        PeerMonitor(None, 2, 2)


def test_graph_acceptor_refuses_a_host_timeout():
    """A collective recorded in a CUDA graph cannot take a host wait."""
    from specdec.dist import ShardedChainAcceptor

    class _Comm:
        world, rank, timeout = 2, 0, 5.0

    class _Sp:
        temperature, top_p, seed, step = 0.8, 0.9, 0, 0

    with pytest.raises(ValueError, match="host timeout"):
        ShardedChainAcceptor(None, None, None, 3, 0, _Sp(), _Comm(), graph=True)
