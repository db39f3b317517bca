"""Request sharding across ranks and the reductions of a timed multi-GPU run.

The speculative step shards by request: every rank (one process per GPU)
holds a full weight replica and a disjoint slice of the sequences, so the
data path needs no collective.  What crosses ranks is bookkeeping only: the
slice each rank owns, and after a timed run the slowest rank's device time
(max) and the tokens all ranks emitted (sum).

These helpers take a `torch.distributed`-style module or process group and a
device for the reduction tensors ("cuda:<local rank>" under NCCL, "cpu" under
gloo), so the same code runs in the benchmark and in CPU tests.
"""
from __future__ import annotations


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of n requests owned by `rank`; slices differ in
    size by at most one and cover 0..n-1 exactly once."""
    if world <= 0 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard: n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _reduce(dist, x: float, device: str, op, timeout: float | None = None) -> float:
    if dist is None:
        return float(x)
    import torch

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    if timeout is None:
        dist.all_reduce(t, op=op)
    else:
        guarded_wait(dist.all_reduce(t, op=op, async_op=True), timeout, "all_reduce")
    return float(t.item())


def reduce_max(dist, x: float, device: str = "cpu", timeout: float | None = None) -> float:
    return _reduce(dist, x, device, None if dist is None else dist.ReduceOp.MAX, timeout)


def reduce_sum(dist, x: float, device: str = "cpu", timeout: float | None = None) -> float:
    return _reduce(dist, x, device, None if dist is None else dist.ReduceOp.SUM, timeout)


def step_throughput(dist, ms: float, tokens: float, device: str = "cpu", timeout: float | None = None) -> dict:
    """Whole-job throughput of a timed run: tokens of all ranks over the
    slowest rank's device time.  Every rank must call it (it is collective);
    with `timeout` a rank that never joins raises RankLost after that many
    seconds."""
    ms_max = reduce_max(dist, ms, device, timeout)
    tok = reduce_sum(dist, tokens, device, timeout)
    return {"ms_max": ms_max, "tokens": tok, "value": tok / (ms_max / 1e3) if ms_max > 0 else 0.0}


# ----------------------------------------------------------------------
# Vocabulary-sharded chain acceptance
# ----------------------------------------------------------------------
class TorchComm:
    """Collectives of a torch.distributed process group (NCCL for CUDA tensors).

    With `timeout` (seconds) every collective is issued asynchronously and
    waited for at most that long on the host, raising RankLost when a peer
    never joins or has gone; without it the collectives are plain (the form
    a CUDA graph can capture)."""

    def __init__(self, dist, group=None, timeout: float | None = None):
        self.dist = dist
        self.group = group
        self.timeout = timeout
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def _run(self, issue, what: str):
        if self.timeout is None:
            issue(False)
        else:
            guarded_wait(issue(True), self.timeout, what)

    def all_gather(self, t):
        import torch

        # flat in, flat out (the form every backend accepts), then [world, *shape]
        out = torch.empty(self.world * t.numel(), dtype=t.dtype, device=t.device)
        src = t.contiguous().view(-1)
        self._run(lambda a: self.dist.all_gather_into_tensor(out, src, group=self.group, async_op=a), "all_gather")
        return out.view((self.world,) + tuple(t.shape))

    def all_reduce_sum(self, t):
        self._run(lambda a: self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group, async_op=a),
                  "all_reduce(sum)")
        return t

    def all_reduce_max(self, t):
        self._run(lambda a: self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group, async_op=a),
                  "all_reduce(max)")
        return t


class ThreadComm:
    """The same collectives among W threads of one process (W virtual ranks
    on one GPU, all on one CUDA stream): each rank deposits its tensor, the
    threads meet at a barrier, and every rank reads all deposits."""

    def __init__(self, world: int):
        import threading

        self.world = world
        self.barrier = threading.Barrier(world)
        self.slots = [None] * world

    def rank_view(self, rank: int):
        comm = self

        class _View:
            world = comm.world

            def __init__(self):
                self.rank = rank

            def _exchange(self, t):
                import torch

                comm.slots[self.rank] = t.clone()
                comm.barrier.wait()
                out = torch.stack(list(comm.slots))
                comm.barrier.wait()
                return out

            def all_gather(self, t):
                return self._exchange(t)

            def all_reduce_sum(self, t):
                t.copy_(self._exchange(t).sum(0))
                return t

            def all_reduce_max(self, t):
                t.copy_(self._exchange(t).max(0).values)
                return t

        return _View()


def vocab_shard(V: int, world: int, rank: int) -> tuple[int, int]:
    """Vocabulary columns [v0, v0 + Vs) of `rank`, in rank order (as shard_range)."""
    lo, hi = shard_range(V, world, rank)
    return lo, hi - lo


SHARD_LIST_CAP = 4096  # listed (key, mass) pairs kept per shard row (~1600 per whole row at N(0, 3), T = 0.7)
SHARD_CAND = 32  # crossing-bin candidates per rank and row (kShardCand)


def accept_chain_vocab_sharded(target, draft, drafts, k: int, v0: int, sampling, comm):
    """Chain acceptance with the vocabulary split across ranks.

    target: this rank's columns [v0, v0 + Vs) of the target logits, fp32
    [B, k+1, Vs] on its GPU; draft: [B, k, Vs] (unused when greedy); drafts:
    the drafted global token ids [B, k] int32.  `comm` provides all_gather /
    all_reduce_sum / all_reduce_max over the ranks (ranks in vocabulary
    order).  Returns (accepted [B] int32, out_tokens [B, k+1] int32) on the
    device, the same on every rank and equal to specdec_accept_chain on the
    whole rows.  The steps and what crosses ranks between them are listed
    with the specdec_shard_* functions in include/specdec.h."""
    import ctypes as C

    import torch

    import specdec as S

    L = S.lib()
    dev = target.device
    B, Vs = int(target.shape[0]), int(target.shape[2])
    rows_p, rows_q = B * (k + 1), B * k
    st = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    W, rank = comm.world, comm.rank
    T, tp = float(sampling.temperature), float(sampling.top_p)
    greedy = not (T > 0.0)
    target = target.contiguous()
    drafts = drafts.to(device=dev, dtype=torch.int32).contiguous()

    # per-row steps run on the target rows and (when sampling) the draft rows
    # together: rows [0, rows_p) target, [rows_p, rows_p + nq) draft
    draft = draft.contiguous() if not greedy else None
    nq = 0 if greedy else rows_q
    rows = rows_p + nq
    z2 = p(draft) if nq else None
    mx = torch.empty(rows, dtype=torch.float32, device=dev)
    am = torch.empty(rows, dtype=torch.int32, device=dev)
    S.check(L.specdec_shard_row_max(p(target), rows_p, z2, nq, Vs, v0, p(mx), p(am), st))
    gm, ga = comm.all_gather(mx), comm.all_gather(am)
    S.check(L.specdec_shard_merge_max(p(gm), p(ga), W, rows, p(mx), p(am), st))
    pmax, parg = mx[:rows_p], am[:rows_p]

    def assemble(acc, tok):
        """(accepted, out_tokens [B, k+1]): accepted drafts, the emitted token, -1."""
        idx = torch.arange(k + 1, device=dev)[None, :]
        a = acc.long()[:, None]
        ext = torch.cat([drafts, torch.full((B, 1), -1, dtype=torch.int32, device=dev)], 1)
        out = torch.where(idx < a, ext, torch.full_like(ext, -1))
        out = torch.where(idx == a, tok.to(torch.int32)[:, None], out)
        return acc, out

    if greedy:
        acc = torch.empty(B, dtype=torch.int32, device=dev)
        S.check(L.specdec_shard_accept_test(p(drafts), B, k, C.byref(sampling), p(parg), None, None, None, None,
                                            p(acc), None, st))
        tok = parg.view(B, k + 1).gather(1, acc.long()[:, None])[:, 0]
    else:
        qmax = mx[rows_p:]

        def finish(tau, nuc):
            """Steps 4-7 at the given nucleus thresholds and masses."""
            ptau, qtau = tau[:rows_p], tau[rows_p:]
            pnuc, qnuc = nuc[:rows_p].contiguous(), nuc[rows_p:].contiguous()
            ep = torch.empty(rows_q, dtype=torch.int64, device=dev)
            eq = torch.empty(rows_q, dtype=torch.int64, device=dev)
            S.check(L.specdec_shard_point_mass(p(target), p(draft), p(drafts), B, k, Vs, v0, T, p(pmax), p(ptau),
                                               p(qmax), p(qtau), p(ep), p(eq), st))
            pq = torch.stack([ep, eq])
            comm.all_reduce_sum(pq)
            ep, eq = pq[0].contiguous(), pq[1].contiguous()
            acc = torch.empty(B, dtype=torch.int32, device=dev)
            S.check(L.specdec_shard_accept_test(p(drafts), B, k, C.byref(sampling), p(parg), p(pnuc), p(qnuc),
                                                p(ep), p(eq), p(acc), None, st))
            win = torch.empty((B, 4), dtype=torch.int32, device=dev)
            S.check(L.specdec_shard_draw_winners(p(target), p(draft), B, k, Vs, v0, C.byref(sampling), p(acc),
                                                 p(pmax), p(ptau), p(qmax), p(qtau), p(pnuc), p(qnuc), p(win), None,
                                                 st))
            gwin = comm.all_gather(win).contiguous()
            tok = torch.empty(B, dtype=torch.int32, device=dev)
            S.check(L.specdec_shard_draw_merge(p(gwin), W, B, k, p(acc), p(tok), st))
            return acc, tok

        done = False
        if tp < 1.0 and W * SHARD_CAND <= 256:
            # the listed path: one shard pass, the stats all-reduce and a small
            # candidate all-gather (steps 2'-3' in include/specdec.h).  The rows'
            # ok flags are read only after the whole acceptance is queued, so
            # the host does not stall the GPU; a row that needs the digit
            # passes (rare: flat rows, NaN logits) redoes the acceptance below.
            lst = torch.empty((rows, SHARD_LIST_CAP, 2), dtype=torch.int32, device=dev)
            lnum = torch.empty(rows, dtype=torch.int32, device=dev)
            stats = torch.empty((rows, 260), dtype=torch.int64, device=dev)
            S.check(L.specdec_shard_mass_hist(p(target), rows_p, z2, nq, Vs, p(mx), T, SHARD_LIST_CAP, p(lst),
                                              p(lnum), p(stats), st))
            comm.all_reduce_sum(stats)
            G = torch.empty(rows, dtype=torch.int64, device=dev)
            cand = torch.empty((rows, SHARD_CAND + 1, 2), dtype=torch.int32, device=dev)
            S.check(L.specdec_shard_cross(p(stats), rows, tp, p(mx), T, p(lst), SHARD_LIST_CAP, p(lnum), p(G),
                                          p(cand), st))
            gcand = comm.all_gather(cand).contiguous()
            tau = torch.empty(rows, dtype=torch.int32, device=dev)
            nuc = torch.empty(rows, dtype=torch.int64, device=dev)
            ok = torch.empty(rows, dtype=torch.int32, device=dev)
            S.check(L.specdec_shard_union_select(p(gcand), W, rows, p(stats), p(G), tp, p(tau), p(nuc), p(ok), st))
            acc, tok = finish(tau, nuc)
            res = assemble(acc, tok)
            done = bool(ok.all().item())  # the same on every rank: computed from exchanged data only
        if not done:
            sums = torch.empty(rows, dtype=torch.int64, device=dev)
            S.check(L.specdec_shard_row_mass(p(target), rows_p, z2, nq, Vs, p(mx), T, p(sums), st))
            comm.all_reduce_sum(sums)
            if tp < 1.0:
                tau = torch.zeros(rows, dtype=torch.int32, device=dev)
                G = torch.zeros(rows, dtype=torch.int64, device=dev)
                last = torch.zeros(rows, dtype=torch.int64, device=dev)
                hist = torch.empty((rows, 256), dtype=torch.int64, device=dev)
                for d in (3, 2, 1, 0):
                    S.check(L.specdec_shard_digit_hist(p(target), rows_p, z2, nq, Vs, p(mx), T, p(tau), d, p(hist),
                                                       st))
                    comm.all_reduce_sum(hist)
                    S.check(L.specdec_shard_select_digit(p(hist), rows, d, p(sums), tp, p(tau), p(G), p(last), st))
                nuc = G + last
            else:
                tau = torch.zeros(rows, dtype=torch.int32, device=dev)
                nuc = sums
            res = assemble(*finish(tau, nuc))
        return res
    return assemble(acc, tok)


class ShardedChainAcceptor:
    """accept_chain_vocab_sharded for fixed shapes and sampling (T > 0, top_p
    < 1, at most 8 ranks) with its buffers allocated once and, when `graph`
    is set, the listed path -- its kernels and collectives -- recorded in one
    CUDA graph, so that a call costs the host one graph launch instead of
    about twenty kernel and collective launches.

    target [B, k+1, Vs], draft [B, k, Vs] and drafts [B, k] are the static
    inputs: write each step's shard logits and drafted tokens into them.  The
    step of the uniforms is a device counter (`__call__(step)` sets it).
    Rows the listed path cannot settle (flat rows, NaN logits) make the call
    redo the acceptance with accept_chain_vocab_sharded.  `close()` releases
    the graph and must run before the process group is destroyed."""

    def __init__(self, target, draft, drafts, k: int, v0: int, sampling, comm, graph: bool = True):
        import torch

        T, tp = float(sampling.temperature), float(sampling.top_p)
        if not (T > 0.0 and tp < 1.0 and comm.world * SHARD_CAND <= 256):
            raise ValueError("ShardedChainAcceptor: needs T > 0, top_p < 1 and at most 8 ranks")
        if graph and getattr(comm, "timeout", None) is not None:
            # a host wait cannot be recorded in a CUDA graph: captured
            # collectives are bounded by the process group's own timeout
            raise ValueError("ShardedChainAcceptor: a graph needs a comm without a host timeout")
        self.target, self.draft, self.drafts = target, draft, drafts
        self.k, self.v0, self.sampling, self.comm = k, v0, sampling, comm
        dev = target.device
        B, Vs = int(target.shape[0]), int(target.shape[2])
        self.B, self.Vs = B, Vs
        rows_p, rows_q = B * (k + 1), B * k
        rows = rows_p + rows_q
        self.rows_p, self.rows_q, self.rows = rows_p, rows_q, rows
        i32, i64 = torch.int32, torch.int64
        self.step_dev = torch.full((1,), int(sampling.step), dtype=i32, device=dev)
        self.mx = torch.empty(rows, dtype=torch.float32, device=dev)
        self.am = torch.empty(rows, dtype=i32, device=dev)
        self.lst = torch.empty((rows, SHARD_LIST_CAP, 2), dtype=i32, device=dev)
        self.lnum = torch.empty(rows, dtype=i32, device=dev)
        self.stats = torch.empty((rows, 260), dtype=i64, device=dev)
        self.G = torch.empty(rows, dtype=i64, device=dev)
        self.cand = torch.empty((rows, SHARD_CAND + 1, 2), dtype=i32, device=dev)
        self.tau = torch.empty(rows, dtype=i32, device=dev)
        self.nuc = torch.empty(rows, dtype=i64, device=dev)
        self.ok = torch.empty(rows, dtype=i32, device=dev)
        self.pq = torch.empty((2, rows_q), dtype=i64, device=dev)
        self.acc = torch.empty(B, dtype=i32, device=dev)
        self.win = torch.empty((B, 4), dtype=i32, device=dev)
        self.tok = torch.empty(B, dtype=i32, device=dev)
        self.out = torch.empty((B, k + 1), dtype=i32, device=dev)
        self.graph = None
        self._issue()  # eager once: warms the collectives up and checks the sequence
        torch.cuda.synchronize(dev)
        if graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._issue()
            self.graph = g

    def _issue(self):
        import ctypes as C

        import torch

        import specdec as S

        L = S.lib()
        p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
        st = C.c_void_p(torch.cuda.current_stream(self.target.device).cuda_stream)
        comm, sp, k, B, Vs, v0 = self.comm, self.sampling, self.k, self.B, self.Vs, self.v0
        T, tp = float(sp.temperature), float(sp.top_p)
        rows_p, rows_q, rows = self.rows_p, self.rows_q, self.rows
        tgt, dr, drafts = self.target, self.draft, self.drafts
        S.check(L.specdec_shard_row_max(p(tgt), rows_p, p(dr), rows_q, Vs, v0, p(self.mx), p(self.am), st))
        gm, ga = comm.all_gather(self.mx), comm.all_gather(self.am)
        S.check(L.specdec_shard_merge_max(p(gm), p(ga), comm.world, rows, p(self.mx), p(self.am), st))
        S.check(L.specdec_shard_mass_hist(p(tgt), rows_p, p(dr), rows_q, Vs, p(self.mx), T, SHARD_LIST_CAP,
                                          p(self.lst), p(self.lnum), p(self.stats), st))
        comm.all_reduce_sum(self.stats)
        S.check(L.specdec_shard_cross(p(self.stats), rows, tp, p(self.mx), T, p(self.lst), SHARD_LIST_CAP,
                                      p(self.lnum), p(self.G), p(self.cand), st))
        gcand = comm.all_gather(self.cand)
        S.check(L.specdec_shard_union_select(p(gcand), comm.world, rows, p(self.stats), p(self.G), tp, p(self.tau),
                                             p(self.nuc), p(self.ok), st))
        pmax, qmax = self.mx[:rows_p], self.mx[rows_p:]
        ptau, qtau = self.tau[:rows_p], self.tau[rows_p:]
        pnuc, qnuc = self.nuc[:rows_p], self.nuc[rows_p:]
        S.check(L.specdec_shard_point_mass(p(tgt), p(dr), p(drafts), B, k, Vs, v0, T, p(pmax), p(ptau), p(qmax),
                                           p(qtau), p(self.pq[0]), p(self.pq[1]), st))
        comm.all_reduce_sum(self.pq)
        S.check(L.specdec_shard_accept_test(p(drafts), B, k, C.byref(sp), p(self.am[:rows_p]), p(pnuc), p(qnuc),
                                            p(self.pq[0]), p(self.pq[1]), p(self.acc), p(self.step_dev), st))
        S.check(L.specdec_shard_draw_winners(p(tgt), p(dr), B, k, Vs, v0, C.byref(sp), p(self.acc), p(pmax),
                                             p(ptau), p(qmax), p(qtau), p(pnuc), p(qnuc), p(self.win),
                                             p(self.step_dev), st))
        gwin = comm.all_gather(self.win)
        S.check(L.specdec_shard_draw_merge(p(gwin), comm.world, B, k, p(self.acc), p(self.tok), st))
        idx = torch.arange(k + 1, device=tgt.device)[None, :]
        a = self.acc.long()[:, None]
        ext = torch.cat([drafts, torch.full((B, 1), -1, dtype=torch.int32, device=tgt.device)], 1)
        out = torch.where(idx < a, ext, torch.full_like(ext, -1))
        self.out.copy_(torch.where(idx == a, self.tok[:, None], out))

    def __call__(self, step: int | None = None):
        """(accepted [B], out_tokens [B, k+1]) on the device, the same on every rank."""
        if step is not None:
            self.step_dev.fill_(int(step))
        if self.graph is not None:
            self.graph.replay()
        else:
            self._issue()
        if bool(self.ok.all().item()):  # the same on every rank: computed from exchanged data only
            return self.acc, self.out
        import specdec as S

        s0 = self.sampling
        sp = S.sampling(s0.temperature, s0.top_p, s0.seed, int(self.step_dev.item()) if step is None else int(step))
        return accept_chain_vocab_sharded(self.target, self.draft, self.drafts, self.k, self.v0, sp, self.comm)

    def close(self):
        self.graph = None


# ----------------------------------------------------------------------
# Rank failure detection (host side)
# ----------------------------------------------------------------------
# A rank that leaves (an exception between steps, a clean or abrupt exit) or
# stops answering must not leave the others waiting for ever.  Two mechanisms,
# both on the host, neither touching a GPU kernel:
#   * guarded collectives: TorchComm(timeout=...) issues each collective
#     asynchronously and waits at most `timeout` seconds for it; a collective
#     that a peer never joins, or whose peer connection closed, raises
#     RankLost (status ETIMEOUT) instead of blocking.  Under NCCL the process
#     group's own watchdog (which polls the communicator's asynchronous error
#     and aborts it after the group timeout) is the outer bound; collectives
#     captured in a CUDA graph cannot take a host wait and rely on it alone;
#   * a step heartbeat through the process group's key-value store
#     (PeerMonitor): before launching step s a rank publishes s and waits, at
#     most `timeout` seconds, until every peer has published s too.  A peer
#     that left between steps has published a "left" mark and is reported at
#     once; a peer that stalled or died silently is reported when the wait
#     runs out.  Either way the rank learns of it before its next launch, with
#     none of its kernels or collectives in flight.
# The reference server has no multi-process path; the failure semantics follow
# its error convention for the new ABI (status codes, here ETIMEOUT).


class RankLost(RuntimeError):
    """A peer rank left, died or did not answer within the timeout.  `code` is
    the library status SPECDEC_ETIMEOUT; `rank` the peer when it is known."""

    def __init__(self, msg: str, rank: int | None = None):
        from specdec import ETIMEOUT

        super().__init__(f"specdec error {ETIMEOUT}: {msg}")
        self.code = ETIMEOUT
        self.rank = rank


def guarded_wait(work, timeout: float, what: str):
    """Waits for an asynchronous collective at most `timeout` seconds; a
    timeout or a closed peer connection becomes RankLost."""
    import datetime

    try:
        work.wait(timeout=datetime.timedelta(seconds=float(timeout)))
    except RuntimeError as e:
        raise RankLost(f"{what}: {e}") from e


class PeerMonitor:
    """Step heartbeat of the ranks through a torch.distributed Store (the one
    the process group was created with: TCPStore, FileStore, ...).

    begin_step(s) publishes s and returns once every peer has published s;
    leave() marks this rank gone (call it when leaving between steps, e.g.
    from an exception handler, or use `with monitor.member(): ...`).  Raises
    RankLost naming the peer that left, or the first one still behind when
    `timeout` seconds have passed."""

    def __init__(self, store, rank: int, world: int, timeout: float = 5.0, prefix: str = "specdec/hb",
                 poll: float = 0.005):
        if world <= 0 or not 0 <= rank < world:
            raise ValueError(f"bad monitor: rank={rank} world={world}")
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.prefix, self.poll = float(timeout), prefix, float(poll)
        self.step = -1

    def _key(self, kind: str, r: int) -> str:
        return f"{self.prefix}/{kind}/{r}"

    def leave(self):
        try:
            self.store.set(self._key("left", self.rank), "1")
        except RuntimeError:
            pass  # the store is gone too: the peers find out from their own waits

    def peer_left(self, r: int) -> bool:
        return self.store.check([self._key("left", r)])

    def begin_step(self, step: int):
        try:
            self._begin_step(int(step))
        except RankLost:
            raise
        except RuntimeError as e:  # the store itself is unreachable (its host rank is gone)
            raise RankLost(f"step store unreachable at step {int(step)}: {e}") from e

    def _begin_step(self, step: int):
        import time

        self.store.set(self._key("step", self.rank), str(step))
        self.step = step
        deadline = time.monotonic() + self.timeout
        waiting = [r for r in range(self.world) if r != self.rank]
        while waiting:
            behind = []
            for r in waiting:
                if self.peer_left(r):
                    raise RankLost(f"rank {r} left before step {step}", r)
                k = self._key("step", r)
                if not (self.store.check([k]) and int(self.store.get(k)) >= step):
                    behind.append(r)
            waiting = behind
            if not waiting:
                break
            if time.monotonic() > deadline:
                r = waiting[0]
                raise RankLost(f"rank {r} did not reach step {step} within {self.timeout:g} s", r)
            time.sleep(self.poll)

    def member(self):
        """Context manager: marks this rank gone if the body raises."""
        import contextlib

        @contextlib.contextmanager
        def _cm():
            try:
                yield self
            except BaseException:
                self.leave()
                raise

        return _cm()
