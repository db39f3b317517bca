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


def _reduce(dist, x: float, device: str, op) -> float:
    if dist is None:
        return float(x)
    import torch

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def reduce_max(dist, x: float, device: str = "cpu") -> float:
    return _reduce(dist, x, device, None if dist is None else dist.ReduceOp.MAX)


def reduce_sum(dist, x: float, device: str = "cpu") -> float:
    return _reduce(dist, x, device, None if dist is None else dist.ReduceOp.SUM)


def step_throughput(dist, ms: float, tokens: float, device: str = "cpu") -> dict:
    """Whole-job throughput of a timed run: tokens of all ranks over the
    slowest rank's device time.  Every rank must call it (it is collective)."""
    ms_max = reduce_max(dist, ms, device)
    tok = reduce_sum(dist, tokens, device)
    return {"ms_max": ms_max, "tokens": tok, "value": tok / (ms_max / 1e3) if ms_max > 0 else 0.0}


# ----------------------------------------------------------------------
# Vocabulary-sharded chain acceptance
# ----------------------------------------------------------------------
class TorchComm:
    """Collectives of a torch.distributed process group (NCCL for CUDA tensors)."""

    def __init__(self, dist, group=None):
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, t):
        import torch

        # flat in, flat out (the form every backend accepts), then [world, *shape]
        out = torch.empty(self.world * t.numel(), dtype=t.dtype, device=t.device)
        self.dist.all_gather_into_tensor(out, t.contiguous().view(-1), group=self.group)
        return out.view((self.world,) + tuple(t.shape))

    def all_reduce_sum(self, t):
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)
        return t

    def all_reduce_max(self, t):
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)
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
                                            p(acc), st))
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
                                                p(ep), p(eq), p(acc), st))
            win = torch.empty((B, 4), dtype=torch.int32, device=dev)
            S.check(L.specdec_shard_draw_winners(p(target), p(draft), B, k, Vs, v0, C.byref(sampling), p(acc),
                                                 p(pmax), p(ptau), p(qmax), p(qtau), p(pnuc), p(qnuc), p(win), st))
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
