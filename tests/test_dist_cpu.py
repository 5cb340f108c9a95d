"""The context-parallel orchestration on CPU ranks over gloo (world size 2),
with the compute steps done by the reference-math oracle: exact candidate
merge and log-sum-exp merge reproduce the single-process result."""
import os
import socket

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


def _problem(seed=0, nb=3000, H=4, D=32, top_k=64):
    g = torch.Generator().manual_seed(seed)
    scores = torch.rand(nb, generator=g) * 10
    scores[100:140] = scores[5]  # exact ties across the shard boundary region
    vals = torch.randn(nb, D, generator=g)
    q = torch.randn(H, D, generator=g)
    sink = torch.randn(H, generator=g)
    win = torch.randn(20, D, generator=g)
    return scores, vals, q, sink, win, top_k


def _topk(scores, ids, k):
    order = sorted(range(len(ids)), key=lambda j: (-float(scores[j]), int(ids[j])))[:k]
    return sorted(int(ids[j]) for j in order)


def _partial(q, src, scale):
    if src.shape[0] == 0:
        return torch.zeros_like(q), torch.stack([torch.full((q.shape[0],), float("-inf")), torch.zeros(q.shape[0])], -1)
    z = (q @ src.T) * scale
    m = z.max(-1).values
    e = torch.exp(z - m[:, None])
    return e @ src, torch.stack([m, e.sum(-1)], -1)


def _merge(po, pml, sink):
    m, l = pml[..., 0], pml[..., 1]
    M = torch.maximum(m.max(0).values, sink)
    a = torch.where(m == float("-inf"), torch.zeros_like(m), torch.exp(m - M))
    L = (a * l).sum(0) + torch.exp(sink - M)
    return (a[..., None] * po).sum(0) / L[:, None]


def _worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "deepseek-v4-codebase_b200"))
    from aether_kernels.dist import context_parallel_step

    scores, vals, q, sink, win, k = _problem()
    nb = scores.numel()
    per = (nb + world - 1) // world
    lo, hi = rank * per, min(nb, (rank + 1) * per)
    scale = 0.2

    def cands():
        local = _topk(scores[lo:hi], list(range(lo, hi)), k)
        ks = torch.tensor([float(scores[i]) for i in local] + [-1.0] * (k - len(local)))
        ids = torch.tensor(local + [-1] * (k - len(local)), dtype=torch.int64)
        return ks, ids

    def attend(all_k, all_i):
        valid = all_i[0] >= 0
        sel = _topk(all_k[0][valid], all_i[0][valid].tolist(), k)
        mine = [i for i in sel if lo <= i < hi]
        src = vals[mine]
        if rank == world - 1:
            src = torch.cat([src, win])
        po, pml = _partial(q, src, scale)
        return po[None], pml[None], torch.tensor(sel)[None]

    out, sel = context_parallel_step(lambda: tuple(t[None] for t in cands()), attend,
                                     lambda po, pml: _merge(po[:, 0], pml[:, 0], sink))
    if rank == 0:
        # by value: a tensor shared through the queue can outlive this process's fd listener
        q_out.put((out.numpy().copy(), sel.numpy().copy()))
    dist.destroy_process_group()


def test_context_parallel_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    out, sel = q_out.get(timeout=120)
    out, sel = torch.from_numpy(out), torch.from_numpy(sel)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    scores, vals, q, sink, win, k = _problem()
    ref_sel = _topk(scores, list(range(scores.numel())), k)
    assert sel[0].tolist() == ref_sel
    src = torch.cat([vals[ref_sel], win])
    z = (q @ src.T) * 0.2
    M = torch.maximum(z.max(-1).values, sink)
    e = torch.exp(z - M[:, None])
    ref = (e @ src) / (e.sum(-1) + torch.exp(sink - M))[:, None]
    torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)
