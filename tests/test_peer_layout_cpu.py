"""The peer-memory exchange layout of PeerContextParallel on two CPU ranks
(gloo): each rank's pushes are emulated by writing its payload, with the
same offsets, strides and columns the GPU push uses, into every rank's byte
buffer; the regions the consuming kernels read (candidate rows in rank
order, keys then ids; strided partial slots) must then hold every rank's
data in place."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

B, H, N = 3, 5, 12


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _push(buf, payload, rows, row_bytes, src_stride, dst_offset, dst_stride, dst_col):
    """What aether_peer_push stores into one rank's buffer."""
    for r in range(rows):
        d0 = dst_offset + dst_col + r * dst_stride
        buf[d0: d0 + row_bytes] = payload[r * src_stride: r * src_stride + row_bytes]


def _worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "deepseek-v4-codebase_b200"))
    from aether_kernels.dist import peer_layout

    lay = peer_layout(B, H, N, world)
    buf = torch.zeros(lay["total"], dtype=torch.uint8)
    # this rank's candidates [2][B][N] (keys, ids) and partial (O then (max, sum))
    cand = torch.arange(2 * B * N, dtype=torch.int32).view(2, B, N) + 10000 * rank
    part = torch.zeros(lay["slot"] // 4, dtype=torch.float32)
    part[: (lay["o_bytes"] + B * H * 8) // 4] = torch.arange((lay["o_bytes"] + B * H * 8) // 4).float() + 0.5 * rank
    payloads = [None] * world
    dist.all_gather_object(payloads, (cand.view(torch.uint8).reshape(-1).clone(), part.view(torch.uint8).clone()))
    for r, (pc, pp) in enumerate(payloads):  # every rank r stores into this rank's buffer
        _push(buf, pc, 2 * B, N * 4, N * 4, lay["off_k"], world * N * 4, r * N * 4)
        _push(buf, pp, 1, lay["slot"], lay["slot"], lay["off_p"], lay["slot"], r * lay["slot"])
    ok = True
    keys = buf[lay["off_k"]: lay["off_k"] + B * world * N * 4].view(torch.int32).view(B, world * N)
    ids = buf[lay["off_i"]: lay["off_i"] + B * world * N * 4].view(torch.int32).view(B, world * N)
    for r in range(world):
        ref = torch.arange(2 * B * N, dtype=torch.int32).view(2, B, N) + 10000 * r
        ok &= bool(torch.equal(keys[:, r * N:(r + 1) * N], ref[0])) and bool(torch.equal(ids[:, r * N:(r + 1) * N], ref[1]))
    # partial views as aether_lse_merge_strided reads them: rank stride slot / 4 floats
    allp = buf[lay["off_p"]: lay["total"]].view(torch.float32).view(world, lay["slot"] // 4)
    for r in range(world):
        o = allp[r, : B * H * 128].view(B, H, 128)
        ml = allp[r, lay["o_bytes"] // 4: lay["o_bytes"] // 4 + B * H * 2].view(B, H, 2)
        base = torch.arange((lay["o_bytes"] + B * H * 8) // 4).float() + 0.5 * r
        ok &= bool(torch.equal(o.reshape(-1), base[: B * H * 128])) and bool(torch.equal(ml.reshape(-1), base[B * H * 128:]))
    ok &= lay["off_k"] % 16 == 0 and lay["off_p"] % 16 == 0 and lay["slot"] % 16 == 0 and (N * 4) % 16 == 0
    q_out.put((rank, ok))
    dist.barrier()
    dist.destroy_process_group()


def test_peer_exchange_layout_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q_out.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(res.values()), res
