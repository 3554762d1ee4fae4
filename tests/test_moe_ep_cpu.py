"""Expert-parallel MoE dispatch/combine plumbing on CPU: gloo, world size 2.

The device path (moe_ep.ExpertParallelMoE) packs its send buffer with the
omni_moe_ep_pack kernel, whose CPU restatement is oracle.ep (dispatch_plan,
pack_rows, part_index; tests/test_moe_ep_gpu.py holds the kernel to it bit for
bit), exchanges fixed blocks with all_to_all_single and combines the returned
partial rows through the part index.  Here the restatement runs on CPU tensors with
a stand-in expert (partial = sum_k w_k * (global expert id + 1)): every token must
reach exactly the ranks that hold its experts, with its own row, ids and weights,
and get back the sum over all of its experts.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
H, E, K, W, CAP = 256, 8, 3, 2, 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(rank: int):
    T = 5 if rank == 0 else 3
    g = torch.Generator().manual_seed(10 + rank)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    if rank == 1:
        ids[0] = torch.tensor([0, 1, 2], dtype=torch.int32)  # all on rank 0
    xq = torch.zeros(T, H, dtype=torch.uint8)
    for t in range(T):
        xq[t] = rank * 50 + t
    xs = torch.tensor([[rank * 100.0 + t] * (H // 128) for t in range(T)], dtype=torch.float32)
    tw = torch.rand(T, K, generator=g)
    return ids, xq, xs, tw


def _worker(rank: int, port: int, out_dir: str) -> None:
    for p in (str(ROOT), str(ROOT / "sglang-omni_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=W)
    try:
        from omni_b200.moe_ep import packed_row_bytes
        from oracle.ep import dispatch_plan, pack_rows, part_index

        e_local = E // W
        ids, xq, xs, tw = _tokens(rank)
        rb = packed_row_bytes(H, K)
        send = torch.zeros(W * CAP + 1, rb, dtype=torch.uint8)
        recv = torch.zeros(W * CAP, rb, dtype=torch.uint8)
        has, pos, flat, local_ids = dispatch_plan(ids, W, e_local, CAP)
        pack_rows(send, H, K, xq, xs, local_ids, tw, flat)
        dist.all_to_all_single(recv, send[: W * CAP])
        G = H // 128
        r_ids = recv[:, H + 4 * G: H + 4 * G + 4 * K].view(torch.int32)
        r_w = recv[:, H + 4 * G + 4 * K: H + 4 * G + 8 * K].view(torch.float32)
        r_s = recv[:, H: H + 4 * G].view(torch.float32)
        # check every received row against its source token
        errors = []
        for src in range(W):
            s_ids, s_xq, s_xs, s_tw = _tokens(src)
            expect = [t for t in range(s_ids.shape[0]) if ((s_ids[t].long() // e_local) == rank).any()]
            for j in range(CAP):
                row = src * CAP + j
                if j < len(expect):
                    t = expect[j]
                    if not torch.equal(recv[row, :H], s_xq[t]) or not torch.equal(r_s[row], s_xs[t]):
                        errors.append(("payload", src, j))
                    want = torch.where(s_ids[t].long() // e_local == rank, s_ids[t].long() - rank * e_local,
                                       torch.full((K,), -1, dtype=torch.long))
                    if r_ids[row].tolist() != want.tolist() or not torch.equal(r_w[row], s_tw[t]):
                        errors.append(("meta", src, j))
                elif (r_ids[row] != -1).any():
                    errors.append(("padding carries an expert", src, j))
        # stand-in expert: partial = sum over local entries of w * (global id + 1)
        ret_send = torch.zeros(W * CAP, H, dtype=torch.float32)
        glob = torch.where(r_ids >= 0, r_ids.long() + rank * e_local, torch.full_like(r_ids, -1).long())
        val = torch.where(r_ids >= 0, r_w * (glob + 1).float(), torch.zeros_like(r_w)).sum(1)
        ret_send[:] = val[:, None]
        ret_recv = torch.zeros_like(ret_send)
        dist.all_to_all_single(ret_recv, ret_send)
        pidx = part_index(has, pos, CAP)
        routed = torch.zeros(ids.shape[0])
        for d in range(W):
            sel = pidx[:, d] >= 0
            routed[sel] += ret_recv[pidx[sel, d].long(), 0]
        want = (tw * (ids.long() + 1).float()).sum(1)
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([len(errors), float((routed - want).abs().max())]))
    finally:
        dist.destroy_process_group()


def test_ep_dispatch_combine_two_gloo_ranks(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(port, str(tmp_path)), nprocs=W, start_method="spawn")
    for r in range(W):
        n_err, max_err = np.load(tmp_path / f"r{r}.npy")
        assert n_err == 0
        assert max_err < 1e-5
