"""Expert-parallel MoE block (NCCL all-to-all over NVLink) against the single-GPU
block on the same tokens: bf16 tolerance (cosine >= 0.999, max-abs <= 2e-2 x scale).
One rank on one GPU, and 2, 4 or 8 ranks where that many GPUs are present."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    for p in (str(ROOT), str(ROOT / "sglang-omni_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from omni_b200.config import MoEConfig
        from omni_b200.moe import MoEBlock, init_moe_weights
        from omni_b200.moe_ep import ExpertParallelMoE

        cfg, H = MoEConfig(), 1024
        g = torch.Generator(device=dev).manual_seed(0)  # identical weights on every rank
        w = init_moe_weights(cfg, H, generator=g, device=dev)
        T = 16 + (37 * rank) % 48  # uneven token counts, within max_tokens (64)
        gt = torch.Generator(device=dev).manual_seed(100 + rank)
        h = torch.randn(T, H, generator=gt, device=dev).to(torch.bfloat16)
        gain = torch.ones(H, device=dev, dtype=torch.bfloat16)
        ss = h.float().view(T, 8, 128).pow(2).sum(-1).t().contiguous()
        ep = ExpertParallelMoE(cfg, H, max_tokens=64, device=dev)
        h_ep, ss_ep = h.clone(), ss.clone()
        ep.forward(h_ep, ss_ep, 8, gain, 1e-6, ep.local_weights(w))
        single = MoEBlock(cfg, H, max_batch=T, device=dev)
        h_1, ss_1 = h.clone(), ss.clone()
        single.forward(h_1, ss_1, 8, gain, 1e-6, w)
        torch.cuda.synchronize()
        a, b = h_ep.float().flatten(), h_1.float().flatten()
        cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
        err = (a - b).abs().max().item()
        d_ep, d_1 = (h_ep.float() - h.float()).flatten(), (h_1.float() - h.float()).flatten()
        cos_d = torch.nn.functional.cosine_similarity(d_ep, d_1, dim=0).item()
        np.save(os.path.join(out_dir, f"ep{rank}.npy"),
                np.array([cos, err, b.abs().max().item(), cos_d, int(torch.equal(ep.local.topk_ids[:T], single.topk_ids[:T]))]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ep_moe_matches_single_gpu(tmp_path, world):
    """world 1 runs the same block (one NCCL rank, local all-to-alls, the shared expert
    on its side stream) on one GPU; world N needs N GPUs (128 experts, 128 / N a rank)."""
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        cos, err, scale, cos_d, same_route = np.load(tmp_path / f"ep{r}.npy")
        assert same_route == 1
        assert cos >= 0.999 and err <= 2e-2 * max(scale, 1.0), (r, cos, err, scale)
        assert cos_d >= 0.99, (r, cos_d)


@pytest.mark.parametrize("world,tokens,cap", [(2, 64, 64), (8, 256, 256), (4, 37, 50), (1, 5, 8)])
def test_ep_pack_kernel_matches_restatement(world, tokens, cap):
    """omni_moe_ep_pack against oracle.ep: every used row, every unused row's ids and the
    part index bit-exact (the config-3 shapes: hidden 1024, top-8 of 128 experts)."""
    from oracle.ep import dispatch_plan, pack_rows, part_index

    from omni_b200.moe_ep import ep_pack, packed_row_bytes

    dev = torch.device("cuda", 0)
    H, E, K = 1024, 128, 8
    g = torch.Generator().manual_seed(world * 100 + tokens)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(tokens)]).to(torch.int32)
    tw = torch.rand(tokens, K, generator=g)
    xq = torch.randint(0, 256, (tokens, H), generator=g, dtype=torch.uint8)
    xs = torch.rand(tokens, H // 128, generator=g)
    rb = packed_row_bytes(H, K)
    e_local = E // world
    has, pos, flat, local_ids = dispatch_plan(ids, world, e_local, cap)
    want = torch.zeros(world * cap + 1, rb, dtype=torch.uint8)
    pack_rows(want, H, K, xq, xs, local_ids, tw, flat)
    want_pidx = part_index(has, pos, cap)
    send = torch.full((world * cap, rb), 0xAB, dtype=torch.uint8, device=dev)
    pidx = torch.full((tokens, world), -7, dtype=torch.int32, device=dev)
    ep_pack(send, H, K, ids.to(dev), tw.to(dev), xq.to(dev), xs.to(dev), world, e_local, cap, pidx)
    torch.cuda.synchronize()
    got = send.cpu()
    assert torch.equal(pidx.cpu(), want_pidx)
    G = H // 128
    got_ids = got[:, H + 4 * G: H + 4 * G + 4 * K].view(torch.int32)
    want_ids = want[: world * cap, H + 4 * G: H + 4 * G + 4 * K].view(torch.int32)
    assert torch.equal(got_ids, want_ids)
    used = want_pidx[want_pidx >= 0].long()
    assert torch.equal(got[used, : H + 4 * G + 8 * K], want[used, : H + 4 * G + 8 * K])
