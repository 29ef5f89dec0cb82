"""Sequence-parallel chain on 2 and 4 GPUs (NCCL) against the same chain on 1 GPU.

Each rank computes its shard of the video and of the text tokens; the shards,
concatenated, must equal the single-GPU block output (same kernels, same weights;
attention sees the same keys, gathered in another order and split at the cache
rows, merged by log-sum-exp).  Each world size is skipped with fewer visible
GPUs than ranks.  Run with NCCL_NVLS_ENABLE=0 semantics not needed: no
rank dies mid-collective here.
"""
import datetime
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent
HID, HEADS, FFN, IMG, TXT, CACHE = 512, 4, 1024, 160, 32, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(dev):
    from joyomni_ops import chain, rope

    g = torch.Generator().manual_seed(5)
    w = chain.random_block_weights(HID, HEADS, FFN, device=dev, seed=9)
    img = torch.randn(IMG, HID, generator=g).to(torch.bfloat16)
    txt = torch.randn(TXT, HID, generator=g).to(torch.bfloat16)
    vec = (0.1 * torch.randn(6, HID, generator=g)).to(torch.bfloat16)
    ck = torch.randn(CACHE, HEADS, 128, generator=g).to(torch.bfloat16)
    cv = torch.randn(CACHE, HEADS, 128, generator=g).to(torch.bfloat16)
    cos, sin = rope.video_chunk_tables(2, 8, IMG // 16, 3)
    return w, img, txt, vec, ck, cv, cos, sin


def _run_chain(dev, world, rank, group):
    from joyomni_ops import chain

    w, img, txt, vec, ck, cv, cos, sin = _inputs(dev)
    b0, b1 = chain.shard_range(IMG, world, rank)
    t0, t1 = chain.shard_range(TXT, world, rank)
    bufs = chain.KVBuffers(CACHE, IMG, TXT, HEADS, 128, world, dev)
    bufs.k[:CACHE].copy_(ck)
    bufs.v[:CACHE].copy_(cv)
    a, b = chain.block_forward(img[b0:b1].to(dev), txt[t0:t1].to(dev), vec.to(dev), cos[b0:b1].to(dev),
                               sin[b0:b1].to(dev), w, bufs, group=group, rank=rank)
    torch.cuda.synchronize()
    return a.cpu(), b.cpu()


def _worker(rank, world, port, q):
    try:
        sys.path[:0] = [str(REPO), str(REPO / "joyai-video-edit_b200")]
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        a, b = _run_chain(torch.device("cuda", rank), world, rank, dist.group.WORLD)
        q.put((rank, a, b, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, None, None, f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=3)}"))


@pytest.mark.parametrize("world", [2, 4])
def test_sp_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ref_img, ref_txt = _run_chain(torch.device("cuda", 0), 1, 0, None)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, a, b, err = q.get(timeout=300)
        res[r] = (a, b, err)
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert res[r][2] is None, res[r][2]
    img_sp = torch.cat([res[r][0] for r in range(world)])
    txt_sp = torch.cat([res[r][1] for r in range(world)])
    for got, want in ((img_sp, ref_img), (txt_sp, ref_txt)):
        d = (got.float() - want.float()).abs().max().item()
        scale = want.float().abs().max().item()
        assert d <= 1e-2 * scale, f"SP result differs from single GPU by {d} (max |ref| {scale})"
