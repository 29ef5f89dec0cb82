"""Copy-engine K/V all-gather (``chain.PeerGather``) on 2, 4 and 8 GPUs, one process per GPU.

* The gather alone: every rank writes rank- and step-dependent rows into its block,
  gathers, and must hold every rank's block bit for bit, over several steps (each step
  rewrites the block after ``before_write``, so a pull of the previous step's rows
  racing the rewrite would show up as a mismatch).
* The block: ``block_forward(..., peers=...)`` for two steps equals the single-GPU
  block and the NCCL-gathered block.
No bounded wait may have expired (device fault counter 0).  Skipped with fewer GPUs
than ranks.
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
sys.path.insert(0, str(Path(__file__).resolve().parent))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    sys.path[:0] = [str(REPO), str(REPO / "joyai-video-edit_b200")]
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


def _gather_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from joyomni_ops import cabi, chain

        dev = torch.device("cuda", rank)
        cache, img, txt, heads = 96, 64 * world, 8 * world, 4
        bufs = chain.KVBuffers(cache, img, txt, heads, 128, world, dev, ipc=True)
        peers = chain.PeerGather(bufs, rank, world, dist.group.WORLD)
        side = torch.cuda.Stream(dev)

        def rows(r, step, t):
            g = torch.Generator().manual_seed(1000 * step + 10 * r + t)
            return torch.randn(bufs.block, heads, 128, generator=g).to(torch.bfloat16)

        bad = []
        for step in range(4):
            cur = torch.cuda.current_stream()
            peers.before_write(cur)
            bufs.k[bufs.block_rows(rank)].copy_(rows(rank, step, 0).to(dev))
            bufs.v[bufs.block_rows(rank)].copy_(rows(rank, step, 1).to(dev))
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                peers.gather(side)
            cur.wait_stream(side)
            torch.cuda.synchronize()
            for r in range(world):
                for t, buf in ((0, bufs.k), (1, bufs.v)):
                    if not torch.equal(buf[bufs.block_rows(r)].cpu(), rows(r, step, t)):
                        bad.append((step, r, t))
        faults = cabi.device_fault_count()
        peers.close()
        bufs.close()
        q.put((rank, bad, faults, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, None, None, f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=4)}"))


def _block_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        import test_sp_gpu as sp
        from joyomni_ops import cabi, chain

        dev = torch.device("cuda", rank)
        w, img, txt, vec, ck, cv, cos, sin = sp._inputs(dev)
        b0, b1 = chain.shard_range(sp.IMG, world, rank)
        t0, t1 = chain.shard_range(sp.TXT, world, rank)
        bufs = chain.KVBuffers(sp.CACHE, sp.IMG, sp.TXT, sp.HEADS, 128, world, dev, ipc=True)
        bufs.k[:sp.CACHE].copy_(ck)
        bufs.v[:sp.CACHE].copy_(cv)
        peers = chain.PeerGather(bufs, rank, world, dist.group.WORLD)
        outs = []
        text = torch.cuda.Stream(dev)
        for step in range(2):  # the second step with the text branches on their own stream
            a, b = chain.block_forward(img[b0:b1].to(dev), txt[t0:t1].to(dev), vec.to(dev), cos[b0:b1].to(dev),
                                       sin[b0:b1].to(dev), w, bufs, group=dist.group.WORLD, rank=rank,
                                       peers=peers, text_stream=text if step else None)
            torch.cuda.synchronize()
            outs.append((a.cpu(), b.cpu()))
        faults = cabi.device_fault_count()
        peers.close()
        bufs.close()
        q.put((rank, outs, faults, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, None, None, f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=4)}"))


def _spawn(target, world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out, faults, err = q.get(timeout=300)
        res[r] = (out, faults, err)
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert res[r][2] is None, res[r][2]
        assert res[r][1] == 0, f"rank {r}: {res[r][1]} bounded waits expired"
    return res


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_gather_every_block_every_step(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(_gather_worker, world)
    for r in range(world):
        assert res[r][0] == [], f"rank {r}: wrong rows (step, source rank, tensor): {res[r][0][:8]}"


@pytest.mark.parametrize("world", [2, 4])
def test_block_with_peer_gather_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import test_sp_gpu as sp

    ref_img, ref_txt = sp._run_chain(torch.device("cuda", 0), 1, 0, None)
    res = _spawn(_block_worker, world)
    for step in range(2):
        img_sp = torch.cat([res[r][0][step][0] for r in range(world)])
        txt_sp = torch.cat([res[r][0][step][1] for r in range(world)])
        for got, want in ((img_sp, ref_img), (txt_sp, ref_txt)):
            d = (got.float() - want.float()).abs().max().item()
            scale = want.float().abs().max().item()
            assert d <= 1e-2 * scale, f"step {step}: differs from single GPU by {d} (max |ref| {scale})"
    for r in range(world):  # the second step repeats the first bit for bit
        assert torch.equal(res[r][0][0][0], res[r][0][1][0]) and torch.equal(res[r][0][0][1], res[r][0][1][1])


def test_peer_flags_one_gpu(dev):
    """The flag kernels on one GPU with this process's own flag array: a signalled word
    releases the wait at once; a word that nothing sets makes the bounded wait expire
    (2 s): the fault counter records it and the device stays usable."""
    import ctypes as C
    import time

    from joyomni_ops import cabi, chain

    cabi.device_fault_count()  # clear
    flags = chain.IpcAlloc(256, dev)
    try:
        world = 4
        tab = (C.c_void_p * world)(*[flags.ptr + 8 * q for q in range(world)])
        st = torch.cuda.current_stream().cuda_stream
        cabi.call("jo_peer_signal", tab, world, 7, st)
        cabi.call("jo_peer_wait", flags.ptr, world, 0, 7, st)
        torch.cuda.synchronize()
        assert cabi.device_fault_count() == 0
        assert flags.tensor((32,), torch.int64)[:world].tolist() == [7] * world
        t0 = time.perf_counter()
        cabi.call("jo_peer_wait", flags.ptr, world, 0, 8, st)  # nothing stores 8
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 >= 1.5
        assert cabi.device_fault_count() == world - 1  # one expiry per waited word (q != skip)
        x = torch.ones(4, device=dev)
        assert (x + 1).sum().item() == 8  # the context is still usable
    finally:
        flags.free()
