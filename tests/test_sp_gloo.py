"""Host logic of the sequence-parallel chain on CPU ranks (gloo, world_size 2 and 4).

Checks the token sharding (video and text tokens) and the in-place K/V
all-gather placement of joyomni_ops.chain (which on GPUs runs over NCCL): every
rank's block [its video | its text] lands in its place, plus the failure path: a rank
that never joins the collective makes the others fail with an error instead of
hanging (short process-group timeout).
"""
import datetime
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        sys.path[:0] = [str(REPO), str(REPO / "joyai-video-edit_b200")]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        timeout = datetime.timedelta(seconds=60 if mode == "ok" else 5)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
        from joyomni_ops import chain

        cache, img, txt, H, D = 6, 8, 4, 2, 4
        b0, b1 = chain.shard_range(img, world, rank)
        assert (b1 - b0) * world == img
        bufs = chain.KVBuffers(cache, img, txt, H, D, world, "cpu", dtype=torch.float32)
        bufs.k.fill_(-1.0)
        bufs.v.fill_(-2.0)
        # each rank writes its own token rows: value = global token index (+0.5 for v),
        # text tokens 100 + index
        def toks(a, b, base=0.0):
            return (base + torch.arange(a, b, dtype=torch.float32)).view(-1, 1, 1).expand(-1, H, D)
        t0, t1 = chain.shard_range(txt, world, rank)
        bufs.k[bufs.img_kv_rows(rank)] = toks(b0, b1)
        bufs.v[bufs.img_kv_rows(rank)] = toks(b0, b1) + 0.5
        bufs.k[bufs.txt_kv_rows(rank)] = toks(t0, t1, 100.0)
        bufs.v[bufs.txt_kv_rows(rank)] = toks(t0, t1, 100.0) + 0.5
        if mode == "absent" and rank == 1:
            q.put((rank, "skipped"))
            return  # never joins the collective
        if mode == "killed" and rank == 1:
            os._exit(17)  # the process dies between steps, with nothing in flight
        if mode == "mismatch" and rank == 1:
            # a rank whose buffers were sized for a different chunk length
            bufs = chain.KVBuffers(cache, img + 2 * world, txt, H, D, world, "cpu", dtype=torch.float32)
        chain.gather_chunk_kv(bufs, rank, None)
        for r in range(world):  # every rank's block, in rank order
            rb0, rb1 = chain.shard_range(img, world, r)
            rt0, rt1 = chain.shard_range(txt, world, r)
            assert torch.equal(bufs.k[bufs.img_kv_rows(r)], toks(rb0, rb1))
            assert torch.equal(bufs.v[bufs.img_kv_rows(r)], toks(rb0, rb1) + 0.5)
            assert torch.equal(bufs.k[bufs.txt_kv_rows(r)], toks(rt0, rt1, 100.0))
            assert torch.equal(bufs.v[bufs.txt_kv_rows(r)], toks(rt0, rt1, 100.0) + 0.5)
        assert (bufs.k[:cache] == -1).all() and (bufs.v[:cache] == -2).all()
        # the gathered rows are exactly every video and text token once
        keys = sorted(bufs.k[bufs.gathered_rows(), 0, 0].tolist())
        assert keys == sorted(list(range(img)) + [100.0 + i for i in range(txt)])
        q.put((rank, "ok"))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, f"error: {type(e).__name__}: {e}\n{traceback.format_exc(limit=2)}"))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    res = {}
    while not q.empty():
        r, msg = q.get()
        res[r] = msg
    _run.exitcodes = [p.exitcode for p in procs]
    return res, alive


def test_shard_range():
    sys.path[:0] = [str(REPO / "joyai-video-edit_b200")]
    from joyomni_ops import chain

    assert chain.shard_range(10800, 8, 7) == (9450, 10800)
    with pytest.raises(ValueError):
        chain.shard_range(10801, 2, 0)


def test_kv_gather_two_ranks():
    res, alive = _run("ok")
    assert not alive and res == {0: "ok", 1: "ok"}, res


def test_kv_gather_four_ranks():
    """Four ranks: two video tokens and one text token each, blocks in rank order."""
    res, alive = _run("ok", world=4)
    assert not alive and res == {r: "ok" for r in range(4)}, res


def test_absent_rank_fails_cleanly():
    res, alive = _run("absent")
    assert not alive, "a rank hung"
    assert res.get(1) == "skipped"
    assert res.get(0, "").startswith("error"), res


def test_killed_rank_fails_cleanly():
    """A rank that dies (process exit) between steps: the survivor's next collective
    ends with an error within the process-group timeout instead of hanging."""
    res, alive = _run("killed")
    assert not alive, "a rank hung"
    assert _run.exitcodes[1] == 17, _run.exitcodes
    assert res.get(0, "").startswith("error"), res


def test_mismatched_shapes_fail_cleanly():
    """Ranks whose K/V buffers disagree on the chunk length: the all-gather reports an
    error on every rank (or times out with one) instead of hanging or writing garbage."""
    res, alive = _run("mismatch")
    assert not alive, "a rank hung"
    assert all(str(res.get(r, "error")).startswith("error") for r in (0, 1)), res
