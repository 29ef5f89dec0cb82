"""One rank's share of the sequence-parallel block at the BASELINE chunk size, on one GPU.

The per-block chain of BASELINE configs[4] (10800 video + 512 text tokens, hidden 3072,
24 x 128 heads, FFN 12288, 4 cached chunks) sharded over P ranks gives every rank
10800/P video and 512/P text tokens: at P = 8, 1350 + 64 rows, the shapes the 8-GPU
run's kernels see (ragged GEMM row tiles, single-CTA text GEMMs, a 1414-query split
attention).  Here one process plays rank r of P: the other ranks' K/V blocks are filled
with the rows the single-GPU block computed for those tokens (exactly what the NCCL
all-gather would deliver), the gather itself is skipped, and the rank's outputs must
match the single-GPU block's rows for its tokens.  The collective is covered by
``test_sp_gpu.py`` (2 and 4 GPUs) and the sharding logic by ``test_sp_gloo.py``.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
HID, HEADS, FFN, IMG, TXT, CACHE = 3072, 24, 12288, 10800, 512, 4 * 10800
HD = HID // HEADS


@pytest.fixture(scope="module")
def single(dev):
    """The single-GPU block: weights, inputs, outputs and the K/V rows it packed."""
    from joyomni_ops import chain, rope

    g = torch.Generator().manual_seed(11)
    w = chain.random_block_weights(HID, HEADS, FFN, device=dev, seed=3)
    img = torch.randn(IMG, HID, generator=g).to(torch.bfloat16).to(dev)
    txt = torch.randn(TXT, HID, generator=g).to(torch.bfloat16).to(dev)
    vec = (0.1 * torch.randn(6, HID, generator=g)).to(torch.bfloat16).to(dev)
    cos, sin = rope.video_chunk_tables(3, 45, 80, 7, dims=(44, 42, 42))
    cos, sin = cos.to(dev), sin.to(dev)
    bufs = chain.KVBuffers(CACHE, IMG, TXT, HEADS, HD, 1, dev)
    gk = torch.Generator(device=dev).manual_seed(2)
    bufs.k[:CACHE].normal_(generator=gk)
    bufs.v[:CACHE].normal_(generator=gk)
    out_img, out_txt = chain.block_forward(img, txt, vec, cos, sin, w, bufs)
    torch.cuda.synchronize()
    return dict(w=w, img=img, txt=txt, vec=vec, cos=cos, sin=sin, k=bufs.k, v=bufs.v,
                out_img=out_img, out_txt=out_txt)


@pytest.mark.parametrize("world,rank", [(8, 0), (8, 7), (4, 2)])
def test_rank_shard_matches_single_gpu(single, dev, monkeypatch, world, rank):
    from joyomni_ops import chain

    s = single
    bufs = chain.KVBuffers(CACHE, IMG, TXT, HEADS, HD, world, dev)
    bufs.k[:CACHE].copy_(s["k"][:CACHE])
    bufs.v[:CACHE].copy_(s["v"][:CACHE])
    for q in range(world):  # every rank's block as the all-gather would leave it
        b0, b1 = chain.shard_range(IMG, world, q)
        t0, t1 = chain.shard_range(TXT, world, q)
        for dst, src in ((bufs.k, s["k"]), (bufs.v, s["v"])):
            dst[bufs.img_kv_rows(q)].copy_(src[CACHE + b0:CACHE + b1])
            dst[bufs.txt_kv_rows(q)].copy_(src[CACHE + IMG + t0:CACHE + IMG + t1])
    mine = [(t[bufs.img_kv_rows(rank)].clone(), t[bufs.txt_kv_rows(rank)].clone()) for t in (bufs.k, bufs.v)]
    bufs.k[bufs.block_rows(rank)].zero_()  # the rank's own block must be written by its pack
    bufs.v[bufs.block_rows(rank)].zero_()
    # the blocks are in place already: the split-attention path runs with no collective
    monkeypatch.setattr(chain, "gather_chunk_kv", lambda bufs, rank, group: None)
    b0, b1 = chain.shard_range(IMG, world, rank)
    t0, t1 = chain.shard_range(TXT, world, rank)
    a, b = chain.block_forward(s["img"][b0:b1], s["txt"][t0:t1], s["vec"], s["cos"][b0:b1], s["sin"][b0:b1],
                               s["w"], bufs, group=object(), rank=rank, side_stream=torch.cuda.Stream())
    torch.cuda.synchronize()
    # per-token ops: the rank's video K/V rows are the single-GPU rows bit for bit (the same
    # CTA-pair GEMM, fewer row tiles); its text rows come from the single-CTA GEMM (at most
    # 128 rows) instead of the CTA-pair one, so they are compared within the block tolerance
    for t, (img_rows, txt_rows) in zip((bufs.k, bufs.v), mine):
        assert torch.equal(t[bufs.img_kv_rows(rank)], img_rows)
        d = (t[bufs.txt_kv_rows(rank)].float() - txt_rows.float()).abs().max().item()
        assert d <= 1e-2 * txt_rows.float().abs().max().item(), d
    assert torch.isfinite(a.float()).all() and torch.isfinite(b.float()).all()
    for got, want in ((a, s["out_img"][b0:b1]), (b, s["out_txt"][t0:t1])):
        d = (got.float() - want.float()).abs().max().item()
        scale = want.float().abs().max().item()
        assert d <= 1e-2 * scale, f"rank {rank}/{world} differs from the single-GPU block by {d} (max |ref| {scale})"


def test_text_stream_same_bits(single, dev, monkeypatch):
    """The text tokens' branches on their own stream (``block_forward(..., text_stream=...)``,
    what the bench does from 4 ranks on) give the same bits as on the current stream, at
    the 8-rank shard shapes."""
    from joyomni_ops import chain

    s = single
    world, rank = 8, 3
    monkeypatch.setattr(chain, "gather_chunk_kv", lambda bufs, rank, group: None)
    b0, b1 = chain.shard_range(IMG, world, rank)
    t0, t1 = chain.shard_range(TXT, world, rank)
    bufs = chain.KVBuffers(CACHE, IMG, TXT, HEADS, HD, world, dev)
    bufs.k.copy_(s["k"][:bufs.k.shape[0]])
    bufs.v.copy_(s["v"][:bufs.v.shape[0]])
    outs = []
    for ts in (None, torch.cuda.Stream()):
        a, b = chain.block_forward(s["img"][b0:b1], s["txt"][t0:t1], s["vec"], s["cos"][b0:b1], s["sin"][b0:b1],
                                   s["w"], bufs, group=object(), rank=rank, side_stream=torch.cuda.Stream(),
                                   text_stream=ts)
        torch.cuda.synchronize()
        outs.append((a.clone(), b.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
