"""GPU parity of the q/k norm + RoPE kernels and the q/k/v packs.

Tolerances: rotated q/k <= 1 bf16 ulp of the single-rounding fp32 oracle (ulp at
max(|ref|, 2^-10)); copied rows (v, cache, image rows of the pack) bit-exact.
"""
import pytest
import torch

from conftest import assert_guard_intact, assert_ulp_close, guarded_empty
from oracle import ops

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def rand(shape, seed, scale=1.0, mean=0.0, dt=BF):
    g = torch.Generator().manual_seed(seed)
    return (mean + scale * torch.randn(*shape, generator=g)).to(dt)


def chunk_tables(frames, h, w, t0, dims):
    from joyomni_ops import rope

    return rope.video_chunk_tables(frames, h, w, t0, dims=dims)


@pytest.mark.parametrize("head_major", [True, False])
def test_qkv_pack_config1(jo, dev, head_major):
    """Benchmark config 1: qkv [10800, 9216], 24 x 128 heads, 3x45x80 grid, t0 in [0, 64)."""
    L, H, D = 10800, 24, 128
    t0 = int(torch.randint(0, 64, (1,), generator=torch.Generator().manual_seed(7)).item())
    qkv = rand((L, 3 * H * D), 1)
    qw, kw = rand((D,), 2, 0.02, 1.0), rand((D,), 3, 0.02, 1.0)
    cos, sin = chunk_tables(3, 45, 80, t0, (44, 42, 42))
    q, k, v = jo.qkv_norm_rope_pack(qkv.to(dev), H, qw.to(dev), kw.to(dev), cos.to(dev), sin.to(dev), 1e-6,
                                    head_major)
    rq, rk, rv = ops.qkv_norm_rope_pack(qkv, H, qw, kw, cos, sin, 1e-6, head_major)
    assert torch.equal(v.cpu(), rv), "v must be a bit-exact copy"
    fq = assert_ulp_close(q, rq, 1.0, what="q")
    fk = assert_ulp_close(k, rk, 1.0, what="k")
    assert fq > 0.99 and fk > 0.99


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("L,H", [(37, 3), (1, 1), (130, 5)])
def test_qkv_pack_shapes_with_pre(jo, dev, D, L, H):
    qkv = rand((L, 3 * H * D), 10 + D)
    qw, kw = rand((D,), 11, 0.02, 1.0), rand((D,), 12, 0.02, 1.0)
    g = torch.Generator().manual_seed(13)
    ang = torch.rand(L, D // 2, generator=g) * 6.28
    cos, sin = ang.cos().to(BF), ang.sin().to(BF)
    pre = torch.empty(H, L, D, dtype=BF, device=dev)
    q, k, v = jo.qkv_norm_rope_pack(qkv.to(dev), H, qw.to(dev), kw.to(dev), cos.to(dev), sin.to(dev), 1e-6, True,
                                    pre)
    rq, rk, rv, rpre = ops.qkv_norm_rope_pack(qkv, H, qw, kw, cos, sin, 1e-6, True, with_pre=True)
    assert torch.equal(v.cpu(), rv)
    assert_ulp_close(q, rq, 1.0, what="q")
    assert_ulp_close(k, rk, 1.0, what="k")
    assert_ulp_close(pre, rpre, 1.0, what="k_pre_rope")


def test_qkv_pack_cabi_guarded_strided(cabi, dev):
    # qkv rows with padding (row stride > 3*H*D), outputs inside canaries
    L, H, D = 300, 4, 128
    W = 3 * H * D
    qkvw = rand((L, W + 64), 20)
    qw, kw = rand((D,), 21, 0.02, 1.0), rand((D,), 22, 0.02, 1.0)
    cos, sin = chunk_tables(3, 10, 10, 5, (44, 42, 42))
    g = {n: t.to(dev) for n, t in dict(qkv=qkvw, qw=qw, kw=kw, cos=cos, sin=sin).items()}
    bufs = [guarded_empty(H * L * D, BF, dev) for _ in range(3)]
    cabi.call("jo_qkv_norm_rope_pack", bufs[0][1].data_ptr(), bufs[1][1].data_ptr(), bufs[2][1].data_ptr(), None,
              L * D, D, g["qkv"].data_ptr(), W + 64, L, H, D, g["qw"].data_ptr(), g["kw"].data_ptr(),
              g["cos"].data_ptr(), g["sin"].data_ptr(), 1e-6, cabi.stream())
    torch.cuda.synchronize()
    for b, _ in bufs:
        assert_guard_intact(b)
    rq, rk, rv = ops.qkv_norm_rope_pack(qkvw[:, :W].contiguous(), H, qw, kw, cos, sin, 1e-6, True)
    assert torch.equal(bufs[2][1].view(H, L, D).cpu(), rv)
    assert_ulp_close(bufs[0][1].view(H, L, D), rq, 1.0, what="q")
    assert_ulp_close(bufs[1][1].view(H, L, D), rk, 1.0, what="k")


def test_qk_norm_rope_reference_case(jo, dev):
    """joyomni_ops/tests/test_parity_light.py:70-110: B1, 128 tokens, 8 heads, D128, k_pre_rope."""
    B, L, H, D = 1, 128, 8, 128
    q, k = rand((B, L * H, D), 30), rand((B, L * H, D), 31)
    qw, kw = rand((D,), 32), rand((D,), 33)
    cos, sin = rand((L, D // 2), 34), rand((L, D // 2), 35)
    qj, kj = q.to(dev), k.to(dev)
    kpre = torch.empty_like(kj)
    jo.fused_qk_norm_rope_3d_paired(qj, kj, L, H, 1e-6, qw.to(dev), kw.to(dev), cos.to(dev), sin.to(dev), kpre)
    rq, rk, rpre = ops.qk_norm_rope_paired(q, k, L, H, 1e-6, qw, kw, cos, sin)
    assert_ulp_close(qj, rq, 1.0, what="q")
    assert_ulp_close(kj, rk, 1.0, what="k")
    assert_ulp_close(kpre, rpre, 1.0, what="k_pre")


@pytest.mark.parametrize("B,L,H,D", [(1, 1560, 32, 128), (2, 50, 3, 64), (1, 17, 2, 256), (3, 1, 1, 128)])
def test_qk_norm_rope_inplace(jo, dev, B, L, H, D):
    q, k = rand((B, L * H, D), 40), rand((B, L * H, D), 41)
    qw, kw = rand((D,), 42, 0.02, 1.0), rand((D,), 43, 0.02, 1.0)
    g = torch.Generator().manual_seed(44)
    ang = torch.rand(L, D // 2, generator=g) * 6.28
    cos, sin = ang.cos().to(BF), ang.sin().to(BF)
    qj, kj = q.to(dev), k.to(dev)
    jo.fused_qk_norm_rope_3d_paired(qj, kj, L, H, 1e-6, qw.to(dev), kw.to(dev), cos.to(dev), sin.to(dev))
    rq, rk, _ = ops.qk_norm_rope_paired(q, k, L, H, 1e-6, qw, kw, cos, sin)
    assert_ulp_close(qj, rq, 1.0, what="q")
    assert_ulp_close(kj, rk, 1.0, what="k")


def test_qk_norm_rope_rejects(jo, dev):
    q = torch.zeros(1, 8 * 2, 96, dtype=BF, device=dev)
    w = torch.ones(96, dtype=BF, device=dev)
    cs = torch.zeros(8, 48, dtype=BF, device=dev)
    with pytest.raises(RuntimeError, match="head_dim"):
        jo.fused_qk_norm_rope_3d_paired(q, q.clone(), 8, 2, 1e-6, w, w, cs, cs)
    q = torch.zeros(1, 8 * 2, 128, dtype=BF, device=dev)
    w = torch.ones(128, dtype=BF, device=dev)
    with pytest.raises(RuntimeError, match="seq_len"):
        jo.fused_qk_norm_rope_3d_paired(q, q.clone(), 7, 2, 1e-6, w, w, cs, cs)


def joint_case(img_len, txt_len, cache_len, heads, seed, odd_stride=False):
    extra = 1 if odd_stride else 0  # a row stride that is not a multiple of 8 elements
    ib = rand((1, img_len, 3 * heads * 128 + extra), seed)
    tb = rand((1, txt_len, 3 * heads * 128 + extra), seed + 1)
    iq, ik, iv = (ib[..., i * heads * 128:(i + 1) * heads * 128].unflatten(-1, (heads, 128)) for i in range(3))
    tq, tk, tv = (tb[..., i * heads * 128:(i + 1) * heads * 128].unflatten(-1, (heads, 128)) for i in range(3))
    ck = rand((1, cache_len, heads, 128), seed + 2) if cache_len else None
    cv = rand((1, cache_len, heads, 128), seed + 3) if cache_len else None
    qw, kw = rand((128,), seed + 4), rand((128,), seed + 5)
    return (ib, tb), (iq, ik, iv, tq, tk, tv, ck, cv, qw, kw)


@pytest.mark.parametrize("img_len,txt_len,cache_len,heads,odd", [
    (17, 11, 9, 4, False),      # the reference test's shape (test_parity_light.py:137)
    (17, 11, 0, 4, False),      # no cache
    (300, 64, 1200, 24, False),
    (33, 5, 7, 3, True),        # unaligned strides -> scalar path
])
def test_joint_qkv_pack(jo, dev, img_len, txt_len, cache_len, heads, odd):
    bases, args = joint_case(img_len, txt_len, cache_len, heads, 50, odd)
    gb = [b.to(dev) for b in bases]
    ga = [None if a is None else a.to(dev) for a in args]
    # rebuild the strided device views from the device bases (same strides as the host views)
    for j, (base, gbase) in enumerate(((bases[0], gb[0]), (bases[0], gb[0]), (bases[0], gb[0]),
                                       (bases[1], gb[1]), (bases[1], gb[1]), (bases[1], gb[1]))):
        ga[j] = gbase.as_strided(args[j].shape, args[j].stride(), args[j].storage_offset())
    oq, ok, ov = jo.fused_joint_qkv_pack(*ga[:8], ga[8], ga[9], 1e-6)
    rq, rk, rv = ops.joint_qkv_pack(*args, 1e-6)
    assert torch.equal(ov.cpu(), rv), "V must be bit-exact (test_parity_light.py:173)"
    n = img_len * 1
    assert torch.equal(oq.cpu()[:, :n], rq[:, :n])
    assert torch.equal(ok.cpu()[:, : cache_len + n], rk[:, : cache_len + n])
    # text rows: the model's double rounding (bf16(x*r), then bf16(. * w)) turns a
    # 1-ulp flip of the first rounding (r differs from torch's in the last fp32
    # bits) into |w| ulps of the output; w ~ N(0, 1) as in the reference test
    fq = assert_ulp_close(oq, rq, 4.0, what="q")
    fk = assert_ulp_close(ok, rk, 4.0, what="k")
    assert fq > 0.99 and fk > 0.99


@pytest.mark.parametrize("len0,len1,heads", [(13, 7, 4), (13, 0, 4), (4000, 1200, 24)])
def test_cached_kv_pack(jo, dev, len0, len1, heads):
    k0, v0 = rand((1, len0, heads, 128), 60), rand((1, len0, heads, 128), 61)
    k1 = rand((1, len1, heads, 128), 62) if len1 else None
    v1 = rand((1, len1, heads, 128), 63) if len1 else None
    g = torch.Generator().manual_seed(64)
    cp, sp = torch.randn(len0 + len1, 64, generator=g), torch.randn(len0 + len1, 64, generator=g)
    cos, sin = cp.repeat_interleave(2, -1).contiguous(), sp.repeat_interleave(2, -1).contiguous()
    d = lambda t: t.to(dev) if t is not None else None
    okk, ov = jo.fused_cached_kv_pack(d(k0), d(v0), d(k1), d(v1), d(cos), d(sin))
    rk, rv = ops.cached_kv_pack(k0, v0, k1, v1, cos, sin)
    assert torch.equal(ov.cpu(), rv)
    assert_ulp_close(okk, rk, 1.0, floor=2.0 ** -6, what="k")
