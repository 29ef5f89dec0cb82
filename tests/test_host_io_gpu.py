"""GPU checks of the pipelined host-buffer q/k/v pack (jo_qkv_norm_rope_pack_host).

Each token is packed by the same kernel whatever the chunking, so the host
outputs must equal the device op's outputs bit for bit, for every chunk size
(including a ragged last chunk), both output layouts and the text mode.
"""
import pytest
import torch

from oracle import ops

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def rand(shape, seed, scale=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return (mean + scale * torch.randn(*shape, generator=g)).to(BF)


def pinned_like(shape):
    return torch.empty(shape, dtype=BF).pin_memory()


@pytest.mark.parametrize("chunk", [1350, 1000, 10800, 20000])
def test_host_pack_config1_matches_device_op(jo, dev, chunk):
    L, H, D = 10800, 24, 128
    qkv = rand((L, 3 * H * D), 1)
    qw, kw = rand((D,), 2, 0.02, 1.0).to(dev), rand((D,), 3, 0.02, 1.0).to(dev)
    (_, _), (cos, sin) = ops.rope_video_tables(3, 45, 80, 17)
    cos, sin = cos.to(dev), sin.to(dev)
    q, k, v = jo.qkv_norm_rope_pack(qkv.to(dev), H, qw, kw, cos, sin, 1e-6, True)
    hq, hk, hv = (pinned_like((H, L, D)) for _ in range(3))
    jo.qkv_norm_rope_pack_host(qkv.pin_memory(), H, qw, kw, cos, sin, hq, hk, hv, 1e-6, True, chunk)
    torch.cuda.synchronize()
    for name, a, b in (("q", hq, q), ("k", hk, k), ("v", hv, v)):
        assert torch.equal(a, b.cpu()), name


def test_host_pack_token_major_text_rows(jo, dev):
    L, H, D = 777, 5, 64
    qkv = rand((L, 3 * H * D), 4)
    qw, kw = rand((D,), 5, 0.02, 1.0).to(dev), rand((D,), 6, 0.02, 1.0).to(dev)
    q, k, v = jo.qkv_norm_rope_pack(qkv.to(dev), H, qw, kw, None, None, 1e-6, False)
    hq, hk, hv = (pinned_like((L, H, D)) for _ in range(3))
    jo.qkv_norm_rope_pack_host(qkv.pin_memory(), H, qw, kw, None, None, hq, hk, hv, 1e-6, False, 100)
    torch.cuda.synchronize()
    for name, a, b in (("q", hq, q), ("k", hk, k), ("v", hv, v)):
        assert torch.equal(a, b.cpu()), name
    rq, rk, rv = ops.qkv_text_pack(qkv, H, qw.cpu(), kw.cpu(), 1e-6)
    assert torch.equal(hv, rv)


def test_host_pack_cabi_consecutive_calls(cabi, jo, dev):
    """Two calls in a row through the C ABI reuse the staging buffers; each is complete
    once the compute stream is synchronised."""
    L, H, D = 2000, 8, 128
    qw, kw = rand((D,), 7, 0.02, 1.0).to(dev), rand((D,), 8, 0.02, 1.0).to(dev)
    g = torch.Generator().manual_seed(9)
    ang = torch.rand(L, D // 2, generator=g) * 6.28
    cos, sin = ang.cos().to(BF).to(dev), ang.sin().to(BF).to(dev)
    dev_qkv = torch.empty(L, 3 * H * D, dtype=BF, device=dev)
    dq, dk, dv = (torch.empty(H, L, D, dtype=BF, device=dev) for _ in range(3))
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    for seed in (10, 11):
        qkv = rand((L, 3 * H * D), seed).pin_memory()
        hq, hk, hv = (pinned_like((H, L, D)) for _ in range(3))
        cabi.call("jo_qkv_norm_rope_pack_host", hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), L * D, D,
                  qkv.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dev_qkv.data_ptr(), L, H, D,
                  qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), 1e-6, 333, cabi.stream(),
                  s_in.cuda_stream, s_out.cuda_stream)
        torch.cuda.current_stream().synchronize()
        q, k, v = jo.qkv_norm_rope_pack(qkv.to(dev), H, qw, kw, cos, sin, 1e-6, True)
        for name, a, b in (("q", hq, q), ("k", hk, k), ("v", hv, v)):
            assert torch.equal(a, b.cpu()), (seed, name)


def test_host_pack_rejects_bad_layout_and_streams(cabi, dev):
    L, H, D = 16, 2, 128
    buf = torch.empty(3 * L * H * D, dtype=BF, device=dev)
    host = torch.empty(3 * L * H * D, dtype=BF).pin_memory()
    w = torch.ones(D, dtype=BF, device=dev)
    p, hp = buf.data_ptr(), host.data_ptr()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    # neither head-major nor token-major strides
    st = cabi.status_of("jo_qkv_norm_rope_pack_host", hp, hp, hp, 3 * D, D, hp, p, p, p, p, L, H, D, w.data_ptr(),
                        w.data_ptr(), None, None, 1e-6, 8, cabi.stream(), s_in.cuda_stream, s_out.cuda_stream)
    assert st == cabi.JO_ERR_SHAPE
    # missing copy streams
    st = cabi.status_of("jo_qkv_norm_rope_pack_host", hp, hp, hp, L * D, D, hp, p, p, p, p, L, H, D, w.data_ptr(),
                        w.data_ptr(), None, None, 1e-6, 8, cabi.stream(), None, None)
    assert st == cabi.JO_ERR_INVALID
