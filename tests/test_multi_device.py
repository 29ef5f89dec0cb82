"""One process driving two GPUs: every kernel family launches on both devices (the
per-device shared-memory reservations and device tables), with results equal to the
same call on device 0.  Skipped with fewer than two visible GPUs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ops_on_two_devices_in_one_process(jo):
    from joyomni_ops import rope

    g = torch.Generator().manual_seed(3)
    x = torch.randn(300, 3072, generator=g).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(3072, generator=g)).to(torch.bfloat16)
    qkv = torch.randn(64, 3 * 4 * 128, generator=g).to(torch.bfloat16)
    qw = torch.ones(128, dtype=torch.bfloat16)
    cos, sin = rope.video_chunk_tables(1, 8, 8, 0)
    aq = torch.randn(300, 512, generator=g).to(torch.float8_e4m3fn)
    bq = torch.randn(256, 512, generator=g).to(torch.float8_e4m3fn).t()
    sa, sb = torch.rand(300, 1) + 0.5, torch.rand(1, 256) + 0.5
    outs = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            y = jo.rmsnorm(x.to(dev), w.to(dev), 1e-6)
            q, k, v = jo.qkv_norm_rope_pack(qkv.to(dev), 4, qw.to(dev), qw.to(dev), cos.to(dev), sin.to(dev), 1e-6,
                                            True)
            m = jo.fp8_scaled_mm(aq.to(dev), bq.to(dev), sa.to(dev), sb.to(dev), torch.bfloat16, None)
            torch.cuda.synchronize(dev)
            outs.append([t.cpu() for t in (y, q, k, v, m)])
    for a, b in zip(*outs):
        assert torch.equal(a, b)
