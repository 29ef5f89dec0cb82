"""The allocation-free timestep MLP entry point (jo_timestep_mlp_noalloc) against the
scratch-taking one (jo_timestep_mlp), through the C ABI, on two calls in a row.

The file is named to be collected last: the static scratch array is shared by every
call on the device, so this must pass both alone in a fresh process and after the
other tests.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _weights(dev, freq, dim, proj, seed):
    g = torch.Generator().manual_seed(seed)
    w = lambda n, k: (torch.randn(n, k, generator=g) / k ** 0.5).to(BF).to(dev)
    b = lambda n: (0.1 * torch.randn(n, generator=g)).to(BF).to(dev)
    return w(dim, freq), b(dim), w(dim, dim), b(dim), w(proj, dim), b(proj)


def _call(name, dev, t, ws, scratch=None):
    from joyomni_ops import cabi

    w1, b1, w2, b2, w3, b3 = ws
    B, dim, freq, proj = t.shape[0], w1.shape[0], w1.shape[1], w3.shape[0]
    vec = torch.full((B, proj), float("nan"), dtype=BF, device=dev)
    args = [vec.data_ptr(), t.data_ptr(), B, w1.data_ptr(), b1.data_ptr(), freq, dim, w2.data_ptr(), b2.data_ptr(),
            w3.data_ptr(), b3.data_ptr(), proj]
    if scratch is not None:
        args += [scratch.data_ptr(), scratch.numel() * scratch.element_size()]
    cabi.call(name, *args, 10000.0, cabi.stream())
    return vec


@pytest.mark.parametrize("B,freq,dim,proj", [(1, 256, 3072, 18432), (16, 256, 4096, 1032)])
def test_noalloc_matches_scratch_entry(dev, B, freq, dim, proj):
    ws = _weights(dev, freq, dim, proj, B)
    scratch = torch.empty(2, B, dim, dtype=BF, device=dev)
    for call in range(2):  # two calls in a row share the static array
        t = (torch.rand(B, generator=torch.Generator().manual_seed(10 * B + call)) * 1000.0).to(dev)
        got = _call("jo_timestep_mlp_noalloc", dev, t, ws)
        want = _call("jo_timestep_mlp", dev, t, ws, scratch)
        torch.cuda.synchronize()
        assert not torch.isnan(got.float()).any(), f"call {call}: output not written"
        assert torch.equal(got, want), f"call {call}: differs from jo_timestep_mlp"


def test_noalloc_rejects_beyond_limit(dev):
    from joyomni_ops import cabi

    ws = _weights(dev, 256, 4096, 64, 3)
    t = torch.zeros(17, device=dev)
    vec = torch.empty(17, 64, dtype=BF, device=dev)
    w1, b1, w2, b2, w3, b3 = ws
    st = cabi.status_of("jo_timestep_mlp_noalloc", vec.data_ptr(), t.data_ptr(), 17, w1.data_ptr(), b1.data_ptr(),
                        256, 4096, w2.data_ptr(), b2.data_ptr(), w3.data_ptr(), b3.data_ptr(), 64, 10000.0,
                        cabi.stream())
    assert st == cabi.JO_ERR_SHAPE
    assert "static scratch limit" in cabi.last_error()
