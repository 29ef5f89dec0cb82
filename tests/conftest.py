"""Shared pytest setup.

* ``gpu`` marker: tests that launch kernels on a B200 (``pytest -m gpu``); they
  are skipped where no CUDA device is visible.
* The repository root (for ``oracle``) and ``joyai-video-edit_b200`` (for the
  ``joyomni_ops`` package) are put on ``sys.path``.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "joyai-video-edit_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden" / "reference_golden.pt"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN, weights_only=False)["cases"]


@pytest.fixture(scope="session")
def jo():
    import joyomni_ops

    return joyomni_ops


@pytest.fixture(scope="session")
def cabi():
    from joyomni_ops import cabi as c

    c.lib()
    return c


@pytest.fixture(scope="session")
def dev():
    return torch.device("cuda", 0)


def assert_bf16_close(out: torch.Tensor, ref: torch.Tensor, max_ulp: float = 1.0, floor: float = 2.0 ** -10,
                      what: str = "") -> float:
    """|out - ref| <= max_ulp bf16 ulps of max(|ref|, floor), elementwise.

    ``floor`` bounds the ulp used near zero: where the fp32 result cancels to a
    tiny value, both sides carry ~2^-24 relative error of the cancelling terms,
    so "1 ulp of a tiny result" would test rounding noise, not the kernel.
    Returns the fraction of bit-exact elements.
    """
    from oracle.ops import bf16_ulp

    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert o.shape == r.shape, f"{what}: shape {tuple(o.shape)} vs {tuple(r.shape)}"
    assert torch.isfinite(o).all(), f"{what}: non-finite output"
    ulp = bf16_ulp(r.abs().clamp_min(floor))
    d = (o - r).abs() / ulp
    worst = d.max().item() if d.numel() else 0.0
    assert worst <= max_ulp, (f"{what}: max diff {worst:.3f} ulp (> {max_ulp}); "
                              f"{(d > max_ulp).sum().item()} of {d.numel()} elements")
    return (o == r).float().mean().item() if d.numel() else 1.0


MANTISSA_BITS = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}
MIN_ULP = {torch.bfloat16: 2.0 ** -133, torch.float16: 2.0 ** -24, torch.float32: 2.0 ** -149}


def assert_ulp_close(out: torch.Tensor, ref: torch.Tensor, max_ulp: float = 1.0, floor: float = 2.0 ** -10,
                     what: str = "", atol: torch.Tensor = None) -> float:
    """Like assert_bf16_close, in ulps of ``ref.dtype`` (bf16 / fp16 / fp32).

    ``atol`` (optional, elementwise) is added to the allowed difference; used
    where the reference formula itself carries a stated absolute error.
    """
    bits = MANTISSA_BITS[ref.dtype]
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert o.shape == r.shape, f"{what}: shape {tuple(o.shape)} vs {tuple(r.shape)}"
    if o.numel() == 0:
        return 1.0
    assert torch.isfinite(o).all(), f"{what}: non-finite output"
    mag = r.abs().clamp_min(floor)
    # ulp of the value, never below the dtype's subnormal spacing
    ulp = torch.pow(2.0, torch.floor(torch.log2(mag)) - bits).clamp_min(MIN_ULP[ref.dtype])
    allowed = max_ulp * ulp + (atol.float().cpu() if atol is not None else 0.0)
    bad = (o - r).abs() > allowed
    if bad.any():
        i = bad.nonzero()[0].tolist()
        raise AssertionError(f"{what}: {bad.sum().item()} of {o.numel()} elements off by more than {max_ulp} ulp; "
                             f"first at {i}: got {o[tuple(i)].item()} want {r[tuple(i)].item()}")
    return (o == r).float().mean().item()


GUARD = 4096  # elements of canary on each side of a guarded output


def guarded_empty(numel: int, dtype, device):
    """A buffer with GUARD canary elements on both sides; returns (buffer, middle view)."""
    buf = torch.empty(numel + 2 * GUARD, dtype=dtype, device=device)
    buf.view(torch.uint8).fill_(0xA5)
    return buf, buf[GUARD:GUARD + numel]


def assert_guard_intact(buf: torch.Tensor):
    raw = buf.view(torch.uint8)
    esz = buf.element_size()
    head = raw[: GUARD * esz]
    tail = raw[raw.numel() - GUARD * esz:]
    assert bool((head == 0xA5).all()) and bool((tail == 0xA5).all()), "write outside the output buffer"
