"""One MMDoubleStreamBlock forward for one streaming chunk, on the B200 ops.

The op chain of deploy/xvideo/models/dit/dit.py:360-558 (FP8 path,
``JOYOMNI_FP8_IMG/TXT``), with the reference's unfused steps replaced by the
fused sm_100a ops of this package:

    img/txt: LN1 + modulate + FP8 quant          norm_scale_shift_quant_fp8      (dit.py:402-408)
             QKV FP8 GEMM (+bias)                fp8_scaled_mm                   (dit.py:408, fp8_linear.py:114-141)
             q/k RMSNorm + 3D RoPE + pack        qkv_norm_rope_pack_into         (dit.py:409-429, 489-496)
               (text rows: RMSNorm only)           -> persistent Q / KV buffers (no concatenation copy)
    joint attention over [cache | img | txt]     torch SDPA (library, as FA4 in the reference, dit.py:498)
    img/txt: attn quant + out-proj GEMM          sgl_per_token_quant_fp8, fp8_scaled_mm
             gated residual + LN2 + mod + quant  gated_residual_norm_scale_shift_quant_fp8 (dit.py:525-535)
             MLP up GEMM, GELU-tanh + quant      fp8_scaled_mm, gelu_quant_fp8   (dit.py:508-513)
             MLP down GEMM + gated residual      fp8_scaled_mm_gated_residual    (dit.py:536-538)

Sequence parallel: the video tokens of the chunk are sharded over the ranks of
``group``; each rank writes its K/V rows into its slice of the persistent KV
buffer and an in-place NCCL ``all_gather_into_tensor`` (on a side stream,
overlapped with the text stream) completes the current chunk's K/V before
attention.  The text stream (512 tokens) is replicated.  The prior-chunk cache
rows of the KV buffer are assumed replicated (gathered once when stored).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

import joyomni_ops as jo

BF16 = torch.bfloat16
FP8 = torch.float8_e4m3fn
NUM_MOD = 6  # dit.py:37 NUM_MODULATION_CHUNKS


@dataclass
class Fp8Weight:
    """A Linear layer in the reference FP8 layout (fp8_linear.py:77-85)."""

    wq: torch.Tensor     # e4m3 [K, N] column-major (= [N, K] row-major, transposed view)
    ws: torch.Tensor     # fp32 [1, N] per-output-channel scale
    bias: Optional[torch.Tensor]  # bf16 [N]

    def __call__(self, xq: torch.Tensor, xs: torch.Tensor) -> torch.Tensor:
        return jo.fp8_scaled_mm(xq, self.wq, xs, self.ws, BF16, self.bias)


def quantize_linear(w: torch.Tensor, bias: Optional[torch.Tensor]) -> Fp8Weight:
    """Per-output-channel FP8 quantisation of a Linear weight [N, K] (fp8_linear.py:77-85)
    with the per-token quant op applied to the weight rows."""
    n, k = w.shape
    q = torch.empty(n, k, dtype=FP8, device=w.device)
    s = torch.empty(n, 1, dtype=torch.float32, device=w.device)
    jo.sgl_per_token_quant_fp8(w.contiguous(), q, s)
    return Fp8Weight(q.t(), s.reshape(1, n), None if bias is None else bias.to(BF16).contiguous())


@dataclass
class StreamWeights:
    """Weights of one stream (img or txt) of a double-stream block (dit.py:316-357)."""

    mod_table: torch.Tensor  # bf16 [6, D]   (ModulateWan.modulate_table, dit.py:103-116)
    qkv: Fp8Weight
    q_norm: torch.Tensor     # bf16 [head_dim]
    k_norm: torch.Tensor
    proj: Fp8Weight
    up: Fp8Weight
    down: Fp8Weight


def random_stream_weights(hidden: int, ffn: int, head_dim: int, device, gen: torch.Generator,
                          std: float = 0.02) -> StreamWeights:
    """Random-init weights of one stream: Linear weights and biases ~N(0, std), RMSNorm
    weights ~N(1, std), modulation table ~N(0, 1)/sqrt(D) (dit.py:107-112)."""
    def lin(n, k):
        w = (std * torch.randn(n, k, generator=gen)).to(BF16).to(device)
        b = (std * torch.randn(n, generator=gen)).to(BF16).to(device)
        return quantize_linear(w, b)

    table = (torch.randn(NUM_MOD, hidden, generator=gen) / math.sqrt(hidden)).to(BF16).to(device)
    qn = (1 + std * torch.randn(head_dim, generator=gen)).to(BF16).to(device)
    kn = (1 + std * torch.randn(head_dim, generator=gen)).to(BF16).to(device)
    return StreamWeights(table, lin(3 * hidden, hidden), qn, kn, lin(hidden, hidden), lin(ffn, hidden),
                         lin(hidden, ffn))


@dataclass
class BlockWeights:
    img: StreamWeights
    txt: StreamWeights
    heads: int
    head_dim: int


def random_block_weights(hidden=3072, heads=24, ffn=12288, device="cuda", seed=0) -> BlockWeights:
    g = torch.Generator().manual_seed(seed)
    hd = hidden // heads
    return BlockWeights(random_stream_weights(hidden, ffn, hd, device, g),
                        random_stream_weights(hidden, ffn, hd, device, g), heads, hd)


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[begin, end) of rank's share of n tokens (equal shares: the K/V all-gather
    concatenates equal slices, so n must divide evenly)."""
    if n % world:
        raise ValueError(f"{n} tokens do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


class KVBuffers:
    """Persistent joint-attention buffers (token-major [tokens, heads, head_dim]).

    KV rows: [ cache (prior chunks, replicated) | current chunk video tokens (all ranks) | text ].
    Q rows:  [ this rank's video tokens | text ].
    """

    def __init__(self, cache_len: int, img_len: int, txt_len: int, heads: int, head_dim: int, world: int,
                 device, dtype=BF16):
        self.cache_len, self.img_len, self.txt_len = cache_len, img_len, txt_len
        self.local = img_len // world
        s_kv = cache_len + img_len + txt_len
        self.k = torch.empty(s_kv, heads, head_dim, dtype=dtype, device=device)
        self.v = torch.empty(s_kv, heads, head_dim, dtype=dtype, device=device)
        self.q = torch.empty(self.local + txt_len, heads, head_dim, dtype=dtype, device=device)

    def img_kv_rows(self, rank: int):
        b = self.cache_len + rank * self.local
        return slice(b, b + self.local)

    def chunk_kv_rows(self):
        return slice(self.cache_len, self.cache_len + self.img_len)

    def txt_kv_rows(self):
        e = self.cache_len + self.img_len
        return slice(e, e + self.txt_len)


def gather_chunk_kv(bufs: KVBuffers, rank: int, group) -> None:
    """In-place all-gather of the current chunk's K/V rows over ``group``: every rank
    contributes its own slice, every rank ends with all video tokens of the chunk."""
    import torch.distributed as dist

    for t in (bufs.k, bufs.v):
        full = t[bufs.chunk_kv_rows()]
        dist.all_gather_into_tensor(full, t[bufs.img_kv_rows(rank)], group=group)


def modulation(table: torch.Tensor, vec: torch.Tensor):
    """ModulateWan (dit.py:103-116): table [6, D] + vec [6, D] -> six [1, D] rows."""
    m = (table + vec).contiguous()
    return [m[i:i + 1] for i in range(NUM_MOD)]


def _stream_qkv(x, w: StreamWeights, m, heads, cos, sin, q_out, k_out, v_out, trace=None, tag=""):
    shift1, scale1 = m[0], m[1]
    xq, xs = jo.norm_scale_shift_quant_fp8(x, None, None, scale1, shift1, "layer", 1e-6)
    qkv = w.qkv(xq, xs)
    jo.qkv_norm_rope_pack_into(qkv, heads, w.q_norm, w.k_norm, cos, sin, q_out, k_out, v_out, 1e-6)
    if trace is not None:
        trace.update({f"{tag}.xq": xq, f"{tag}.xs": xs, f"{tag}.qkv": qkv})


def _stream_out(x, attn, w: StreamWeights, m, trace=None, tag=""):
    gate1, shift2, scale2, gate2 = m[2], m[3], m[4], m[5]
    aq = torch.empty(attn.shape, dtype=FP8, device=attn.device)
    asc = torch.empty(attn.shape[0], 1, dtype=torch.float32, device=attn.device)
    jo.sgl_per_token_quant_fp8(attn, aq, asc)
    proj = w.proj(aq, asc)
    h, hq, hs = jo.gated_residual_norm_scale_shift_quant_fp8(x, proj, gate1, scale2, shift2, "layer", 1e-6)
    up = w.up(hq, hs)
    gq, gs = jo.gelu_quant_fp8(up)
    # down projection with the gated residual in the GEMM epilogue
    out = jo.fp8_scaled_mm_gated_residual(gq, w.down.wq, gs, w.down.ws, BF16, w.down.bias, h, gate2)
    if trace is not None:
        trace.update({f"{tag}.attn": attn, f"{tag}.aq": aq, f"{tag}.as": asc, f"{tag}.proj": proj, f"{tag}.h": h,
                      f"{tag}.hq": hq, f"{tag}.hs": hs, f"{tag}.up": up, f"{tag}.gq": gq, f"{tag}.gs": gs,
                      f"{tag}.out": out})
    return out


def _event(stream) -> torch.cuda.Event:
    e = torch.cuda.Event(enable_timing=True)
    e.record(stream)
    return e


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Non-causal joint attention on token-major [S, H, D] buffers -> [Sq, H*D]."""
    out = F.scaled_dot_product_attention(q.unsqueeze(0).transpose(1, 2), k.unsqueeze(0).transpose(1, 2),
                                         v.unsqueeze(0).transpose(1, 2), is_causal=False)
    return out.transpose(1, 2).reshape(q.shape[0], -1)


def block_forward(img: torch.Tensor, txt: torch.Tensor, vec: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  w: BlockWeights, bufs: KVBuffers, group=None, rank: int = 0,
                  side_stream: Optional[torch.cuda.Stream] = None, trace: Optional[dict] = None,
                  events: Optional[dict] = None):
    """One double-stream block for one chunk.

    img: bf16 [L_local, D] (this rank's video tokens), txt: bf16 [L_txt, D],
    vec: bf16 [6, D] (time_proj output, dit.py:1165-1166), cos/sin: bf16 [L_local, head_dim/2]
    for this rank's video tokens.  The cache rows of ``bufs.k/v`` hold the prior chunks.
    Returns (img_out [L_local, D], txt_out [L_txt, D]).  ``trace`` (a dict), if
    given, receives every intermediate tensor (for stage-by-stage parity tests).
    ``events`` (a dict), if given with a group, receives timing CUDA events:
    "gather_start" / "gather_end" around the K/V all-gather on the side stream and
    "overlap_end" on the compute stream once the work that overlaps it is queued,
    so the gather's exposed time is max(0, overlap_end -> gather_end).
    """
    H = w.heads
    L = img.shape[0]
    mi = modulation(w.img.mod_table, vec)
    mt = modulation(w.txt.mod_table, vec)
    _stream_qkv(img, w.img, mi, H, cos, sin, bufs.q[:L], bufs.k[bufs.img_kv_rows(rank)],
                bufs.v[bufs.img_kv_rows(rank)], trace, "img")
    gathered = None
    if group is not None:
        # complete the chunk's K/V on a side stream while the text stream runs
        side = side_stream or torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            if events is not None:
                events["gather_start"] = _event(side)
            gather_chunk_kv(bufs, rank, group)
            if events is not None:
                events["gather_end"] = _event(side)
        gathered = side
    _stream_qkv(txt, w.txt, mt, H, None, None, bufs.q[L:], bufs.k[bufs.txt_kv_rows()], bufs.v[bufs.txt_kv_rows()],
                trace, "txt")
    if gathered is not None:
        if events is not None:
            events["overlap_end"] = _event(torch.cuda.current_stream())
        torch.cuda.current_stream().wait_stream(gathered)
    attn = attention(bufs.q, bufs.k, bufs.v)
    if trace is not None:
        trace.update({"q": bufs.q, "k": bufs.k, "v": bufs.v, "mi": mi, "mt": mt})
    img_out = _stream_out(img, attn[:L], w.img, mi, trace, "img")
    txt_out = _stream_out(txt, attn[L:], w.txt, mt, trace, "txt")
    return img_out, txt_out
