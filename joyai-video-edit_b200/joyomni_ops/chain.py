"""One MMDoubleStreamBlock forward for one streaming chunk, on the B200 ops.

The op chain of deploy/xvideo/models/dit/dit.py:360-558 (FP8 path,
``JOYOMNI_FP8_IMG/TXT``), with the reference's unfused steps replaced by the
fused sm_100a ops of this package:

    img/txt: LN1 + modulate + FP8 quant          norm_scale_shift_quant_fp8      (dit.py:402-408)
             QKV FP8 GEMM (+bias)                fp8_scaled_mm                   (dit.py:408, fp8_linear.py:114-141)
             q/k RMSNorm + 3D RoPE + pack        qkv_norm_rope_pack_into         (dit.py:409-429, 489-496)
               (text rows: RMSNorm only)           -> persistent Q / KV buffers (no concatenation copy)
    joint attention over [cache | img | txt]     cuDNN attention (library, as FA4 in the reference, dit.py:498);
                                                 split at the cache rows + attn_merge when sequence parallel
    img/txt: attn quant + out-proj GEMM          sgl_per_token_quant_fp8, fp8_scaled_mm
             gated residual + LN2 + mod + quant  gated_residual_norm_scale_shift_quant_fp8 (dit.py:525-535)
             MLP up GEMM + GELU-tanh + quant     fp8_scaled_mm_gelu_quant        (dit.py:508-513)
               (GELU and the row amax in the GEMM epilogue, one quantisation pass)
             MLP down GEMM + gated residual      fp8_scaled_mm_gated_residual    (dit.py:536-538)

Sequence parallel: the video and the text tokens of the chunk are both sharded
over the ranks of ``group`` (every op but attention is per token); each rank
writes its K/V rows, [its video | its text], as one block of the persistent KV
buffer and one in-place NCCL ``all_gather_into_tensor`` per tensor (on a side
stream) completes the chunk's K/V.  The gather overlaps the attention over the
cache rows, which every rank holds already: attention is split into the cache
rows and the gathered rows, and the two partial results are merged by their
log-sum-exps (``attn_merge``).  The cache rows are replicated when a chunk is
stored (``store_chunk_kv``: one gather of the stored chunk's pre-RoPE K and V)
and rotated into the buffer once per window (``rotate_cache``).

The modulation rows of every block come from one launch of the timestep MLP
(``timestep_mlp_modulate``: the ModulateWan add of dit.py:103-116 folded into
time_proj), or are formed here from the block's tables and ``vec``.
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

    KV rows: [ cache (prior chunks, replicated) | rank 0's block | rank 1's block | ... ],
             a rank's block = [ its video tokens of the chunk | its text tokens ].
    Q rows:  [ this rank's video tokens | this rank's text tokens ].

    Both token streams are sharded over the ranks and every rank's K/V rows are one
    contiguous block, so a single in-place all-gather completes the keys; the order of
    the keys does not matter to (non-causal) attention.  With one rank the rows are
    [ cache | video | text ].

    The cache rows are ``slots`` chunk-sized slots (attention does not depend on the
    order of its keys, so a new chunk takes the slot of the one it evicts).  For the
    store path the buffers also keep every cached chunk's pre-RoPE keys (``k_pre``,
    one more slot than the window: the chunk being stored goes to the spare one while
    the window still attends over the chunk it will evict) and a staging block for
    the stored chunk's values (``v_stage``); ``k_pre_of[i]`` is the ``k_pre`` slot of
    cache slot i.
    """

    def __init__(self, cache_len: int, img_len: int, txt_len: int, heads: int, head_dim: int, world: int,
                 device, dtype=BF16, store: bool = False, ipc: bool = False):
        self.cache_len, self.img_len, self.txt_len = cache_len, img_len, txt_len
        if img_len % world or txt_len % world:
            raise ValueError(f"{img_len} video / {txt_len} text tokens do not split evenly over {world} ranks")
        self.local = img_len // world
        self.txt_local = txt_len // world
        self.block = self.local + self.txt_local
        s_kv = cache_len + img_len + txt_len
        self.row_bytes = heads * head_dim * torch.tensor([], dtype=dtype).element_size()
        self._ipc = []
        if ipc:  # whole allocations that the other ranks can map (the copy-engine gather)
            self._ipc = [IpcAlloc(s_kv * self.row_bytes, device) for _ in range(2)]
            self.k, self.v = (a.tensor((s_kv, heads, head_dim), dtype) for a in self._ipc)
        else:
            self.k = torch.empty(s_kv, heads, head_dim, dtype=dtype, device=device)
            self.v = torch.empty(s_kv, heads, head_dim, dtype=dtype, device=device)
        self.q = torch.empty(self.block, heads, head_dim, dtype=dtype, device=device)
        self.slots = cache_len // img_len
        self.k_pre = self.v_stage = None
        if store:
            if cache_len % img_len:
                raise ValueError(f"a storing cache ({cache_len} rows) must hold whole chunks of {img_len} rows")
            self.k_pre = torch.empty(self.slots + 1, img_len, heads, head_dim, dtype=dtype, device=device)
            self.v_stage = torch.empty(img_len, heads, head_dim, dtype=dtype, device=device)
        self.k_pre_of = list(range(self.slots))
        self.spare = self.slots

    def close(self) -> None:
        """Frees IPC-allocated K/V buffers (after every peer has unmapped them:
        ``PeerGather.close`` first)."""
        self.k = self.v = None
        for a in self._ipc:
            a.free()
        self._ipc = []

    def cache_slot_rows(self, slot: int):
        return slice(slot * self.img_len, (slot + 1) * self.img_len)

    def block_rows(self, rank: int):
        b = self.cache_len + rank * self.block
        return slice(b, b + self.block)

    def img_kv_rows(self, rank: int):
        b = self.cache_len + rank * self.block
        return slice(b, b + self.local)

    def txt_kv_rows(self, rank: int):
        b = self.cache_len + rank * self.block + self.local
        return slice(b, b + self.txt_local)

    def gathered_rows(self):
        """Every rank's block (all rows after the cache)."""
        return slice(self.cache_len, self.cache_len + self.img_len + self.txt_len)


class IpcAlloc:
    """A whole device allocation of ``nbytes`` (``jo_ipc_alloc``, zeroed) on ``device``, which
    other processes on the node can map (``jo_ipc_handle`` / ``jo_ipc_open``).  ``tensor``
    views it; ``free`` releases it (no view may be used afterwards)."""

    def __init__(self, nbytes: int, device):
        import ctypes as C

        from joyomni_ops import cabi

        self.device = torch.device(device)
        with torch.cuda.device(self.device):
            p = C.c_void_p()
            cabi.call("jo_ipc_alloc", nbytes, C.byref(p))
        self.ptr, self.nbytes = p.value, nbytes
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (self.ptr, False),
                                         "version": 3, "strides": None, "stream": None}

    def tensor(self, shape, dtype) -> torch.Tensor:
        return torch.as_tensor(self, device=self.device).view(dtype).view(shape)

    def handle(self) -> bytes:
        import ctypes as C

        from joyomni_ops import cabi

        h = C.create_string_buffer(cabi.JO_IPC_HANDLE_BYTES)
        cabi.call("jo_ipc_handle", self.ptr, h)
        return h.raw

    def free(self) -> None:
        from joyomni_ops import cabi

        if self.ptr is not None:
            with torch.cuda.device(self.device):
                cabi.call("jo_ipc_free", self.ptr)
            self.ptr = None


class PeerGather:
    """Copy-engine all-gather of the chunk's K/V blocks over the ranks of ``group`` (one
    process per GPU of one node), in place of the NCCL ``all_gather_into_tensor`` of
    ``gather_chunk_kv``: every rank maps the other ranks' K/V buffers (``KVBuffers(...,
    ipc=True)``, CUDA IPC) and pulls each peer's block with one copy-engine transfer per
    (peer, tensor), on a stream of its own, so the gather takes no SMs from the attention
    over the cache rows that it overlaps.

    Ordering (two 8-byte flag words per peer in each rank's IPC-mapped flag array):
    ``gather`` (step e) stores e into ready[r] on every peer once this rank's block is
    written, waits until every peer's ready word on this rank reaches e, pulls, then stores
    e into done[r] on every peer; ``before_write`` (on the compute stream, before the rank's
    pack overwrites its block for step e + 1) waits until every peer's done word reaches e.
    Every wait is a bounded kernel (2 s, then the device fault counter is raised)."""

    def __init__(self, bufs: KVBuffers, rank: int, world: int, group):
        import ctypes as C

        import torch.distributed as dist

        from joyomni_ops import cabi

        if not bufs._ipc:
            raise ValueError("PeerGather needs KVBuffers(..., ipc=True)")
        self.bufs, self.rank, self.world, self.group = bufs, rank, world, group
        dev = bufs.k.device
        self._flags = IpcAlloc(max(256, 16 * world), dev)  # ready[world] | done[world], zeroed
        mine = [bufs._ipc[0].handle(), bufs._ipc[1].handle(), self._flags.handle()]
        every = [None] * world
        dist.all_gather_object(every, mine, group=group)
        self._mapped = []
        self.peer_k, self.peer_v = {}, {}
        self._ready_tab = (C.c_void_p * world)()
        self._done_tab = (C.c_void_p * world)()
        err = None
        with torch.cuda.device(dev):
            try:
                for q in range(world):
                    if q == rank:
                        continue
                    ptrs = []
                    for h in every[q]:
                        p = C.c_void_p()
                        cabi.call("jo_ipc_open", C.create_string_buffer(h, len(h)), C.byref(p))
                        ptrs.append(p.value)
                        self._mapped.append(p.value)
                    self.peer_k[q], self.peer_v[q] = ptrs[0], ptrs[1]
                    self._ready_tab[q] = ptrs[2] + 8 * rank
                    self._done_tab[q] = ptrs[2] + 8 * (world + rank)
            except RuntimeError as e:
                err = e
            # every rank learns whether every rank mapped its peers, so all of them either use
            # the gather or raise (and can fall back to the collective together)
            ok = torch.tensor([0.0 if err else 1.0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if ok.item() < 1.0:
                for p in self._mapped:
                    cabi.status_of("jo_ipc_close", p)
                self._mapped = []
                dist.barrier(group=group)
                self._flags.free()
                raise RuntimeError(f"copy-engine K/V gather unavailable (rank {rank}: {err or 'a peer failed'})")
        self._local_ready = self._flags.ptr
        self._local_done = self._flags.ptr + 8 * world
        self.step = 0
        self._streams = {(q, t): torch.cuda.Stream(dev) for q in self.peer_k for t in range(2)}
        dist.barrier(group=group)

    def before_write(self, stream: torch.cuda.Stream) -> None:
        """On ``stream``, before this rank's pack rewrites its block: every peer has pulled
        the previous step's block."""
        from joyomni_ops import cabi

        if self.step > 0:
            cabi.call("jo_peer_wait", self._local_done, self.world, self.rank, self.step, stream.cuda_stream)

    def gather(self, stream: torch.cuda.Stream) -> None:
        """On ``stream`` (after this rank's block is written): publish the block, wait for
        every peer's, pull them all; ``stream`` then orders after every pull."""
        from joyomni_ops import cabi

        self.step += 1
        s = stream.cuda_stream
        cabi.call("jo_peer_signal", self._ready_tab, self.world, self.step, s)
        cabi.call("jo_peer_wait", self._local_ready, self.world, self.rank, self.step, s)
        ready = torch.cuda.Event()
        ready.record(stream)
        b = self.bufs
        n = b.block * b.row_bytes
        for (q, t), cs in self._streams.items():
            cs.wait_event(ready)
            off = b.block_rows(q).start * b.row_bytes
            dst, src = (b.k, self.peer_k[q]) if t == 0 else (b.v, self.peer_v[q])
            cabi.call("jo_peer_copy", dst.data_ptr() + off, src + off, n, cs.cuda_stream)
            stream.wait_stream(cs)
        cabi.call("jo_peer_signal", self._done_tab, self.world, self.step, s)

    def close(self) -> None:
        """Unmaps the peers' buffers and frees the flag array; every rank calls it (it
        ends with a barrier, after which ``bufs.close()`` may free the K/V buffers)."""
        import torch.distributed as dist

        from joyomni_ops import cabi

        torch.cuda.synchronize()
        with torch.cuda.device(self._flags.device):
            for p in self._mapped:
                cabi.call("jo_ipc_close", p)
        self._mapped = []
        dist.barrier(group=self.group)
        self._flags.free()


def store_chunk_kv(bufs: KVBuffers, rank: int, group) -> None:
    """After a store forward (``block_forward(..., store=True)``): the chunk's pre-RoPE keys
    (in the spare ``k_pre`` slot, each rank's own rows) and values (each rank's chunk rows
    of ``v``) are gathered once, so every rank holds the whole stored chunk
    (dit.py:445-459: the K/V handed to the cache writer; pre-RoPE keys, dit.py:413-429)."""
    k_spare = bufs.k_pre[bufs.spare]
    mine = slice(rank * bufs.local, (rank + 1) * bufs.local)
    if group is None:
        bufs.v_stage.copy_(bufs.v[bufs.img_kv_rows(rank)])
        return
    import torch.distributed as dist

    dist.all_gather_into_tensor(k_spare, k_spare[mine], group=group)
    dist.all_gather_into_tensor(bufs.v_stage, bufs.v[bufs.img_kv_rows(rank)], group=group)


def advance_window(bufs: KVBuffers, evict_slot: int) -> None:
    """The stored chunk replaces cache slot ``evict_slot``: its values move into the slot's
    rows of ``v``, its pre-RoPE keys' slot is swapped in (the evicted chunk's becomes the
    spare).  Call ``rotate_cache`` afterwards: the window's temporal positions changed."""
    bufs.v[bufs.cache_slot_rows(evict_slot)].copy_(bufs.v_stage)
    bufs.k_pre_of[evict_slot], bufs.spare = bufs.spare, bufs.k_pre_of[evict_slot]


def rotate_cache(bufs: KVBuffers, cos: torch.Tensor, sin: torch.Tensor) -> None:
    """RoPE of every cached chunk's pre-RoPE keys into the cache rows of ``k`` with the
    window-relative fp32 full-width tables cos/sin [cache_len, head_dim] (row r for cache
    row r): the key half of fused_cached_kv_pack (fused_joint_qkv_pack.cu:166-220;
    dit.py:216-271), done once per window instead of once per block call."""
    for i in range(bufs.slots):
        rows = bufs.cache_slot_rows(i)
        jo.cached_k_rotate_into(bufs.k_pre[bufs.k_pre_of[i]], cos[rows], sin[rows], bufs.k[rows])


def gather_chunk_kv(bufs: KVBuffers, rank: int, group) -> None:
    """In-place all-gather of the current chunk's K/V rows over ``group``: every rank
    contributes its block (its video and text tokens), every rank ends with all of them."""
    import torch.distributed as dist

    for t in (bufs.k, bufs.v):
        dist.all_gather_into_tensor(t[bufs.gathered_rows()], t[bufs.block_rows(rank)], group=group)


def modulation(table: torch.Tensor, vec: torch.Tensor):
    """ModulateWan (dit.py:103-116): table [6, D] + vec [6, D] -> six [1, D] rows."""
    return mod_rows((table + vec).contiguous())


def mod_rows(m: torch.Tensor):
    """Six [1, D] modulation rows (shift1, scale1, gate1, shift2, scale2, gate2) of m [6, D]
    (or [6 * D]), e.g. one block's rows of timestep_mlp_modulate's output."""
    m = m.reshape(NUM_MOD, -1)
    return [m[i:i + 1] for i in range(NUM_MOD)]


def _stream_qkv(x, w: StreamWeights, m, heads, cos, sin, q_out, k_out, v_out, trace=None, tag="", k_pre_out=None):
    shift1, scale1 = m[0], m[1]
    xq, xs = jo.norm_scale_shift_quant_fp8(x, None, None, scale1, shift1, "layer", 1e-6)
    qkv = w.qkv(xq, xs)
    jo.qkv_norm_rope_pack_into(qkv, heads, w.q_norm, w.k_norm, cos, sin, q_out, k_out, v_out, 1e-6, k_pre_out)
    if trace is not None:
        trace.update({f"{tag}.xq": xq, f"{tag}.xs": xs, f"{tag}.qkv": qkv})


def _stream_out(x, attn, w: StreamWeights, m, trace=None, tag=""):
    gate1, shift2, scale2, gate2 = m[2], m[3], m[4], m[5]
    aq = torch.empty(attn.shape, dtype=FP8, device=attn.device)
    asc = torch.empty(attn.shape[0], 1, dtype=torch.float32, device=attn.device)
    jo.sgl_per_token_quant_fp8(attn, aq, asc)
    proj = w.proj(aq, asc)
    h, hq, hs = jo.gated_residual_norm_scale_shift_quant_fp8(x, proj, gate1, scale2, shift2, "layer", 1e-6)
    gq, gs = jo.fp8_scaled_mm_gelu_quant(hq, w.up.wq, hs, w.up.ws, BF16, w.up.bias)
    # down projection with the gated residual in the GEMM epilogue
    out = jo.fp8_scaled_mm_gated_residual(gq, w.down.wq, gs, w.down.ws, BF16, w.down.bias, h, gate2)
    if trace is not None:
        trace.update({f"{tag}.attn": attn, f"{tag}.aq": aq, f"{tag}.as": asc, f"{tag}.proj": proj, f"{tag}.h": h,
                      f"{tag}.hq": hq, f"{tag}.hs": hs, f"{tag}.gq": gq, f"{tag}.gs": gs,
                      f"{tag}.out": out})
    return out


def _event(stream) -> torch.cuda.Event:
    e = torch.cuda.Event(enable_timing=True)
    e.record(stream)
    return e


def attention_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """Non-causal attention of token-major [S, H, D] buffers with its log-sum-exp: the
    library (cuDNN) kernel, as SDPA picks it for these shapes.  Returns (o [1, H, Sq, D],
    lse fp32 [1, H, Sq])."""
    qh, kh, vh = (t.unsqueeze(0).transpose(1, 2) for t in (q, k, v))
    r = torch.ops.aten._scaled_dot_product_cudnn_attention(qh, kh, vh, None, True, 0.0, False, False)
    lse = r[1]
    if lse.dim() == 4:  # [1, H, Sq, 1] on some library versions
        lse = lse.squeeze(-1)
    return r[0], lse


def attention_split(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, split: int, before_rest=None):
    """Attention of q over all rows of k/v as two parts merged by log-sum-exp: rows [0, split)
    first, then ``before_rest()`` (e.g. a wait for the rest of the rows), then rows [split, S).
    Returns [Sq, H*D] like ``attention``."""
    oa, la = attention_lse(q, k[:split], v[:split])
    if before_rest is not None:
        before_rest()
    ob, lb = attention_lse(q, k[split:], v[split:])
    return jo.attn_merge(oa, la, ob, lb).reshape(q.shape[0], -1)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Non-causal joint attention on token-major [S, H, D] buffers -> [Sq, H*D]."""
    out = F.scaled_dot_product_attention(q.unsqueeze(0).transpose(1, 2), k.unsqueeze(0).transpose(1, 2),
                                         v.unsqueeze(0).transpose(1, 2), is_causal=False)
    return out.transpose(1, 2).reshape(q.shape[0], -1)


def block_forward(img: torch.Tensor, txt: torch.Tensor, vec: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  w: BlockWeights, bufs: KVBuffers, group=None, rank: int = 0,
                  side_stream: Optional[torch.cuda.Stream] = None, trace: Optional[dict] = None,
                  events: Optional[dict] = None, mods: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                  store: bool = False, peers: Optional[PeerGather] = None,
                  text_stream: Optional[torch.cuda.Stream] = None):
    """One double-stream block for one chunk.

    img: bf16 [L_local, D] (this rank's video tokens), txt: bf16 [T_local, D] (this rank's
    text tokens), vec: bf16 [6, D] (time_proj output, dit.py:1165-1166), cos/sin: bf16
    [L_local, head_dim/2] for this rank's video tokens.  The cache rows of ``bufs.k/v``
    hold the prior chunks.  Returns (img_out [L_local, D], txt_out [T_local, D]).  ``trace`` (a dict), if
    given, receives every intermediate tensor (for stage-by-stage parity tests).
    ``events`` (a dict), if given with a group, receives timing CUDA events:
    "gather_start" / "gather_end" around the K/V all-gather on the side stream and
    "overlap_end" on the compute stream once the work that overlaps it is queued,
    so the gather's exposed time is max(0, overlap_end -> gather_end).
    ``mods`` (img rows, txt rows), each [6, D], replaces the ModulateWan add of ``vec``
    and the block's tables (rows of ``timestep_mlp_modulate``'s output).
    ``store``: a store forward (buffers made with ``store=True``): the image pack also
    writes this rank's pre-RoPE keys into the spare ``k_pre`` slot; ``store_chunk_kv``
    then replicates the chunk.
    ``peers`` (with ``group``): gather the chunk's K/V with the copy engines
    (``PeerGather``) instead of the NCCL all-gather.
    ``text_stream``: run the text tokens' branches (LN + QKV + pack before attention, the
    output projection and MLP after it) on this stream, beside the video tokens' branches on
    the current stream: sharded over 8 ranks the text GEMMs fill 12-48 tiles only, so alone
    they leave most SMs idle (with 128 or more text rows per GPU the overlap was slower);
    the current stream waits for the text stream before attention and before returning.
    """
    H = w.heads
    L = img.shape[0]
    if mods is not None:
        mi, mt = mod_rows(mods[0]), mod_rows(mods[1])
    else:
        mi = modulation(w.img.mod_table, vec)
        mt = modulation(w.txt.mod_table, vec)
    k_pre = bufs.k_pre[bufs.spare][rank * bufs.local:(rank + 1) * bufs.local] if store else None
    if group is not None and peers is not None:
        peers.before_write(torch.cuda.current_stream())
    cur = torch.cuda.current_stream()
    if text_stream is not None:
        text_stream.wait_stream(cur)
        with torch.cuda.stream(text_stream):
            _stream_qkv(txt, w.txt, mt, H, None, None, bufs.q[L:], bufs.k[bufs.txt_kv_rows(rank)],
                        bufs.v[bufs.txt_kv_rows(rank)], trace, "txt")
    _stream_qkv(img, w.img, mi, H, cos, sin, bufs.q[:L], bufs.k[bufs.img_kv_rows(rank)],
                bufs.v[bufs.img_kv_rows(rank)], trace, "img", k_pre)
    if text_stream is not None:
        cur.wait_stream(text_stream)
    else:
        _stream_qkv(txt, w.txt, mt, H, None, None, bufs.q[L:], bufs.k[bufs.txt_kv_rows(rank)],
                    bufs.v[bufs.txt_kv_rows(rank)], trace, "txt")
    gathered = None
    if group is not None:
        # complete the chunk's K/V (every rank's block) on a side stream; the attention
        # over the cache rows runs meanwhile
        side = side_stream or torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            if events is not None:
                events["gather_start"] = _event(side)
            if peers is not None:
                peers.gather(side)
            else:
                gather_chunk_kv(bufs, rank, group)
            if events is not None:
                events["gather_end"] = _event(side)
        gathered = side

    def join_gather():
        if events is not None:
            events["overlap_end"] = _event(torch.cuda.current_stream())
        torch.cuda.current_stream().wait_stream(gathered)

    if gathered is not None and bufs.cache_len > 0:
        # the cache rows are here already: attend over them while the chunk's K/V arrive
        attn = attention_split(bufs.q, bufs.k, bufs.v, bufs.cache_len, join_gather)
    else:
        if gathered is not None:
            join_gather()
        attn = attention(bufs.q, bufs.k, bufs.v)
    if trace is not None:
        trace.update({"q": bufs.q, "k": bufs.k, "v": bufs.v, "mi": mi, "mt": mt})
    if text_stream is not None:
        text_stream.wait_stream(cur)
        with torch.cuda.stream(text_stream):
            txt_out = _stream_out(txt, attn[L:], w.txt, mt, trace, "txt")
        img_out = _stream_out(img, attn[:L], w.img, mi, trace, "img")
        cur.wait_stream(text_stream)
        txt_out.record_stream(cur)  # made on the text stream, used and freed on the caller's
    else:
        img_out = _stream_out(img, attn[:L], w.img, mi, trace, "img")
        txt_out = _stream_out(txt, attn[L:], w.txt, mt, trace, "txt")
    return img_out, txt_out
