"""GPU parity of the per-block chain (benchmark config 4) and the fused ops it adds.

Stage by stage, each op of joyomni_ops.chain.block_forward is checked against the
oracle applied to the GPU's own inputs of that stage (the per-op tolerances of
the other test files); end to end, the block output is checked against the
oracle chain (oracle.ops.block_forward) with the north-star FP8 gate (relative
Frobenius error <= 2e-2): every FP8 requantisation can move an element by one
e4m3 step when its bf16 input differs by one ulp, so bit-level agreement is
only meaningful stage by stage.
"""
import pytest
import torch

from conftest import assert_ulp_close
from oracle import ops

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def rand(shape, seed, scale=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return (mean + scale * torch.randn(*shape, generator=g)).to(BF)


def rel_err(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def gemm_close(out, ref, what):
    o, r = out.float().cpu(), ref.float().cpu()
    rms = r.pow(2).mean().sqrt().item()
    ulp = torch.pow(2.0, torch.floor(torch.log2(r.abs().clamp_min(1e-30))) - 7)
    bad = (o - r).abs() > 2 * ulp + rms * 2.0 ** -12
    assert not bad.any(), f"{what}: {bad.sum().item()} elements off"


def quant_matches(q, s, y):
    """(q, s) == per_token_quant(y) bit-exactly."""
    rq, rs = ops.per_token_quant_fp8(y.cpu())
    return torch.equal(s.cpu().reshape(-1), rs.reshape(-1)) and torch.equal(q.cpu().view(torch.uint8),
                                                                             rq.view(torch.uint8))


# ------------------------------------------------------------------ new fused ops
@pytest.mark.parametrize("L,H", [(512, 24), (37, 3)])
def test_text_pack(jo, dev, L, H):
    qkv = rand((L, 3 * H * 128), 1)
    qw, kw = rand((128,), 2, 0.02, 1.0), rand((128,), 3, 0.5, 1.0)
    q, k, v = jo.qkv_norm_rope_pack(qkv.to(dev), H, qw.to(dev), kw.to(dev), None, None, 1e-6, False)
    rq, rk, rv = ops.qkv_text_pack(qkv, H, qw, kw, 1e-6)
    assert torch.equal(v.cpu(), rv)
    # double rounding: a 1-ulp flip of bf16(x*r) becomes |w| ulps of the output
    assert assert_ulp_close(q, rq, 2.0, what="text q") > 0.99
    assert assert_ulp_close(k, rk, 4.0, what="text k") > 0.99


def test_pack_into_buffer_slices(jo, dev):
    L, H = 300, 4
    qkv = rand((L, 3 * H * 128), 4)
    qw, kw = rand((128,), 5, 0.02, 1.0), rand((128,), 6, 0.02, 1.0)
    from joyomni_ops import rope

    cos, sin = rope.video_chunk_tables(3, 10, 10, 2)
    Q = torch.full((L + 50, H, 128), 7.0, dtype=BF, device=dev)
    K = torch.full((100 + L + 50, H, 128), 7.0, dtype=BF, device=dev)
    V = torch.full_like(K, 7.0)
    jo.qkv_norm_rope_pack_into(qkv.to(dev), H, qw.to(dev), kw.to(dev), cos.to(dev), sin.to(dev), Q[:L],
                               K[100:100 + L], V[100:100 + L])
    rq, rk, rv = ops.qkv_norm_rope_pack(qkv, H, qw, kw, cos, sin, 1e-6, head_major=False)
    assert torch.equal(V[100:100 + L].cpu(), rv)
    assert_ulp_close(Q[:L], rq, 1.0, what="q")
    assert_ulp_close(K[100:100 + L], rk, 1.0, what="k")
    for t, rows in ((Q, slice(L, None)), (K, slice(0, 100)), (K, slice(100 + L, None)), (V, slice(0, 100))):
        assert (t[rows] == 7.0).all(), "write outside the target rows"


@pytest.mark.parametrize("M,N", [(10800, 12288), (512, 12288), (5, 3072), (3, 100)])
def test_gelu_quant(jo, dev, M, N):
    x = rand((M, N), 7, 2.0)
    xg = x.to(dev)
    q, s = jo.gelu_quant_fp8(xg)
    y = jo.gelu_tanh(xg)  # same GELU arithmetic: the exact bf16 intermediate of the fused op
    assert quant_matches(q, s, y)
    # against the full oracle: bit-exact on every row whose bf16 GELU matches torch's
    ry = ops.gelu_tanh(x)
    same = (y.cpu() == ry).all(dim=1)
    rq, rs = ops.per_token_quant_fp8(ry)
    assert torch.equal(q.cpu()[same].view(torch.uint8), rq[same].view(torch.uint8))
    assert torch.equal(s.cpu()[same], rs[same])


@pytest.mark.parametrize("M,N", [(10800, 3072), (512, 3072), (7, 4096)])
def test_gated_residual_norm_quant(jo, dev, M, N):
    res, x = rand((M, N), 8), rand((M, N), 9)
    gate, scale, shift = rand((1, N), 10, 0.1), rand((1, N), 11, 0.1), rand((1, N), 12, 0.1)
    g = lambda t: t.to(dev)
    h, q, s = jo.gated_residual_norm_scale_shift_quant_fp8(g(res), g(x), g(gate), g(scale), g(shift), "layer", 1e-6)
    assert_ulp_close(h, ops.gated_residual(res, x, gate), 1.0, what="h")
    _, y = jo.gated_residual_norm_scale_shift(g(res), g(x), g(gate), g(scale), g(shift), "layer", 1e-6)
    assert quant_matches(q, s, y)
    assert_ulp_close(y, ops.norm_scale_shift(h.cpu(), None, None, scale, shift, "layer", 1e-6), 1.0, what="y")


# ------------------------------------------------------------------ the chain
class CpuLinear:
    def __init__(self, w):
        self.wq, self.ws = w.wq.cpu(), w.ws.cpu()
        self.bias = None if w.bias is None else w.bias.cpu()


class CpuStream:
    def __init__(self, s):
        self.mod_table, self.q_norm, self.k_norm = s.mod_table.cpu(), s.q_norm.cpu(), s.k_norm.cpu()
        self.qkv, self.proj, self.up, self.down = (CpuLinear(w) for w in (s.qkv, s.proj, s.up, s.down))


class CpuBlock:
    def __init__(self, w):
        self.img, self.txt = CpuStream(w.img), CpuStream(w.txt)


@pytest.mark.parametrize("hidden,heads,ffn,img_len,txt_len,cache_len", [(256, 2, 1024, 96, 16, 32),
                                                                       (384, 3, 768, 200, 24, 100)])
def test_block_chain(dev, hidden, heads, ffn, img_len, txt_len, cache_len):
    from joyomni_ops import chain, rope

    w = chain.random_block_weights(hidden, heads, ffn, device=dev, seed=3)
    img, txt = rand((img_len, hidden), 20), rand((txt_len, hidden), 21)
    vec = rand((6, hidden), 22, 0.1)
    cos, sin = rope.video_chunk_tables(1, 8, img_len // 8, 5)
    bufs = chain.KVBuffers(cache_len, img_len, txt_len, heads, 128, 1, dev)
    ck, cv = rand((cache_len, heads, 128), 23), rand((cache_len, heads, 128), 24)
    bufs.k[:cache_len].copy_(ck)
    bufs.v[:cache_len].copy_(cv)
    tr = {}
    img_out, txt_out = chain.block_forward(img.to(dev), txt.to(dev), vec.to(dev), cos.to(dev), sin.to(dev), w,
                                           bufs, trace=tr)
    torch.cuda.synchronize()
    T = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in tr.items()}
    W = CpuBlock(w)
    L = img_len
    # --- stage by stage, each against the oracle on the GPU's own stage inputs
    for tag, x, ws, m in (("img", img, W.img, T["mi"]), ("txt", txt, W.txt, T["mt"])):
        m = [r.cpu() for r in m]
        xq, xs = ops.norm_scale_shift_quant_fp8(x, None, None, m[1], m[0], "layer", 1e-6)
        same = (xs.reshape(-1) == T[f"{tag}.xs"].reshape(-1))
        assert same.float().mean() > 0.9, f"{tag}: LN+quant scales"
        gemm_close(T[f"{tag}.qkv"], ops.fp8_linear(T[f"{tag}.xq"], T[f"{tag}.xs"], ws.qkv), f"{tag} qkv")
        assert quant_matches(T[f"{tag}.aq"], T[f"{tag}.as"], T[f"{tag}.attn"])
        gemm_close(T[f"{tag}.proj"], ops.fp8_linear(T[f"{tag}.aq"], T[f"{tag}.as"], ws.proj), f"{tag} proj")
        assert_ulp_close(T[f"{tag}.h"], ops.gated_residual(x, T[f"{tag}.proj"], m[2]), 1.0, what=f"{tag} h")
        # fc1 -> GELU -> FP8 (one fused op): dequantised against the oracle's GELU of its own fc1
        g_ref = ops.gelu_tanh(ops.fp8_linear(T[f"{tag}.hq"], T[f"{tag}.hs"], ws.up)).float()
        g_got = T[f"{tag}.gq"].float() * T[f"{tag}.gs"]
        assert rel_err(g_got, g_ref) < 0.05, f"{tag} up + GELU + quant"
        s_ref = g_ref.abs().amax(dim=1, keepdim=True).clamp_min(1e-8) / 448
        assert torch.allclose(T[f"{tag}.gs"], s_ref, rtol=2e-2), f"{tag} GELU row scales"
        out_ref = ops.fp8_scaled_mm_gated_residual(T[f"{tag}.gq"], ws.down.wq, T[f"{tag}.gs"], ws.down.ws,
                                                   ws.down.bias, T[f"{tag}.h"], m[5])
        gemm_close(T[f"{tag}.out"], out_ref, f"{tag} down + gated residual")
    q_img, k_img, v_img = ops.qkv_norm_rope_pack(T["img.qkv"], heads, W.img.q_norm, W.img.k_norm, cos, sin, 1e-6,
                                                 head_major=False)
    q_txt, k_txt, v_txt = ops.qkv_text_pack(T["txt.qkv"], heads, W.txt.q_norm, W.txt.k_norm, 1e-6)
    assert_ulp_close(T["q"][:L], q_img, 1.0, what="q img")
    assert_ulp_close(T["k"][cache_len:cache_len + L], k_img, 1.0, what="k img")
    assert torch.equal(T["v"][cache_len:cache_len + L], v_img)
    assert_ulp_close(T["q"][L:], q_txt, 4.0, what="q txt")
    assert torch.equal(T["v"][cache_len + L:], v_txt)
    assert torch.equal(T["k"][:cache_len], ck) and torch.equal(T["v"][:cache_len], cv)
    attn_ref = ops.attention(T["q"], T["k"], T["v"])
    assert rel_err(torch.cat([T["img.attn"], T["txt.attn"]]), attn_ref) < 1e-2
    # --- end to end against the oracle chain
    r_img, r_txt = ops.block_forward(img, txt, vec, cos, sin, W, ck, cv, heads)
    assert rel_err(img_out, r_img) < 2e-2 and rel_err(txt_out, r_txt) < 2e-2


# ------------------------------------------------------------------ attention split + merge
@pytest.mark.parametrize("Sq,S,split,H", [(300, 1000, 700, 4), (129, 257, 1, 2), (64, 4096, 3072, 24)])
def test_attention_split_merge(jo, dev, Sq, S, split, H):
    """Attention over [0, split) and [split, S) merged by log-sum-exp equals attention over
    all rows: against the fp32 oracle within the tolerance of the single-call attention, and
    the merge kernel against its own formula on the same partial results."""
    from joyomni_ops import chain

    q, k, v = rand((Sq, H, 128), 30).to(dev), rand((S, H, 128), 31).to(dev), rand((S, H, 128), 32).to(dev)
    merged = chain.attention_split(q, k, v, split)
    full = chain.attention(q, k, v)
    ref = ops.attention(q.cpu(), k.cpu(), v.cpu())
    err_full, err_split = rel_err(full, ref), rel_err(merged, ref)
    assert err_split < 1e-2 and err_split <= 2 * err_full + 1e-3, (err_split, err_full)
    # the merge kernel on the same partial results, against the formula in fp32 (the
    # log-sum-exps are natural logarithms of the scaled scores)
    oa, la = chain.attention_lse(q, k[:split], v[:split])
    ob, lb = chain.attention_lse(q, k[split:], v[split:])
    got = jo.attn_merge(oa, la, ob, lb)
    m = torch.maximum(la, lb)
    wa, wb = torch.exp(la - m), torch.exp(lb - m)
    want = ((wa / (wa + wb))[..., None] * oa.float() + (wb / (wa + wb))[..., None] * ob.float())
    want = want[0].transpose(0, 1).to(BF)  # [Sq, H, D]
    assert_ulp_close(got, want, 1.0, what="attn_merge")
    # the log-sum-exp convention: natural log of sum(exp(q.k / sqrt(D)))
    s = (q[:4].float().transpose(0, 1) @ k[:split].float().permute(1, 2, 0)) / 128 ** 0.5
    assert torch.allclose(la[0, :, :4].float(), torch.logsumexp(s, dim=-1), rtol=1e-3, atol=1e-2)


# ------------------------------------------------------------------ KV store path
def test_store_advance_rotate(dev):
    """A store forward writes the chunk's pre-RoPE keys into the spare slot and its values
    into the staging block; advancing the window moves them into the evicted slot; the
    rotation of the cache equals the reference's cached K/V pack on the pre-RoPE keys."""
    from joyomni_ops import chain, rope

    hidden, heads, ffn, L, T = 256, 2, 512, 64, 16
    w = chain.random_block_weights(hidden, heads, ffn, device=dev, seed=4)
    bufs = chain.KVBuffers(2 * L, L, T, heads, 128, 1, dev, store=True)
    for i in range(2):  # a window of two cached chunks with known pre-RoPE keys and values
        bufs.k_pre[i].copy_(rand((L, heads, 128), 40 + i))
        bufs.v[bufs.cache_slot_rows(i)].copy_(rand((L, heads, 128), 50 + i))
    pre_before = bufs.k_pre.clone()
    img, txt, vec = rand((L, hidden), 60).to(dev), rand((T, hidden), 61).to(dev), rand((6, hidden), 62, 0.1).to(dev)
    cos, sin = rope.video_chunk_tables(1, 8, L // 8, 5)
    tr = {}
    chain.block_forward(img, txt, vec, cos.to(dev), sin.to(dev), w, bufs, trace=tr, store=True)
    chain.store_chunk_kv(bufs, 0, None)
    torch.cuda.synchronize()
    W = CpuBlock(w)
    _, _, rv, rpre = ops.qkv_norm_rope_pack(tr["img.qkv"].cpu(), heads, W.img.q_norm, W.img.k_norm, cos, sin, 1e-6,
                                            head_major=False, with_pre=True)
    assert_ulp_close(bufs.k_pre[bufs.spare], rpre, 1.0, what="stored pre-RoPE keys")
    assert torch.equal(bufs.v_stage.cpu(), rv)
    assert torch.equal(bufs.k_pre[:2], pre_before[:2]), "the window's own slots must not change"
    spare = bufs.spare
    chain.advance_window(bufs, 1)  # the stored chunk replaces cache slot 1
    assert bufs.k_pre_of == [0, spare] and bufs.spare == 1
    assert torch.equal(bufs.v[bufs.cache_slot_rows(1)].cpu(), rv)
    # window-relative tables for the two slots: full-width fp32 [2L, 128]
    (cf, sf), _ = ops.rope_video_tables(2, 8, L // 8, 3)
    chain.rotate_cache(bufs, cf.to(dev), sf.to(dev))
    torch.cuda.synchronize()
    want_k, _ = ops.cached_kv_pack(bufs.k_pre[0].cpu()[None], bufs.v[:L].cpu()[None],
                                   bufs.k_pre[spare].cpu()[None], bufs.v[L:2 * L].cpu()[None], cf, sf)
    assert_ulp_close(bufs.k[:2 * L], want_k[0], 1.0, what="rotated cache keys")
