"""Same-GPU timing of this library's kernels against the reference's own kernels.

    python tests/ref_race.py [--steps K] [--out gpurun_out/ref_race.json]

The reference's light CUDA kernels (compiled unmodified from joyomni_ops/csrc by
oracle/build_ref.py into oracle/_ref/libjoyomni_ref.so, torch.ops.joyomni_ref.*)
and ours (torch.ops.joyomni_ops.*) run the same op on the same inputs on the same
GPU, each timed the way bench.py times its workloads: K steps captured in one CUDA
graph over rotating buffer sets larger than twice the 126 MB L2, one replay timed
with CUDA events (best of three replays).  Shapes are the BASELINE configs, plus
the reference model's cache assembly.  For config 1 the reference arm is the chain
the reference runs on the GPU for that step (dit.py:409-429 with
sgl_fused_ops.py:137-168): q.contiguous(), k.contiguous() and the in-place paired
kernel, and v.contiguous() for a materialised V.

Test infrastructure: the reference library is a checker and a baseline here,
never part of the product.  Prints one JSON object per op and writes them all to
--out.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
for _p in (str(REPO), str(REPO / "joyai-video-edit_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

REF_LIB = REPO / "oracle" / "_ref" / "libjoyomni_ref.so"
L2 = 126 * 1024 * 1024
BF = torch.bfloat16


def rand(shape, seed, scale=1.0, mean=0.0, dt=BF):
    g = torch.Generator().manual_seed(seed)
    return (mean + scale * torch.randn(*shape, generator=g)).to(dt).cuda()


def time_op(make, step, set_bytes, steps):
    """Best-of-three replay time (µs per step) of `steps` captured steps over rotating sets."""
    nsets = max(2, min(16, -(-2 * L2 // set_bytes)))
    sets = [make(i) for i in range(nsets)]
    ring = [None] * nsets

    def run(i):
        ring[i % nsets] = step(sets[i % nsets])

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(steps):
            run(i)
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e3 / steps)
    del g, sets, ring
    torch.cuda.empty_cache()
    return best


def cases(jo, ref):
    from oracle import ops

    L, H, D, N = 10800, 24, 128, 3072
    out = []

    # config 0: RMSNorm [3600, 3072]
    def mk_rms(i):
        return dict(x=rand((3600, N), 100 + i), w=rand((N,), 1, 0.02, 1.0))
    out.append(("rmsnorm [3600,3072] (configs[0])", mk_rms, 2 * 2 * 3600 * N,
                lambda s: jo.rmsnorm(s["x"], s["w"], 1e-6), lambda s: ref.rmsnorm(s["x"], s["w"], 1e-6)))

    # config 2a: LayerNorm + modulate, broadcast [1, N]
    def mk_ln(i):
        return dict(x=rand((L, N), 200 + i), sc=rand((1, N), 2, 0.1), sh=rand((1, N), 3, 0.1))
    out.append(("LN+modulate [10800,3072] (configs[2])", mk_ln, 2 * 2 * L * N,
                lambda s: jo.fused_norm_scale_shift(s["x"], None, None, s["sc"], s["sh"], "layer", 1e-6),
                lambda s: ref.fused_norm_scale_shift(s["x"], None, None, s["sc"], s["sh"], 0, 1e-6)))

    # config 3: per-token FP8 quant [10800, 3072]
    def mk_q(i):
        return dict(x=rand((L, N), 300 + i), q=torch.empty(L, N, dtype=torch.float8_e4m3fn, device="cuda"),
                    s=torch.empty(L, 1, device="cuda"))
    out.append(("per-token FP8 quant [10800,3072] (configs[3])", mk_q, 3 * L * N + 4 * L,
                lambda s: jo.sgl_per_token_quant_fp8(s["x"], s["q"], s["s"]),
                lambda s: ref.sgl_per_token_quant_fp8(s["x"], s["q"], s["s"])))

    # config 1: qkv [10800, 9216] -> q/k/v
    (_, _), (cos, sin) = ops.rope_video_tables(3, 45, 80, 17)
    cos, sin = cos.cuda(), sin.cuda()
    qw, kw = rand((D,), 4, 0.02, 1.0), rand((D,), 5, 0.02, 1.0)

    def mk_qkv(i):
        return dict(qkv=rand((L, 3 * H * D), 400 + i))

    def ref_chain(s):
        q, k, v = s["qkv"].view(1, L, 3, H, D).unbind(2)
        q, k = q.contiguous(), k.contiguous()
        ref.fused_qk_norm_rope_3d_paired(q.view(1, L * H, D), k.view(1, L * H, D), L, H, 1e-6, qw, kw, cos, sin,
                                         None)
        return q, k, v.contiguous()
    bytes1 = 2 * 2 * L * 3 * H * D + 2 * L * (D // 2) * 2
    out.append(("qkv pack + q/k RMSNorm + RoPE, config 1 (ours: one kernel, token-major; reference: "
                "2 contiguous copies + paired kernel + v copy)", mk_qkv, bytes1,
                lambda s: jo.qkv_norm_rope_pack(s["qkv"], H, qw, kw, cos, sin, 1e-6, False), ref_chain))

    # the paired in-place kernel alone, config-1 size
    def mk_paired(i):
        return dict(q=rand((1, L * H, D), 500 + i), k=rand((1, L * H, D), 600 + i))
    out.append(("fused_qk_norm_rope_3d_paired in place, 10800 x 24 x 128", mk_paired, 2 * 2 * 2 * L * H * D,
                lambda s: jo.fused_qk_norm_rope_3d_paired(s["q"], s["k"], L, H, 1e-6, qw, kw, cos, sin, None),
                lambda s: ref.fused_qk_norm_rope_3d_paired(s["q"], s["k"], L, H, 1e-6, qw, kw, cos, sin, None)))

    # joint pack at the chain's shape: cache 4 chunks + 10800 image + 512 text tokens
    C, T = 4 * L, 512

    def mk_joint(i):
        img = rand((1, L, 3, H, D), 700 + i)
        txt = rand((1, T, 3, H, D), 701 + i)
        return dict(img=img.unbind(2), txt=txt.unbind(2), ck=rand((1, C, H, D), 702 + i),
                    cv=rand((1, C, H, D), 703 + i), tw=rand((D,), 6), kw=rand((D,), 7))
    jb = 2 * ((L + T) * H * D * 2 + 2 * (C + L + T) * H * D * 2)
    out.append(("fused_joint_qkv_pack, cache 43200 + img 10800 + txt 512, 24 heads", mk_joint, jb,
                lambda s: jo.fused_joint_qkv_pack(*s["img"], *s["txt"], s["ck"], s["cv"], s["tw"], s["kw"], 1e-6),
                lambda s: ref.fused_joint_qkv_pack(*s["img"], *s["txt"], s["ck"], s["cv"], s["tw"], s["kw"], 1e-6)))

    # cached K/V assembly: sink chunk + 3-chunk local window (two segments)
    ang = torch.rand(C, D // 2, generator=torch.Generator().manual_seed(8)) * 6.28
    fcos = ang.cos().repeat_interleave(2, dim=-1).contiguous().cuda()
    fsin = ang.sin().repeat_interleave(2, dim=-1).contiguous().cuda()

    def mk_cached(i):
        return dict(k0=rand((1, L, H, D), 800 + i), v0=rand((1, L, H, D), 801 + i),
                    k1=rand((1, C - L, H, D), 802 + i), v1=rand((1, C - L, H, D), 803 + i))
    cb = 2 * 2 * 2 * C * H * D + 2 * C * D * 4
    out.append(("fused_cached_kv_pack, 10800 + 32400 cached tokens, 24 heads", mk_cached, cb,
                lambda s: jo.fused_cached_kv_pack(s["k0"], s["v0"], s["k1"], s["v1"], fcos, fsin),
                lambda s: ref.fused_cached_kv_pack(s["k0"], s["v0"], s["k1"], s["v1"], fcos, fsin)))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--out", default=str(REPO / "gpurun_out" / "ref_race.json"))
    args = ap.parse_args()
    import joyomni_ops as jo

    torch.ops.load_library(str(REF_LIB))
    ref = torch.ops.joyomni_ref
    rows = []
    for name, make, nbytes, ours, theirs in cases(jo, ref):
        set_bytes = 2 * nbytes  # inputs + the outputs each step allocates
        t_ours = time_op(make, ours, set_bytes, args.steps)
        t_ref = time_op(make, theirs, set_bytes, args.steps)
        row = {"op": name, "algo_bytes": nbytes, "ours_us": round(t_ours, 2), "ref_us": round(t_ref, 2),
               "ours_over_ref": round(t_ours / t_ref, 4), "ours_gbs": round(nbytes / t_ours / 1e3, 1),
               "ref_gbs": round(nbytes / t_ref / 1e3, 1)}
        print(json.dumps(row), flush=True)
        rows.append(row)
    os.makedirs(os.path.dirname(args.out), exist_ok=True)
    Path(args.out).write_text(json.dumps({"gpu": torch.cuda.get_device_name(), "steps": args.steps, "ops": rows},
                                         indent=1))


if __name__ == "__main__":
    main()
