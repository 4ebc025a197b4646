"""Small single-kernel workloads for ncu captures.

Each case builds inputs larger than L2 where the kernel streams memory (so
DRAM counters mean something) but holds at most a few GB, runs the kernel
once as a warm-up and once more for the capture, then synchronises and
exits.  Usage (one GPU):

    python -m rusteeze_b200.utils.profile_cases --case rms_norm
    ncu --set full --clock-control none -k regex:rms_norm -s 1 -c 1 -o prof \\
        python -m rusteeze_b200.utils.profile_cases --case rms_norm

`--list` prints the cases with the kernel-name regex to pass to `-k`.
"""
from __future__ import annotations

import argparse
import sys

import torch

from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref

CASES = {}


def case(name: str, kernel: str):
    def deco(fn):
        CASES[name] = (fn, kernel)
        return fn
    return deco


def _bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@case("rms_norm", "rms_norm_kernel")
def _rms_norm():
    x, r, w = _bf(16384, 4096), _bf(16384, 4096), _bf(4096)
    return lambda: ops.fused_add_rms_norm(x, r, w, 1e-5)


@case("rope_cache", "rope_cache_kernel")
def _rope_cache():
    T, Hq, Hkv, D = 16384, 32, 8, 128
    qkv = _bf(T, (Hq + 2 * Hkv) * D)
    pos = torch.randint(0, 8192, (T,), device="cuda")
    cs = ref.rope_cos_sin_cache(D, 8192, 500000.0, None, device="cuda")
    nb = T // 16 + 8
    kc, vc = _bf(nb, Hkv, 16, D), _bf(nb, Hkv, 16, D)
    slots = torch.randperm(nb * 16, device="cuda")[:T]
    return lambda: ops.rope_and_cache(qkv, pos, cs, kc, vc, slots, Hq, Hkv, D)


@case("silu_mul", "act_mul_kernel")
def _silu_mul():
    x = _bf(8192, 2 * 14336)
    return lambda: ops.silu_mul(x)


@case("gemm_bf16", "gemm_tcgen05")
def _gemm_bf16():
    x, w = _bf(1256, 4096), _bf(28672, 4096, scale=0.02)
    return lambda: ops.linear(x, w)


@case("gemm_mxf8", "gemm_tcgen05")
def _gemm_mxf8():
    x = _bf(1256, 4096)
    wq, ws = ref.quant_mxf8_weight(torch.randn(28672, 4096, device="cuda") * 0.02)
    wsf = ref.pack_block_scales_ue8m0(ws)
    xq, sfa = ops.quant_mxf8_act(x)
    y = torch.empty(1256, 28672, device="cuda", dtype=torch.bfloat16)
    return lambda: ops.cuda_ext().gemm_mxf8(y, xq, sfa, wq, wsf, None, None, 0, 0, 0)


@case("quant_mxf8", "quant_mxf8_act_kernel")
def _quant_mxf8():
    x = _bf(8192, 14336)
    return lambda: ops.quant_mxf8_act(x)


@case("gemm_fp8_promote", "gemm_fp8")
def _gemm_fp8_promote():
    x = _bf(1256, 4096)
    wq, ws = ref.quant_fp8_weight(torch.randn(28672, 4096, device="cuda") * 0.02)
    return lambda: ops.linear_fp8(x, wq, ws)


@case("decode_attention", "decode_attn_kernel")
def _decode():
    B, ctx, Hq, Hkv, D = 256, 1232, 32, 8, 128
    from rusteeze_b200.engine.model_runner import choose_num_splits
    nblk = (ctx + 15) // 16
    nb = B * nblk + 16
    cache = _bf(nb, 1, 2, Hkv, 16, D)
    bt = torch.randperm(nb, device="cuda")[: B * nblk].view(B, nblk).int().contiguous()
    sl = torch.full((B,), ctx, device="cuda", dtype=torch.int32)
    q = _bf(B, Hq, D)
    sp = choose_num_splits(B, Hkv, nblk)
    ws = torch.empty(B * Hq * sp * (D + 2), device="cuda")
    o = torch.empty_like(q)
    return lambda: ops.cuda_ext().decode_attention(o, q, cache[:, 0, 0], cache[:, 0, 1], sl, bt, ws, B,
                                                   D ** -0.5, 0, 0.0, sp)


def _prefill_setup():
    S, L, Hq, Hkv, D = 4, 1024, 32, 8, 128
    nblk = (L + 15) // 16
    cache = _bf(S * nblk + 8, 1, 2, Hkv, 16, D)
    bt = torch.arange(S * nblk, device="cuda").view(S, nblk).int().contiguous()
    sl = torch.full((S,), L, device="cuda", dtype=torch.int32)
    qsl = torch.arange(0, (S + 1) * L, L, device="cuda", dtype=torch.int32)
    q = _bf(S * L, Hq, D)
    return cache, bt, sl, qsl, q, torch.empty_like(q), S, L, D


@case("prefill_attention_tc", "prefill_tc_kernel")
def _prefill_tc():
    cache, bt, sl, qsl, q, o, S, L, D = _prefill_setup()
    return lambda: ops.cuda_ext().prefill_attention_impl(o, q, cache[:, 0, 0], cache[:, 0, 1], qsl, sl, bt, 0, S, L,
                                                         D ** -0.5, 0, 0.0, 2)


@case("prefill_attention", "prefill_attn_kernel")
def _prefill():
    S, L, Hq, Hkv, D = 4, 1024, 32, 8, 128
    nblk = (L + 15) // 16
    cache = _bf(S * nblk + 8, 1, 2, Hkv, 16, D)
    bt = torch.arange(S * nblk, device="cuda").view(S, nblk).int().contiguous()
    sl = torch.full((S,), L, device="cuda", dtype=torch.int32)
    qsl = torch.arange(0, (S + 1) * L, L, device="cuda", dtype=torch.int32)
    q = _bf(S * L, Hq, D)
    o = torch.empty_like(q)
    return lambda: ops.cuda_ext().prefill_attention(o, q, cache[:, 0, 0], cache[:, 0, 1], qsl, sl, bt, 0, S, L,
                                                    D ** -0.5, 0, 0.0)


@case("sample_topk_topp", "sample_cluster_kernel")
def _sample():
    B, V = 256, 128256
    logits = torch.randn(B, V, device="cuda") * 3
    f = lambda v, dt: torch.full((B,), v, dtype=dt, device="cuda")  # noqa: E731
    args = (f(0.7, torch.float32), f(-1, torch.int32), f(0.9, torch.float32), f(0.0, torch.float32),
            torch.arange(B, device="cuda"), f(0, torch.int64))
    return lambda: ops.sample(logits, *args, greedy_all=False)


@case("spec_verify", "spec_verify_kernel")
def _spec_verify():
    B, k, V = 64, 4, 128256
    tl = torch.randn(B * (k + 1), V, device="cuda") * 3
    dl = torch.randn(B * k, V, device="cuda") * 3
    dt = torch.randint(0, V, (B, k), device="cuda")
    temps = torch.full((B,), 0.8, device="cuda")
    seeds = torch.arange(B, device="cuda")
    offs = torch.zeros(B, dtype=torch.int64, device="cuda")
    out = torch.empty(B, k + 1, dtype=torch.int64, device="cuda")
    nacc = torch.empty(B, dtype=torch.int32, device="cuda")
    return lambda: ops.cuda_ext().spec_verify(out, nacc, tl, dl, dt, temps, seeds, offs)


@case("moe_route", "moe_route_kernel")
def _moe_route():
    M, H, E = 16384, 4096, 8
    h, wr = _bf(M, H), _bf(E, H, scale=0.05)
    tw = torch.empty(M, 2, device="cuda")
    tid = torch.empty(M, 2, device="cuda", dtype=torch.int32)
    cnt = torch.zeros(E, device="cuda", dtype=torch.int32)
    return lambda: ops.cuda_ext().moe_route(tw, tid, cnt, h, wr, 2, 0, E, True)


@case("moe_grouped_gemm", "gemm_tcgen05")
def _moe_grouped():
    M, H, I, E = 2048, 4096, 14336, 8
    h, router = _bf(M, H), _bf(E, H, scale=0.05)
    w13 = ops.interleave_gate_up_experts(_bf(E, 2 * I, H, scale=0.02))
    w2 = _bf(E, H, I, scale=0.02)
    return lambda: ops.moe_forward(h, router, w13, w2, 2)


_TP1 = {}


def _fused_tp_one_rank(M=4096, H=4096, K=2048, N=3072):
    """A one-rank FusedTP group (Llama-3-8B TP2 shapes per rank): the fused boundary
    kernels run as they do at TP > 1, with every peer store landing locally -- ncu never
    wraps a multi-rank command, so this is how their tensor / DRAM counters are read.
    The setup launches one GEMM and one rs_norm_ag of its own: skip 2 matching launches
    (`-s 2`) to capture the timed one."""
    if not _TP1:
        import os
        import socket
        import torch.distributed as dist
        from rusteeze_b200.parallel.fused_tp import FusedTP
        if not dist.is_initialized():
            sk = socket.socket()
            sk.bind(("127.0.0.1", 0))
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", str(sk.getsockname()[1]))
            sk.close()
            dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
        F = FusedTP(dist.group.WORLD, 0, 1, torch.device("cuda", 0), M, H)
        x, w_o, w_qkv, h0 = _bf(M, K), _bf(H, K, scale=0.02), _bf(N, H, scale=0.02), _bf(M, H)
        w_n = torch.ones(H, device="cuda", dtype=torch.bfloat16)
        F.start(h0, w_n, 1e-5, 0.0)
        F.gemm_rs(x, w_o, 1)                       # flags of boundary 1 carry this step's epoch
        g = F.rs_norm_ag(M, w_n, 1e-5, 0.0, 1)
        torch.cuda.synchronize()
        _TP1.update(F=F, x=x, w_o=w_o, w_qkv=w_qkv, w_n=w_n, g=g, M=M)
    return _TP1


@case("gemm_peer_rs_1rank", "gemm_tcgen05")
def _gemm_peer_rs():
    t = _fused_tp_one_rank()
    return lambda: t["F"].gemm_rs(t["x"], t["w_o"], 1)


@case("rs_norm_ag_1rank", "rs_norm_ag_kernel")
def _rs_norm_ag():
    t = _fused_tp_one_rank()
    return lambda: t["F"].rs_norm_ag(t["M"], t["w_n"], 1e-5, 0.0, 1)


@case("gemm_ag_1rank", "gemm_tcgen05")
def _gemm_ag():
    t = _fused_tp_one_rank()
    return lambda: t["F"].gemm_ag(t["g"], t["w_qkv"], 1)


@case("moe_combine_peer_1rank", "moe_combine_peer_kernel")
def _moe_combine_peer():
    """Mixtral-8x7B expert layer on a one-rank FusedTP group (all 8 experts local, 2048
    tokens): route, grouped expert GEMMs and the combine kernel that stores every weighted
    expert row into its owner's slot -- the capture selects the combine.  A one-rank group
    has one slot per row, so the case routes top-1 (the combine kernel is the same)."""
    t = _fused_tp_one_rank(M=2048, H=4096, K=4096, N=4096)
    if "moe" not in t:
        E, I = 8, 14336
        router = _bf(E, 4096, scale=0.05)
        w13 = ops.interleave_gate_up_experts(_bf(E, 2 * I, 4096, scale=0.02))
        w2 = _bf(E, 4096, I, scale=0.02)
        t["moe"] = (router, w13, w2)
    router, w13, w2 = t["moe"]
    return lambda: t["F"].moe(t["g"], router, w13, w2, 1, 0, 1, 2)


@case("peer_all_reduce_1rank", "peer_all_reduce_kernel")
def _peer_all_reduce():
    """The peer all-reduce on a one-rank group (the 256 x 4096 decode message of
    Llama-3-8B and its two-shot path at 4096 x 4096 share the kernel)."""
    t = _fused_tp_one_rank()
    if "ar" not in t:
        import torch.distributed as dist
        from rusteeze_b200.parallel.comm import PeerAllReduce
        t["ar"] = PeerAllReduce(dist.group.WORLD, 0, 1, torch.device("cuda", 0), 4096 * 4096)
        t["ar_x"] = _bf(4096, 4096)
    return lambda: t["ar"].all_reduce(t["ar_x"])


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None)
    ap.add_argument("--list", action="store_true")
    a = ap.parse_args()
    if a.list or not a.case:
        for n, (_, k) in CASES.items():
            print(f"{n}\t{k}")
        return 0
    fn = CASES[a.case][0]()
    fn()
    torch.cuda.synchronize()
    fn()
    torch.cuda.synchronize()
    status = int(ops.cuda_ext().status()[0])
    print(f"{a.case}: ok status={status}")
    if _TP1:
        import torch.distributed as dist
        _TP1.clear()
        dist.destroy_process_group()
    return 0 if status == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
