"""Kernel microbenchmarks with CUDA-event timing and roofline fractions.

    python -m rusteeze_b200.utils.kernel_bench [--only gemm,decode,decode_fp8,prefill,norm,sample] [--json out.json]

Each case: warm-up launches, then N timed launches bracketed by events on the
launching stream (synchronize on both sides), inputs sized above the 126 MB
L2 where the op is memory-bound (weights / KV caches), and the achieved
rate divided by the measured peaks in MEASURED_PEAKS.json (HBM copy GB/s and
cuBLAS bf16 TFLOP/s) when present.  cuBLAS (torch.matmul) is timed on the
same shapes as the library baseline for the GEMM.  GEMM rows report the tile plan
(bn, k_splits).
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Callable, Dict, List

import torch

from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref


def peaks() -> Dict[str, float]:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    p = os.path.join(here, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


ITERS = [20, 5]     # timed iterations, warm-up launches (overridable from the command line)


def time_ms(fn: Callable[[], None], iters: int = 0, warmup: int = -1) -> float:
    iters = iters or ITERS[0]
    warmup = ITERS[1] if warmup < 0 else warmup
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(pk, shapes=None) -> List[dict]:
    shapes = shapes or [(1, 4096, 4096), (8, 6144, 4096), (64, 28672, 4096), (256, 6144, 4096),
                        (256, 28672, 4096), (256, 4096, 14336), (1256, 6144, 4096), (1256, 28672, 4096),
                        (1256, 4096, 14336), (4096, 4096, 4096), (8192, 8192, 8192), (256, 128256, 4096)]
    out = []
    for M, N, K in shapes:
        # several weight copies so consecutive launches do not hit in L2
        ncopies = max(1, min(8, int(3 * 126e6 // (N * K * 2)) + 1))
        ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(ncopies)]
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        it = [0]

        def ours():
            it[0] = (it[0] + 1) % ncopies
            ops.linear(x, ws[it[0]], out=y)

        def cublas():
            it[0] = (it[0] + 1) % ncopies
            torch.matmul(x, ws[it[0]].t(), out=y)

        t = time_ms(ours)
        tc = time_ms(cublas)
        flops = 2.0 * M * N * K
        bytes_ = (N * K + M * K + M * N) * 2
        C = ops.cuda_ext()
        plan = C.gemm_plan(M, N, K, 0)
        out.append({"kernel": "gemm_bf16_tcgen05", "M": M, "N": N, "K": K, "bn": plan[0], "k_splits": plan[1],
                    "ms": round(t, 4), "tflops": round(flops / t / 1e9, 1),
                    "frac_of_measured_bf16": round(flops / t / 1e9 / pk["bf16_tflops"], 3),
                    "gbs": round(bytes_ / t / 1e6, 1), "frac_of_measured_hbm": round(bytes_ / t / 1e6 / pk["hbm_gbs"], 3),
                    "cublas_ms": round(tc, 4), "speedup_vs_cublas": round(tc / t, 3)})
        del ws
    return out


def bench_gemm_fp8(pk, shapes=None) -> List[dict]:
    """Block-scaled fp8 GEMM incl. the 1x128 activation quantisation kernel."""
    shapes = shapes or [(8, 6144, 4096), (256, 28672, 4096), (256, 4096, 14336), (1256, 28672, 4096),
                        (1256, 4096, 14336), (4096, 4096, 4096), (8192, 8192, 8192)]
    out = []
    for M, N, K in shapes:
        ncopies = max(1, min(8, int(3 * 126e6 // (N * K)) + 1))
        qs = [ref.quant_fp8_weight(torch.randn(N, K, device="cuda") * 0.02) for _ in range(ncopies)]
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        it = [0]

        def ours():
            it[0] = (it[0] + 1) % ncopies
            ops.linear_fp8(x, *qs[it[0]])

        t = time_ms(ours)
        flops = 2.0 * M * N * K
        bytes_ = N * K + M * K * 2 + M * N * 2
        out.append({"kernel": "gemm_fp8_block_tcgen05", "M": M, "N": N, "K": K, "ms": round(t, 4),
                    "tflops": round(flops / t / 1e9, 1), "gbs": round(bytes_ / t / 1e6, 1),
                    "frac_of_measured_hbm": round(bytes_ / t / 1e6 / pk["hbm_gbs"], 3)})
        del qs
    return out


def bench_gemm_mxf8(pk, shapes=None, bns=(0, 128, 256)) -> List[dict]:
    """MXFP8 GEMM (UE8M0 block scales applied in the MMA) incl. the activation
    quantisation kernel; bn=0 is the planner's choice."""
    shapes = shapes or [(8, 6144, 4096), (256, 28672, 4096), (256, 4096, 14336), (1256, 6144, 4096),
                        (1256, 28672, 4096), (1256, 4096, 14336), (4096, 4096, 4096), (8192, 8192, 8192)]
    out = []
    C = ops.cuda_ext()
    for M, N, K in shapes:
        ncopies = max(1, min(8, int(3 * 126e6 // (N * K)) + 1))
        ws = []
        for _ in range(ncopies):
            q, s = ref.quant_mxf8_weight(torch.randn(N, K, device="cuda") * 0.02)
            ws.append((q, ref.pack_block_scales_ue8m0(s)))
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        for bn in bns:
            it = [0]

            def ours():
                it[0] = (it[0] + 1) % ncopies
                xq, sfa = ops.quant_mxf8_act(x)
                C.gemm_mxf8(y, xq, sfa, ws[it[0]][0], ws[it[0]][1], None, None, 0, bn, 1 if bn else 0)

            t = time_ms(ours)
            flops = 2.0 * M * N * K
            bytes_ = N * K + M * K * 2 + M * N * 2
            plan = list(C.gemm_plan_mxf8(M, N, K, 0)) if bn == 0 else [bn, 1]
            out.append({"kernel": "gemm_mxf8_tcgen05", "M": M, "N": N, "K": K, "bn": plan[0], "k_splits": plan[1],
                        "ms": round(t, 4), "tflops": round(flops / t / 1e9, 1), "gbs": round(bytes_ / t / 1e6, 1),
                        "frac_of_measured_hbm": round(bytes_ / t / 1e6 / pk["hbm_gbs"], 3)})
        del ws
    return out


def bench_decode(pk, cases=None, kv: str = "bf16") -> List[dict]:
    """Split-KV decode attention over a paged cache of bf16 or fp8 (e4m3) pages; bytes are
    the KV bytes the step must read (half for fp8)."""
    cases = cases or [(1, 1024, 32, 8), (16, 1024, 32, 8), (64, 2048, 32, 8), (256, 1232, 32, 8),
                      (256, 4096, 32, 8)]
    out = []
    D = 128
    esz = 1 if kv == "fp8" else 2
    for B, ctx, Hq, Hkv in cases:
        nblk = (ctx + 15) // 16
        nb = B * nblk + 16
        cache = torch.randn(nb, 1, 2, Hkv, 16, D, device="cuda", dtype=torch.bfloat16)
        if kv == "fp8":
            cache = cache.to(torch.float8_e4m3fn)
        bt = torch.randperm(nb, device="cuda")[: B * nblk].view(B, nblk).int().contiguous()
        sl = torch.full((B,), ctx, device="cuda", dtype=torch.int32)
        q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
        from rusteeze_b200.engine.model_runner import choose_num_splits
        sp = choose_num_splits(B, Hkv, nblk)
        wsp = torch.empty(B * Hq * sp * (D + 2), device="cuda")
        o = torch.empty_like(q)

        def fn():
            ops.cuda_ext().decode_attention(o, q, cache[:, 0, 0], cache[:, 0, 1], sl, bt, wsp, B, D ** -0.5, 0, 0.0,
                                            sp)

        t = time_ms(fn)
        bytes_ = B * ctx * Hkv * D * 2 * esz
        out.append({"kernel": "decode_attention" + ("_fp8kv" if kv == "fp8" else ""), "B": B, "ctx": ctx,
                    "Hq": Hq, "Hkv": Hkv, "splits": sp,
                    "ms": round(t, 4), "gbs": round(bytes_ / t / 1e6, 1),
                    "frac_of_measured_hbm": round(bytes_ / t / 1e6 / pk["hbm_gbs"], 3)})
    return out


def bench_decode_fp8(pk, cases=None) -> List[dict]:
    return bench_decode(pk, cases, kv="fp8")


def bench_prefill(pk, cases=None) -> List[dict]:
    cases = cases or [(1, 2048, 32, 8), (4, 1024, 32, 8), (8, 512, 32, 8)]
    out = []
    D = 128
    for S, L, Hq, Hkv in cases:
        nblk = (L + 15) // 16
        nb = S * nblk + 8
        cache = torch.randn(nb, 1, 2, Hkv, 16, D, device="cuda", dtype=torch.bfloat16)
        bt = torch.arange(S * nblk, device="cuda").view(S, nblk).int().contiguous()
        sl = torch.full((S,), L, device="cuda", dtype=torch.int32)
        qsl = torch.arange(0, (S + 1) * L, L, device="cuda", dtype=torch.int32)
        q = torch.randn(S * L, Hq, D, device="cuda", dtype=torch.bfloat16)
        o = torch.empty_like(q)

        for impl, name in ((1, "prefill_attention_mma_sync"), (2, "prefill_attention_tcgen05")):
            def fn():
                ops.cuda_ext().prefill_attention_impl(o, q, cache[:, 0, 0], cache[:, 0, 1], qsl, sl, bt, 0, S, L,
                                                      D ** -0.5, 0, 0.0, impl)

            t = time_ms(fn)
            flops = 4.0 * S * Hq * D * L * (L + 1) / 2      # causal
            out.append({"kernel": name, "seqs": S, "len": L, "Hq": Hq, "Hkv": Hkv, "ms": round(t, 4),
                        "tflops": round(flops / t / 1e9, 1),
                        "frac_of_measured_bf16": round(flops / t / 1e9 / pk["bf16_tflops"], 3)})
    return out


def bench_norm(pk) -> List[dict]:
    out = []
    for rows, H in [(256, 4096), (4096, 4096), (16384, 4096)]:
        x = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16)
        r = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
        t = time_ms(lambda: ops.fused_add_rms_norm(x, r, w, 1e-5))
        bytes_ = rows * H * 2 * 4
        out.append({"kernel": "fused_add_rms_norm", "rows": rows, "H": H, "ms": round(t, 4),
                    "gbs": round(bytes_ / t / 1e6, 1), "frac_of_measured_hbm": round(bytes_ / t / 1e6 / pk["hbm_gbs"], 3)})
    return out


def bench_sample(pk) -> List[dict]:
    """Cluster sampler, top-p 0.9 at T 0.7 and greedy, fp32 and bf16 logits.  Four logit
    buffers are used in turn, so every launch reads its rows from DRAM (L2 is 126 MB)."""
    out = []
    for dt in (torch.float32, torch.bfloat16):
        for B in (1, 64, 256):
            V = 128256
            bufs = [(torch.randn(B, V, device="cuda") * 3).to(dt) for _ in range(4)]
            f = lambda v, t: torch.full((B,), v, dtype=t, device="cuda")  # noqa: E731
            args = (f(0.7, torch.float32), f(-1, torch.int32), f(0.9, torch.float32), f(0.0, torch.float32),
                    torch.arange(B, device="cuda"), f(0, torch.int64))
            it = [0]

            def run(greedy):
                it[0] += 1
                x = bufs[it[0] % 4]
                if greedy:
                    ops.sample(x, None, None, None, None, None, None, greedy_all=True)
                else:
                    ops.sample(x, *args, greedy_all=False)
            t = time_ms(lambda: run(False))
            tg = time_ms(lambda: run(True))
            nbytes = B * V * bufs[0].element_size()
            out.append({"kernel": "sample_cluster", "dtype": str(dt).split(".")[-1], "B": B, "V": V,
                        "ms": round(t, 4), "greedy_ms": round(tg, 4), "gbs": round(nbytes / t / 1e6, 1),
                        "frac_of_measured_hbm": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,decode,prefill,norm,sample")
    ap.add_argument("--json", default=None)
    ap.add_argument("--gemm", default=None, help="single GEMM case M,N,K")
    ap.add_argument("--decode", default=None, help="single decode case B,ctx,Hq,Hkv")
    ap.add_argument("--prefill", default=None, help="single prefill case seqs,len,Hq,Hkv")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    ITERS[0], ITERS[1] = a.iters, a.warmup
    pk = peaks()
    res = {"peaks": pk}
    cases = {"gemm": a.gemm, "gemm_fp8": a.gemm, "gemm_mxf8": a.gemm, "decode": a.decode, "decode_fp8": a.decode,
             "prefill": a.prefill}
    for name in a.only.split(","):
        c = cases.get(name)
        if c:
            res[name] = globals()[f"bench_{name}"](pk, [tuple(int(x) for x in c.split(","))])
        else:
            res[name] = globals()[f"bench_{name}"](pk)
        for row in res[name]:
            print(json.dumps(row), flush=True)
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
