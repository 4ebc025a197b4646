"""Fused tensor-parallel layer boundary vs the NCCL baseline, per rank of a TP group.

Chain timed (Llama-3-8B shapes, TP = world size):
  fused     o_proj GEMM whose epilogue reduce-scatters into the owners' slots over
            NVLink -> add + RMSNorm + all-gather kernel -> QKV GEMM that starts per
            A tile as its gathered rows land           (parallel.fused_tp)
  baseline  o_proj GEMM -> NCCL all-reduce -> fused add + RMSNorm -> QKV GEMM

Each variant runs `--iters` times after warm-up, eagerly and as one CUDA graph
of `--iters` chains replayed `--replays` times (the speedup and roofline
fraction use the graph numbers: the engine replays decode steps from graphs);
CUDA events on the launching stream, MAX over ranks.  The per-kernel split
(gemm_rs / rs_norm_ag / gemm_ag) is eager, with a barrier per iteration, so it
also carries the ranks' launch skew.  Roofline of the fused chain = the slower of
  compute: FLOPs of both GEMMs / measured bf16 GEMM peak, and
  NVLink:  bytes each rank must send (reduce-scatter + all-gather of M x H bf16,
           (W-1)/W of it leaves the GPU each way) / 770 GB/s per direction.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m rusteeze_b200.utils.tp_bench
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from rusteeze_b200 import ops

NVLINK_GBS = 770.0   # measured peer copy per direction per GPU on this pool


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="256,1024,4096")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--replays", type=int, default=5)
    a = ap.parse_args()
    from rusteeze_b200.parallel.dist import init_distributed
    from rusteeze_b200.parallel.fused_tp import FusedTP
    info = init_distributed(timeout_s=120)
    W, rank, dev = info.world_size, info.rank, info.device
    H, Hq, Hkv, D = 4096, 32, 8, 128
    qkv_n = (Hq + 2 * Hkv) * D // W              # column-parallel QKV rows per rank
    o_k = Hq * D // W                            # row-parallel o_proj K per rank
    Mmax = max(int(x) for x in a.tokens.split(","))
    F = FusedTP(dist.group.WORLD, rank, W, dev, Mmax, H)
    peaks = json.load(open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json"))) \
        if os.path.exists(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")) else \
        {"bf16_tflops": 1590.0}
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    w_o = (torch.randn(H, o_k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w_qkv = (torch.randn(qkv_n, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w_n = torch.ones(H, device=dev, dtype=torch.bfloat16)
    rows = []
    for M in (int(x) for x in a.tokens.split(",")):
        x = (torch.randn(M, o_k, device=dev, generator=g)).to(torch.bfloat16)
        h0 = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
        res = h0.clone()

        def fused():
            F.start(h0, w_n, 1e-5, 0.0)
            F.gemm_rs(x, w_o, 1)
            gg = F.rs_norm_ag(M, w_n, 1e-5, 0.0, 1)
            F.gemm_ag(gg, w_qkv, 1)
            F.end_step()

        def baseline():
            y = ops.linear(x, w_o)
            dist.all_reduce(y)
            x2, _ = ops.fused_add_rms_norm(y, res, w_n, 1e-5)
            ops.linear(x2, w_qkv)

        def start_only():
            F.start(h0, w_n, 1e-5, 0.0)
            F.end_step()

        def local_o():
            ops.linear(x, w_o)

        def local_qkv():
            ops.linear(h0, w_qkv)

        out = {"M": M, "world": W}
        # per-kernel split of the fused chain: events between its launches on the stream
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        split = [0.0, 0.0, 0.0]
        for it in range(a.warmup + a.iters):
            F.start(h0, w_n, 1e-5, 0.0)
            ev[0].record()
            F.gemm_rs(x, w_o, 1)
            ev[1].record()
            gg = F.rs_norm_ag(M, w_n, 1e-5, 0.0, 1)
            ev[2].record()
            F.gemm_ag(gg, w_qkv, 1)
            ev[3].record()
            F.end_step()
            torch.cuda.synchronize()
            dist.barrier()
            if it >= a.warmup:
                for i in range(3):
                    split[i] += ev[i].elapsed_time(ev[i + 1]) / a.iters
        st = torch.tensor(split, device=dev)
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
        out.update(gemm_rs_ms=round(st[0].item(), 4), rs_norm_ag_ms=round(st[1].item(), 4),
                   gemm_ag_ms=round(st[2].item(), 4))
        for name, fn in (("fused", fused), ("baseline", baseline), ("start", start_only),
                         ("local_o_gemm", local_o), ("local_qkv_gemm", local_qkv)):
            for _ in range(a.warmup):
                fn()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out[name + "_ms"] = round(t.item(), 4)
        # the same chains replayed from CUDA graphs (as the engine runs them): no host launch gaps
        for name, fn in (("fused", fused), ("baseline", baseline), ("start", start_only)):
            s2 = torch.cuda.Stream()
            s2.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s2):
                for _ in range(2):
                    fn()
            torch.cuda.current_stream().wait_stream(s2)
            dist.barrier()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for _ in range(a.iters):
                    fn()
            for _ in range(2):
                gr.replay()
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.replays):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / (a.iters * a.replays)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out[name + "_graph_ms"] = round(t.item(), 4)
            del gr                       # graphs holding NCCL calls go before the process group
            torch.cuda.synchronize()
        # the fused chain includes one `start` boundary (it seeds the residual shard): report without it
        chain = out["fused_graph_ms"] - out["start_graph_ms"]
        flops = 2.0 * M * o_k * H + 2.0 * M * H * qkv_n
        t_compute = flops / (peaks["bf16_tflops"] * 1e12) * 1e3
        bytes_out = 2 * M * H * 2 * (W - 1) / W          # RS + AG bytes leaving each GPU
        t_link = bytes_out / (NVLINK_GBS * 1e9) * 1e3
        roof = max(t_compute, t_link)
        out.update(fused_chain_ms=round(chain, 4), roofline_ms=round(roof, 4),
                   roofline_frac=round(roof / chain, 3) if chain > 0 else None,
                   speedup_vs_nccl=round(out["baseline_graph_ms"] / chain, 3) if chain > 0 else None,
                   status=int(ops.cuda_ext().status()[0]))
        rows.append(out)
        if rank == 0:
            print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
