"""Device memory report.

The reference keeps an offset-based allocator and a GPU memory tracker as
pure bookkeeping (crates/rusteeze-tensor/src/memory.rs:96-529) that nothing
allocates through.  Here memory is the torch caching allocator plus ONE
up-front KV pool sized from `gpu_memory_utilization`; this module reports
what is where (weights, KV cache, allocator reserve, free) for `/health`,
`rusteeze info` and the engine log.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch


def tensor_bytes(module: torch.nn.Module) -> int:
    seen, total = set(), 0
    for t in list(module.parameters()) + list(module.buffers()):
        if t.data_ptr() in seen:
            continue
        seen.add(t.data_ptr())
        total += t.numel() * t.element_size()
    return total


def memory_report(engine=None, device: Optional[int] = None) -> Dict[str, float]:
    gib = float(1 << 30)
    rep: Dict[str, float] = {}
    if engine is not None:
        rep["weights_gib"] = tensor_bytes(engine.model) / gib
        r = engine.runner
        kv = getattr(r, "kv_cache", None)
        if kv is not None:
            rep["kv_cache_gib"] = kv.numel() * kv.element_size() / gib
            rep["kv_blocks"] = float(engine.bm.num_gpu_blocks)
            rep["kv_blocks_free"] = float(engine.bm.num_free_gpu_blocks())
            rep["kv_tokens_capacity"] = float(engine.bm.num_gpu_blocks * 16)
    if torch.cuda.is_available():
        dev = torch.cuda.current_device() if device is None else device
        free, total = torch.cuda.mem_get_info(dev)
        rep.update(device=float(dev), total_gib=total / gib, free_gib=free / gib,
                   allocated_gib=torch.cuda.memory_allocated(dev) / gib,
                   reserved_gib=torch.cuda.memory_reserved(dev) / gib,
                   peak_allocated_gib=torch.cuda.max_memory_allocated(dev) / gib)
    return rep
