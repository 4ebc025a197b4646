"""Block manager front door.

The engine uses the C++ implementation (`rusteeze_b200._host.BlockManager`,
csrc/host/block_manager.cpp).  `PyBlockManager` is a line-by-line
behavioural mirror in Python used as the oracle of the property tests
(random allocate/append/fork/free/swap sequences must leave both in the
same state) -- it is not used by the engine.
"""
from __future__ import annotations

import importlib
from collections import OrderedDict
from typing import Dict, List, Tuple



def host_ext():
    try:
        return importlib.import_module("rusteeze_b200._host")
    except ImportError as e:
        raise RuntimeError("rusteeze_b200._host is not built; run `python setup.py build_ext --inplace`") from e


def make_block_manager(block_size: int, num_gpu_blocks: int, num_cpu_blocks: int, enable_prefix_caching: bool):
    return host_ext().BlockManager(block_size, num_gpu_blocks, num_cpu_blocks, enable_prefix_caching)


_M = (1 << 64) - 1


def _mix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & _M
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _M
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _M
    return x ^ (x >> 31)


def _block_key(parent: int, toks) -> int:
    h = _mix64(parent ^ 0x51ED270B27A3C4F1)
    for t in toks:
        h = _mix64(h ^ (int(t) & _M))
    return h


class _Seq:
    def __init__(self):
        self.blocks: List[int] = []
        self.on_cpu = False
        self.num_hashed = 0
        self.last_key = 0


class PyBlockManager:
    def __init__(self, block_size: int, num_gpu_blocks: int, num_cpu_blocks: int, enable_prefix_caching=True):
        self.bs, self.ngpu, self.ncpu, self.prefix = block_size, num_gpu_blocks, num_cpu_blocks, enable_prefix_caching
        self.gpu_free = list(range(num_gpu_blocks - 1, -1, -1))
        self.cpu_free = list(range(num_cpu_blocks - 1, -1, -1))
        self.gpu_ref = [0] * num_gpu_blocks
        self.cpu_ref = [0] * num_cpu_blocks
        self.meta: Dict[int, Tuple[int, tuple]] = {}       # block -> (key, tokens) when hashed
        self.key_to_block: Dict[int, int] = {}
        self.lru: "OrderedDict[int, None]" = OrderedDict()
        self.seqs: Dict[int, _Seq] = {}

    @property
    def num_gpu_blocks(self):
        return self.ngpu

    @property
    def block_size(self):
        return self.bs

    def num_free_gpu_blocks(self):
        return len(self.gpu_free) + len(self.lru)

    def num_free_cpu_blocks(self):
        return len(self.cpu_free)

    def has_seq(self, sid):
        return sid in self.seqs

    def blocks_for(self, n):
        return (n + self.bs - 1) // self.bs

    def cached_prefix_len(self, toks) -> int:
        if not self.prefix:
            return 0
        n = len(toks)
        full = (n - 1) // self.bs if n > 0 else 0
        key, hit = 0, 0
        for b in range(full):
            blk_t = tuple(int(x) for x in toks[b * self.bs:(b + 1) * self.bs])
            key = _block_key(key, blk_t)
            blk = self.key_to_block.get(key)
            if blk is None or self.meta.get(blk) != (key, blk_t):
                break
            hit += 1
        return hit * self.bs

    def allocate_prompt(self, sid, toks) -> int:
        assert sid not in self.seqs
        st = _Seq()
        cached = self.cached_prefix_len(toks)
        key = 0
        for b in range(cached // self.bs):
            key = _block_key(key, toks[b * self.bs:(b + 1) * self.bs])
            blk = self.key_to_block[key]
            if self.gpu_ref[blk] == 0:
                self.lru.pop(blk, None)
            self.gpu_ref[blk] += 1
            st.blocks.append(blk)
        st.num_hashed = cached // self.bs
        st.last_key = key
        self.seqs[sid] = st
        return cached

    def _take(self) -> int:
        if self.gpu_free:
            return self.gpu_free.pop()
        if self.lru:
            b, _ = self.lru.popitem(last=False)
            key, _t = self.meta.pop(b)
            if self.key_to_block.get(key) == b:
                del self.key_to_block[key]
            return b
        return -1

    def _release_gpu(self, b):
        assert self.gpu_ref[b] > 0
        self.gpu_ref[b] -= 1
        if self.gpu_ref[b] == 0:
            if b in self.meta:
                self.lru[b] = None
            else:
                self.gpu_free.append(b)

    def ensure_capacity(self, sid, num_tokens, write_from):
        st = self.seqs[sid]
        cow = []
        need = self.blocks_for(num_tokens)
        for b in range(write_from // self.bs, min(len(st.blocks), need)):
            blk = st.blocks[b]
            if self.gpu_ref[blk] > 1:
                nb = self._take()
                assert nb >= 0
                self.gpu_ref[blk] -= 1
                self.gpu_ref[nb] = 1
                st.blocks[b] = nb
                cow.append((blk, nb))
                if b < st.num_hashed:
                    st.num_hashed, st.last_key = b, 0
        while len(st.blocks) < need:
            nb = self._take()
            assert nb >= 0, "out of KV blocks"
            self.gpu_ref[nb] = 1
            st.blocks.append(nb)
        return cow

    def blocks_to_grow(self, sid, num_tokens, write_from):
        st = self.seqs[sid]
        need = self.blocks_for(num_tokens)
        extra = max(0, need - len(st.blocks))
        for b in range(write_from // self.bs, min(len(st.blocks), need)):
            if self.gpu_ref[st.blocks[b]] > 1:
                extra += 1
        return extra

    def try_grow(self, sid, num_tokens, write_from):
        if self.blocks_to_grow(sid, num_tokens, write_from) > self.num_free_gpu_blocks():
            return None
        return self.ensure_capacity(sid, num_tokens, write_from)

    def commit(self, sid, toks, num_computed):
        if not self.prefix:
            return
        st = self.seqs[sid]
        full = min(num_computed, len(toks)) // self.bs
        if st.num_hashed > 0 and st.last_key == 0:
            k = 0
            for b in range(st.num_hashed):
                k = _block_key(k, toks[b * self.bs:(b + 1) * self.bs])
            st.last_key = k
        while st.num_hashed < full and st.num_hashed < len(st.blocks):
            b = st.num_hashed
            t = tuple(int(x) for x in toks[b * self.bs:(b + 1) * self.bs])
            key = _block_key(st.last_key, t)
            blk = st.blocks[b]
            if key not in self.key_to_block and blk not in self.meta:
                self.key_to_block[key] = blk
                self.meta[blk] = (key, t)
            st.last_key = key
            st.num_hashed = b + 1

    def free(self, sid):
        st = self.seqs.pop(sid, None)
        if st is None:
            return
        for b in reversed(st.blocks):
            if st.on_cpu:
                self.cpu_ref[b] -= 1
                if self.cpu_ref[b] == 0:
                    self.cpu_free.append(b)
            else:
                self._release_gpu(b)

    def fork(self, parent, child):
        p = self.seqs[parent]
        c = _Seq()
        c.blocks, c.on_cpu, c.num_hashed, c.last_key = list(p.blocks), p.on_cpu, p.num_hashed, p.last_key
        for b in c.blocks:
            if p.on_cpu:
                self.cpu_ref[b] += 1
            else:
                self.gpu_ref[b] += 1
        self.seqs[child] = c

    def can_swap_out(self, sid):
        return len(self.seqs[sid].blocks) <= len(self.cpu_free)

    def swap_out(self, sid):
        st = self.seqs[sid]
        m = []
        for i, b in enumerate(st.blocks):
            c = self.cpu_free.pop()
            self.cpu_ref[c] = 1
            m.append((b, c))
            self._release_gpu(b)
            st.blocks[i] = c
        st.on_cpu, st.num_hashed, st.last_key = True, 0, 0
        return m

    def swap_in(self, sid):
        st = self.seqs[sid]
        m = []
        for i, c in enumerate(st.blocks):
            g = self._take()
            self.gpu_ref[g] = 1
            m.append((c, g))
            self.cpu_ref[c] -= 1
            if self.cpu_ref[c] == 0:
                self.cpu_free.append(c)
            st.blocks[i] = g
        st.on_cpu = False
        return m

    def block_table(self, sid):
        return list(self.seqs[sid].blocks)

    def ref_count(self, b):
        return self.gpu_ref[b]
