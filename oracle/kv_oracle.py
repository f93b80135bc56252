"""PagedKVCache bookkeeping restatement -- TEST INFRASTRUCTURE ONLY.

Pure-Python restatement of the block allocator of the reference's
PagedKVCache (src/kv_cache.rs:29-93): a free stack initialised to
(0..max_blocks).rev(), one block table per (layer, seq_id), a block popped
when a table is empty or its last block is full, free_seq pushing every block
of the sequence back. Values are tracked as Python lists.
"""
from __future__ import annotations


class KVOracle:
    def __init__(self, num_layers, num_heads, head_dim, block_size, max_blocks):
        self.block_size = block_size
        self.max_blocks = max_blocks
        self.free_blocks = list(range(max_blocks))[::-1]  # src/kv_cache.rs:43
        self.tables = {}  # (layer, seq) -> [block ids]
        self.fill = {}    # block -> tokens in it
        self.data = {}    # (layer, seq) -> [(k, v)]

    def append_kv(self, layer, seq, k, v):
        """src/kv_cache.rs:54-67"""
        t = self.tables.setdefault((layer, seq), [])
        if not t or self.fill[t[-1]] >= self.block_size:
            if not self.free_blocks:
                raise RuntimeError("KV cache out of blocks")
            b = self.free_blocks.pop()
            t.append(b)
            self.fill[b] = 0
        self.fill[t[-1]] += 1
        self.data.setdefault((layer, seq), []).append((k, v))

    def get_kv(self, layer, seq):
        """src/kv_cache.rs:69-80"""
        d = self.data.get((layer, seq), [])
        return [k for k, _ in d], [v for _, v in d]

    def free_seq(self, seq):
        """src/kv_cache.rs:82-89 (layers visited in ascending order)."""
        for key in sorted(k for k in self.tables if k[1] == seq):
            for b in self.tables.pop(key):
                self.fill[b] = 0
                self.free_blocks.append(b)
            self.data.pop(key, None)

    def used_blocks(self):
        return self.max_blocks - len(self.free_blocks)

    def free_block_count(self):
        return len(self.free_blocks)

    def num_tables(self):
        return len(self.tables)
