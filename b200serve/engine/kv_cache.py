"""Paged KV cache: device storage plus the host-side block allocator.

Storage per layer is [num_blocks, kv_heads, 16, head_dim] for K and for V, so
one (page, head) is a contiguous 16 x head_dim tile. Blocks are handed out by
``BlockAllocator``, which also keeps a prefix index (hash of the token ids of
each full block chained with its predecessor's hash) so a new request whose
prompt starts with cached blocks reuses them (reference idea: KV-session reuse
on exact prefix extension, webgpu/src/engine/generate.ts:89-117).
"""

from __future__ import annotations

import hashlib
from collections import OrderedDict

import torch

BLOCK = 16


class KVCache:
    """Paged K/V storage. ``bf16``: k, v [layers, blocks, kv_heads, 16, head_dim].
    ``int4g128``: k, v hold 4-bit codes [layers, blocks, kv_heads, 16, head_dim/2] (uint8,
    interleaved nibbles per 8 dims) and k_scale, v_scale one fp16 per (token, head)
    [layers, blocks, kv_heads, 16]: 4-bit K/V with an fp16 scale per group of 128 values.
    ``turboquant``: k, v hold one TurboQuant code (``key_bits`` / ``value_bits``) per dim as a
    nibble [layers, blocks, kv_heads, 16, head_dim/2] (byte m = dims 2m | 2m+1 << 4); k_sign the
    QJL sign bits [.., head_dim/8]; k_scale (norm, gamma) fp16 [.., 2]; v_scale the V norm."""

    def __init__(self, num_layers, num_blocks, kv_heads, head_dim, dtype=torch.bfloat16, device="cpu",
                 kv_format="bf16", key_bits=4, value_bits=4):
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        self.kv_format = kv_format
        self.key_bits, self.value_bits = key_bits, value_bits
        self.k_scale = self.v_scale = self.k_sign = None
        if kv_format == "turboquant":
            if head_dim != 128:
                raise ValueError("turboquant KV needs head_dim 128")
            base = (num_layers, num_blocks, kv_heads, BLOCK)
            self.k = torch.zeros(base + (head_dim // 2,), dtype=torch.uint8, device=device)
            self.v = torch.zeros(base + (head_dim // 2,), dtype=torch.uint8, device=device)
            self.k_sign = torch.zeros(base + (head_dim // 8,), dtype=torch.uint8, device=device)
            self.k_scale = torch.zeros(base + (2,), dtype=torch.float16, device=device)
            self.v_scale = torch.zeros(base, dtype=torch.float16, device=device)
        elif kv_format == "int4g128":
            if head_dim != 128:
                raise ValueError("int4g128 KV needs head_dim 128")
            shape = (num_layers, num_blocks, kv_heads, BLOCK, head_dim // 2)
            self.k = torch.zeros(shape, dtype=torch.uint8, device=device)
            self.v = torch.zeros(shape, dtype=torch.uint8, device=device)
            sshape = (num_layers, num_blocks, kv_heads, BLOCK)
            self.k_scale = torch.zeros(sshape, dtype=torch.float16, device=device)
            self.v_scale = torch.zeros(sshape, dtype=torch.float16, device=device)
        else:
            shape = (num_layers, num_blocks, kv_heads, BLOCK, head_dim)
            self.k = torch.zeros(shape, dtype=dtype, device=device)
            self.v = torch.zeros(shape, dtype=dtype, device=device)

    @staticmethod
    def bytes_per_block(num_layers, kv_heads, head_dim, elem_bytes=2, kv_format="bf16") -> int:
        if kv_format == "turboquant":
            # codes (4 bits per dim) for K and V, K sign bits, K (norm, gamma), V norm
            return num_layers * kv_heads * BLOCK * (head_dim + head_dim // 8 + 6)
        if kv_format == "int4g128":
            return 2 * num_layers * kv_heads * BLOCK * (head_dim // 2 + 2)
        return 2 * num_layers * kv_heads * BLOCK * head_dim * elem_bytes


def _block_hash(prev: bytes, tokens) -> bytes:
    h = hashlib.blake2b(prev, digest_size=16)
    h.update(bytes(memoryview(torch.as_tensor(list(tokens), dtype=torch.int32).numpy())))
    return h.digest()


class BlockAllocator:
    """Reference-counted page allocator with an LRU prefix cache of freed full blocks."""

    def __init__(self, num_blocks: int, enable_prefix_cache: bool = True):
        self.num_blocks = num_blocks
        self.free = list(range(num_blocks - 1, -1, -1))
        self.ref = [0] * num_blocks
        self.hash_of = {}                  # block -> hash (full, registered blocks)
        self.by_hash = {}                  # hash -> block
        self.evictable = OrderedDict()     # hash -> block (ref == 0, still cached)
        self.prefix = enable_prefix_cache

    @property
    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def _take(self) -> int:
        if self.free:
            return self.free.pop()
        if self.evictable:
            hsh, blk = self.evictable.popitem(last=False)
            del self.by_hash[hsh]
            del self.hash_of[blk]
            return blk
        raise MemoryError("KV cache out of blocks")

    def allocate(self, n: int) -> list:
        if n > self.num_free:
            raise MemoryError(f"need {n} KV blocks, {self.num_free} free")
        out = []
        for _ in range(n):
            b = self._take()
            self.ref[b] = 1
            out.append(b)
        return out

    def release(self, blocks) -> None:
        for b in blocks:
            self.ref[b] -= 1
            assert self.ref[b] >= 0
            if self.ref[b] == 0:
                h = self.hash_of.get(b)
                if h is not None and self.prefix:
                    self.evictable[h] = b
                else:
                    self.hash_of.pop(b, None)
                    self.free.append(b)

    def match_prefix(self, tokens) -> tuple:
        """Longest run of cached full blocks that starts ``tokens``: (blocks, hashes)."""
        if not self.prefix:
            return [], []
        blocks, hashes, prev = [], [], b""
        for i in range(len(tokens) // BLOCK):
            hsh = _block_hash(prev, tokens[i * BLOCK:(i + 1) * BLOCK])
            b = self.by_hash.get(hsh)
            if b is None:
                break
            blocks.append(b)
            hashes.append(hsh)
            prev = hsh
        for hsh, b in zip(hashes, blocks):
            if self.ref[b] == 0:
                self.evictable.pop(hsh, None)
            self.ref[b] += 1
        return blocks, hashes

    def register(self, blocks, tokens, start_block: int = 0, prev_hash: bytes = b"") -> bytes:
        """Index the full blocks of a sequence (blocks[i] holds tokens[16i:16i+16])."""
        if not self.prefix:
            return prev_hash
        prev = prev_hash
        for i in range(start_block, len(tokens) // BLOCK):
            hsh = _block_hash(prev, tokens[i * BLOCK:(i + 1) * BLOCK])
            b = blocks[i]
            if hsh not in self.by_hash and b not in self.hash_of:
                self.by_hash[hsh] = b
                self.hash_of[b] = hsh
            prev = hsh
        return prev
