"""Paged bf16 KV cache: the ``past_key_values`` object of the decode path.

The reference keeps one contiguous [1, 8, S_MAX=1024, 64] cache per layer in
NxDI's KV manager, a flat list [K0, V0, K1, V1, ...] that its kernel updates in
place (llama_with_megakernel.py:134-139, nki_kernels/attention.py:450-492).
Here the cache is paged so context length is bounded by the pool, not by a
per-sequence S_MAX:

* ``k_pages`` / ``v_pages``: [num_layers, num_pages, num_kv_heads, page_size,
  head_dim] bf16. One page holds ``page_size`` consecutive positions of one
  sequence for every kv head; a head's rows in a page are contiguous, so the
  kernel fetches them with a single bulk copy.
* ``block_tables``: [max_batch, max_blocks] int32, logical block -> page id,
  shared by all layers. Position p of sequence b is slot p % page_size of
  page ``block_tables[b, p // page_size]``.

The kernel writes each new K/V row in place at its position and reads
positions [0, pos) for attention.
"""
from __future__ import annotations

import torch

from .config import LlamaDecodeConfig


class PagedKVCache:
    def __init__(self, cfg: LlamaDecodeConfig, max_batch: int, max_seq_len: int,
                 page_size: int = 64, num_pages: int | None = None, device="cuda"):
        if page_size % 8:
            raise ValueError("page_size must be a multiple of 8")
        self.cfg = cfg
        self.page_size = page_size
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.max_blocks = (max_seq_len + page_size - 1) // page_size
        if num_pages is None:
            num_pages = max_batch * self.max_blocks
        self.num_pages = num_pages
        self.device = torch.device(device)
        shape = (cfg.num_layers, num_pages, cfg.num_kv_heads, page_size, cfg.head_dim)
        self.k_pages = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v_pages = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.block_tables = torch.full((max_batch, self.max_blocks), -1, dtype=torch.int32,
                                       device=self.device)
        self._host_tables = [[] for _ in range(max_batch)]
        self._free = list(range(num_pages - 1, -1, -1))
        self.seq_lens = [0] * max_batch

    # ------------------------------------------------------------ allocation
    def reserve(self, seq: int, length: int) -> None:
        """Make positions [0, length) of sequence ``seq`` addressable."""
        if length > self.max_blocks * self.page_size:
            raise ValueError(f"length {length} exceeds max_seq_len {self.max_seq_len}")
        need = (length + self.page_size - 1) // self.page_size
        table = self._host_tables[seq]
        changed = False
        while len(table) < need:
            if not self._free:
                raise RuntimeError("KV page pool exhausted")
            table.append(self._free.pop())
            changed = True
        if changed:
            row = torch.tensor(table + [-1] * (self.max_blocks - len(table)), dtype=torch.int32)
            self.block_tables[seq].copy_(row.to(self.device))

    def shuffle_free_pages(self, seed: int) -> None:
        """Hand out free pages in a seeded random order (exercises the page indirection)."""
        g = torch.Generator().manual_seed(seed)
        order = torch.randperm(len(self._free), generator=g).tolist()
        self._free = [self._free[i] for i in order]

    def release(self, seq: int) -> None:
        self._free.extend(reversed(self._host_tables[seq]))
        self._host_tables[seq] = []
        self.seq_lens[seq] = 0
        self.block_tables[seq].fill_(-1)

    def reset(self) -> None:
        for b in range(self.max_batch):
            self.release(b)

    def pages_of(self, seq: int) -> list[int]:
        return list(self._host_tables[seq])

    # ------------------------------------------------------------ contents
    def fill(self, seq: int, k_rows: torch.Tensor, v_rows: torch.Tensor) -> None:
        """Write positions [0, n) of ``seq`` from [num_layers, nkv, n, head_dim] tensors."""
        n = k_rows.shape[2]
        self.reserve(seq, n)
        ps = self.page_size
        table = self._host_tables[seq]
        for blk in range((n + ps - 1) // ps):
            p0, p1 = blk * ps, min(n, (blk + 1) * ps)
            page = table[blk]
            self.k_pages[:, page, :, : p1 - p0] = k_rows[:, :, p0:p1].to(self.device)
            self.v_pages[:, page, :, : p1 - p0] = v_rows[:, :, p0:p1].to(self.device)
        self.seq_lens[seq] = max(self.seq_lens[seq], n)

    def gather(self, seq: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Rows [0, n) of ``seq`` as [num_layers, nkv, n, head_dim] (contiguous copy)."""
        ps = self.page_size
        nb = (n + ps - 1) // ps
        pages = torch.tensor(self._host_tables[seq][:nb], dtype=torch.long, device=self.device)
        L, _, nkv, _, hd = self.k_pages.shape
        k = self.k_pages[:, pages].permute(0, 2, 1, 3, 4).reshape(L, nkv, nb * ps, hd)[:, :, :n]
        v = self.v_pages[:, pages].permute(0, 2, 1, 3, 4).reshape(L, nkv, nb * ps, hd)[:, :, :n]
        return k.contiguous(), v.contiguous()

    def nbytes(self) -> int:
        return 2 * self.k_pages.numel() * 2
