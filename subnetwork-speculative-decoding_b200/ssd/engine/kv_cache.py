"""The shared target/draft KV cache (API of ssd/engine/kv_cache.py:21-73).

One device buffer ``[num_slots, 2, n_kv_heads, max_length, head_dim]`` (slot =
base layer index), so a layer's K (or V) for one KV head is a contiguous
``[max_length, head_dim]`` run: tree attention streams it, the fused QKV
epilogue writes new rows straight into it, and KV compaction gathers every
layer in one launch. The buffer is allocated on the first write (or by
``allocate``), on the device and in the dtype of the model using it.

Write protocol, as in the reference: a forward over q new tokens writes
positions [len, len + q) of every layer it runs, then ``advance(q)``.
"""

from __future__ import annotations

from typing import Optional, Sequence, Union

import torch


class KVCache:
    def __init__(self, num_slots: int, max_length: int):
        self.num_slots = num_slots
        self.max_length = max_length
        self.seq_len = 0
        self.buf: Optional[torch.Tensor] = None

    # ------------------------------------------------------------ storage
    def allocate(self, n_kv_heads: int, head_dim: int, dtype: torch.dtype, device) -> torch.Tensor:
        if self.buf is None:
            self.buf = torch.zeros(self.num_slots, 2, n_kv_heads, self.max_length, head_dim, dtype=dtype,
                                   device=device)
        elif self.buf.shape[2:] != (n_kv_heads, self.max_length, head_dim) or self.buf.dtype != dtype:
            raise ValueError("KVCache already holds a cache of another shape/dtype")
        return self.buf

    def layer(self, slot: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(k, v) of one base layer, each [n_kv, max_length, head_dim]."""
        return self.buf[slot, 0], self.buf[slot, 1]

    @property
    def k(self) -> list:
        """Per-slot [1, n_kv, max_length, head_dim] key buffers (reference layout)."""
        return [None if self.buf is None else self.buf[s, 0].unsqueeze(0) for s in range(self.num_slots)]

    @property
    def v(self) -> list:
        return [None if self.buf is None else self.buf[s, 1].unsqueeze(0) for s in range(self.num_slots)]

    # ------------------------------------------------------------ protocol
    def get_seq_length(self) -> int:
        return self.seq_len

    def check_room(self, q_len: int) -> None:
        end = self.seq_len + q_len
        if end > self.max_length:
            raise RuntimeError(f"KVCache overflow: {end} > max_length={self.max_length}")

    def update(self, slot: int, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Write k/v [1, n_kv, q, head_dim] at [len, len + q) and return the
        [1, n_kv, len + q, head_dim] views (kv_cache.py:32-43). The model's own
        forward never calls this: its QKV kernel writes the cache directly."""
        bsz, n_kv, q_len, hd = k.shape
        if bsz != 1:
            raise ValueError("the B200 KV cache holds batch size 1")
        self.check_room(q_len)
        self.allocate(n_kv, hd, k.dtype, k.device)
        end = self.seq_len + q_len
        self.buf[slot, 0, :, self.seq_len:end] = k[0]
        self.buf[slot, 1, :, self.seq_len:end] = v[0]
        return self.buf[slot, 0, :, :end].unsqueeze(0), self.buf[slot, 1, :, :end].unsqueeze(0)

    def advance(self, n: int) -> None:
        self.seq_len += n

    def crop(self, length: int) -> None:
        """Discard everything at positions >= length (kv_cache.py:48-52)."""
        if length > self.seq_len:
            raise ValueError(f"cannot crop to {length} > current length {self.seq_len}")
        self.seq_len = length

    def keep_positions(self, start: int, positions: Union[torch.Tensor, Sequence[int]]) -> None:
        """Move cache entries ``positions`` (absolute, >= start) to [start,
        start + n) in every layer: one in-place compaction kernel
        (kv_cache.py:54-70)."""
        pos = positions.tolist() if isinstance(positions, torch.Tensor) else list(positions)
        n = len(pos)
        if n == 0 or pos == list(range(start, start + n)) or self.buf is None:
            self.seq_len = start + n
            return
        if any(p < start or p >= self.max_length for p in pos):
            raise ValueError("keep_positions: positions must lie in [start, max_length)")
        from ssd import ops

        dev = self.buf.device
        slots = torch.tensor(pos, dtype=torch.int32, device=dev)
        meta = torch.tensor([start, n], dtype=torch.int32, device=dev)
        ops.kv_compact(self.buf, meta[0:1], slots, meta[1:2], max_keep=max(1, n))
        self.seq_len = start + n

    def reset(self) -> None:
        self.seq_len = 0
