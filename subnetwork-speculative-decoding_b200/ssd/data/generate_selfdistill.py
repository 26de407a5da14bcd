"""Batched continuation of prompts (API of generate_batch,
ssd/data/generate_selfdistill.py:64-108 in the reference).

The reference decodes a left-padded batch with one masked forward per step.
Here every row runs through the device-resident decode engine of its own
(the cached kernels serve one sequence at a time): with padding masked out and
positions counted from each row's first real token, a row's continuation in
the padded batch is the continuation of the row alone, so greedy decoding
(temperature 0) returns the same tokens. With temperature > 0 each row draws
from the nucleus of the full vocabulary with a counter-based generator seeded
per row from `generator` (the reference first cuts the logits to their 64
largest values, then applies the nucleus; the draws are not the same stream).
"""

from __future__ import annotations

from typing import Optional

import torch

from ssd.engine.speculative import TargetRunner, autoregressive_generate


@torch.no_grad()
def generate_batch(target: TargetRunner, prompts: list[list[int]], max_new_tokens: int, eos_ids: set[int],
                   temperature: float, top_p: float, pad_id: int,
                   generator: Optional[torch.Generator] = None) -> list[list[int]]:
    """New tokens per row, cut after the first EOS (inclusive). pad_id is
    accepted for the reference's signature; rows are never padded here."""
    if not prompts:
        return []
    if any(len(p) == 0 for p in prompts):
        raise ValueError("generate_batch: empty prompt")
    if max_new_tokens <= 0:
        return [[] for _ in prompts]
    rows = []
    for p in prompts:
        seed = None
        if temperature > 0:
            g = generator if generator is not None else torch.Generator().manual_seed(0)
            seed = int(torch.randint(0, 2 ** 62, (1,), generator=g).item())
        res = autoregressive_generate(target, torch.tensor([p], dtype=torch.long), max_new_tokens, eos_ids,
                                      temperature=temperature, top_p=top_p, seed=seed)
        out = res.tokens[:max_new_tokens]
        cut = next((i + 1 for i, t in enumerate(out) if t in eos_ids), len(out))
        rows.append(out[:cut])
    return rows
