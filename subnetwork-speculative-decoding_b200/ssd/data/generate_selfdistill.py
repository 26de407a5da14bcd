"""Batched continuation of prompts (API of generate_batch,
ssd/data/generate_selfdistill.py:64-108 in the reference) on the batched
device decoder (ssd.engine.batch.BatchDecoder): one forward per step over all
rows, each sequence in its own cache slot range, so a row's continuation is
the same as in the reference's left-padded, masked batch (positions count
from each row's first real token). Greedy rows (temperature 0) therefore
equal the reference's; sampled rows draw from the 64 largest logits under
temperature and top_p as the reference's sample_next (:51-61) does, with a
counter-based generator keyed by one draw from `generator` (the reference's
torch.Generator stream cannot be reproduced).
"""

from __future__ import annotations

from typing import Optional

import torch

from ssd.engine.batch import BatchDecoder
from ssd.engine.speculative import TargetRunner

SAMPLE_TOP_K = 64  # sample_next's cut (generate_selfdistill.py:55-58)


@torch.no_grad()
def generate_batch(target: TargetRunner, prompts: list[list[int]], max_new_tokens: int, eos_ids: set[int],
                   temperature: float, top_p: float, pad_id: int,
                   generator: Optional[torch.Generator] = None) -> list[list[int]]:
    """New tokens per row, cut after the first EOS (inclusive). pad_id is
    accepted for the reference's signature; no row is padded here."""
    if not prompts:
        return []
    if any(len(p) == 0 for p in prompts):
        raise ValueError("generate_batch: empty prompt")
    if max_new_tokens <= 0:
        return [[] for _ in prompts]
    seed = None
    if temperature > 0:
        g = generator if generator is not None else torch.Generator().manual_seed(0)
        seed = int(torch.randint(0, 2 ** 62, (1,), generator=g).item())
    region = -(-(max(len(p) for p in prompts) + max_new_tokens + 1) // 64) * 64
    rows = sum(len(p) for p in prompts)
    dec = BatchDecoder(target, len(prompts), region, rows)
    out = dec.generate([list(map(int, p)) for p in prompts], max_new_tokens, set(eos_ids), temperature, top_p,
                       SAMPLE_TOP_K, seed)
    res = []
    for r in out:
        r = r[:max_new_tokens]
        cut = next((i + 1 for i, t in enumerate(r) if t in eos_ids), len(r))
        res.append(r[:cut])
    return res
