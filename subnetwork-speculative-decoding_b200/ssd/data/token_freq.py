"""Draft-vocabulary selection (API of ssd/data/token_freq.py).

``top_vocab`` picks the ``size`` most frequent token ids (ties in stable
descending-count order, ids in ``always`` forced in) sorted ascending
(token_freq.py:49-55). Counting frequencies over a dataset is part of the
reference's training pipeline and not of this package; counts come from a
``token_freq.pt`` file or from ssd.synthetic.zipf_counts.
"""

from __future__ import annotations

from pathlib import Path

import torch


def token_freq_path(cfg) -> Path:
    return Path(cfg.training.output_dir) / "token_freq.pt"


def top_vocab(counts: torch.Tensor, size: int, always: set[int] = frozenset()) -> torch.Tensor:
    """The ``size`` most frequent token ids (always including ``always``), sorted ascending."""
    order = counts.argsort(descending=True, stable=True)
    forced = [t for t in always if 0 <= t < counts.numel()]
    keep = torch.tensor(forced, dtype=torch.long)
    rest = order[~torch.isin(order, keep)][: max(0, size - len(forced))]
    return torch.cat([keep, rest]).sort().values
