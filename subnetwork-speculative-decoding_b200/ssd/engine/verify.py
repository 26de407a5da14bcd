"""Tree verification (API of ssd/engine/verify.py).

The target scores ``[root] + tree nodes`` in one forward; each node attends
to the committed prefix, the root and its own ancestors. From the root:

* greedy: move to the child whose token equals the target's argmax; the
  argmax at the first mismatch is the bonus token (output identical to
  greedy decoding with the target alone);
* sampling: multi-candidate speculative sampling without replacement
  (accept child x with prob min(1, p(x)/q(x)); on rejection p <- norm(max(p -
  q, 0)), q <- q without x; bonus ~ p when every child is rejected).

These functions take a host ``DraftTree`` and logits, as in the reference.
The generator itself never materialises logits: its verify head fuses the
lm_head with the argmax and walks the tree on the device.
"""

from __future__ import annotations

from typing import Optional

import torch

from ssd.engine.tree_drafter import ROOT, DraftTree


def verify_inputs(tree: DraftTree, root_token: int, root_pos: int, past_len: int, device) -> tuple:
    """ids [1, n+1], positions [1, n+1], bool mask [n+1, past+n+1]; row 0 is the
    root (verify.py:32-42)."""
    n = len(tree)
    ids = torch.tensor([[root_token] + tree.tokens], device=device)
    pos = torch.tensor([[root_pos] + [root_pos + d for d in tree.depths]], device=device)
    mask = torch.zeros(n + 1, past_len + n + 1, dtype=torch.bool)
    mask[:, : past_len + 1] = True
    for i in range(n):
        for a in tree.ancestors(i):
            mask[i + 1, past_len + 1 + a] = True
    return ids, pos, mask.to(device)


def greedy_verify(tree: DraftTree, target_logits: torch.Tensor) -> tuple[list[int], int]:
    """target_logits [n+1, V] (row 0 = root) -> (accepted node indices, bonus)
    (verify.py:45-57)."""
    argmax = target_logits.argmax(-1).tolist()
    kids = tree.children()
    accepted: list[int] = []
    cur = ROOT
    while True:
        want = argmax[cur + 1]
        nxt = next((c for c in kids.get(cur, []) if tree.tokens[c] == want), None)
        if nxt is None:
            return accepted, want
        accepted.append(nxt)
        cur = nxt


def sample_verify(tree: DraftTree, target_logits: torch.Tensor, temperature: float, top_p: float,
                  generator: Optional[torch.Generator] = None) -> tuple[list[int], int]:
    """Multi-candidate speculative sampling without replacement (verify.py:60-95)
    on the device sampling kernels."""
    from ssd.engine.sampling import sample_verify_device

    return sample_verify_device(tree, target_logits, temperature, top_p, generator)
