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
    root (verify.py:32-42).

    Every row sees the committed prefix and the root. Nodes are stored parents
    first, so a node's row is built from its parent's row plus its own column
    (one pass over the nodes instead of one ancestor walk per node)."""
    n = len(tree)
    ids = torch.tensor([[root_token, *tree.tokens]], device=device)
    pos = (root_pos + torch.tensor([0, *tree.depths])).unsqueeze(0).to(device)
    tree_cols = torch.zeros(n + 1, n + 1, dtype=torch.bool)
    tree_cols[:, 0] = True
    for node, parent in enumerate(tree.parents):
        if parent != ROOT and parent >= node:
            raise ValueError(f"verify_inputs: node {node} precedes its parent {parent}")
        tree_cols[node + 1] = tree_cols[parent + 1]  # ROOT (-1) -> the root's row
        tree_cols[node + 1, node + 1] = True
    mask = torch.cat([torch.ones(n + 1, past_len, dtype=torch.bool), tree_cols], dim=1)
    return ids, pos, mask.to(device)


def greedy_verify(tree: DraftTree, target_logits: torch.Tensor) -> tuple[list[int], int]:
    """target_logits [n+1, V] (row 0 = root) -> (accepted node indices, bonus)
    (verify.py:45-57). Each row's first maximum (torch.argmax's tie rule, as
    the reference) feeds the device tree walk (ssd_tree_walk_greedy), the
    kernel the speculative round runs."""
    from ssd import ops
    from ssd.engine.round import DeviceTree

    if not target_logits.is_cuda:
        raise ValueError("greedy_verify: target_logits must be a CUDA tensor (the B200 path has no CPU fallback)")
    dev = target_logits.device
    n = len(tree)
    dt = DeviceTree(max(n, 1), dev)
    i32 = dict(dtype=torch.int32, device=dev)
    if n:
        dt.tokens[:n] = torch.tensor(tree.tokens, **i32)
        dt.parents[:n] = torch.tensor(tree.parents, **i32)
        dt.ranks[:n] = torch.tensor(tree.ranks, **i32)
    dt.n_nodes.fill_(n)
    best = target_logits.argmax(-1).to(torch.int32)
    accepted, keep = torch.zeros(n + 1, **i32), torch.zeros(n + 2, **i32)
    out = torch.zeros(4, **i32)  # n_accepted, bonus, n_keep, root position (0: only the walk is used)
    ops.tree_walk_greedy(dt, best, out[3:4], accepted, out[0:1], out[1:2], keep, out[2:3], max(n, 1))
    na, bonus = out[:2].tolist()
    return accepted[:na].tolist(), int(bonus)


def sample_verify(tree: DraftTree, target_logits: torch.Tensor, temperature: float, top_p: float,
                  generator: Optional[torch.Generator] = None) -> tuple[list[int], int]:
    """Multi-candidate speculative sampling without replacement (verify.py:60-95)
    on the device sampling kernels."""
    from ssd.engine.sampling import sample_verify_device

    return sample_verify_device(tree, target_logits, temperature, top_p, generator)
