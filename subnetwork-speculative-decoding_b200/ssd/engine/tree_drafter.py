"""Tree drafting with the sub-network draft (API of ssd/engine/tree_drafter.py).

Each round: feed the pending root; for depth d = 1..K every node kept at
depth d-1 proposes ``branch[d]`` children (greedy: top tokens; sampling:
Gumbel top-k without replacement), the ``width[d]`` children with the best
cumulative draft log-prob are kept, and (unless d == K) the level goes
through the draft in one batched forward where each node attends to the
committed prefix and its own ancestors. The best ``max_nodes`` nodes form the
verified tree (ancestor-closed).

``TreeDrafter.build`` runs that on the device (ssd/engine/round.py: one
top-k head launch and one prune kernel per level) and returns the tree as a
host ``DraftTree``; the generator uses the same kernels without reading the
tree back.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch

from ssd.config import DraftingConfig
from ssd.engine.kv_cache import KVCache
from ssd.models.subnetwork_draft import SubnetworkDraftModel

ROOT = -1


def warp_probs(logits: torch.Tensor, temperature: float, top_p: float) -> torch.Tensor:
    """Temperature + nucleus filtering -> fp32 probabilities (tree_drafter.py:
    34-45), on the device kernel."""
    from ssd.engine.sampling import warp_probs_device

    return warp_probs_device(logits, temperature, top_p)


@dataclass
class DraftTree:
    tokens: list[int] = field(default_factory=list)
    parents: list[int] = field(default_factory=list)  # ROOT (-1) or node index
    depths: list[int] = field(default_factory=list)  # 1..K
    scores: list[float] = field(default_factory=list)  # cumulative draft log-prob
    ranks: list[int] = field(default_factory=list)  # proposal order among siblings
    draft_pos: list[int] = field(default_factory=list)  # draft-cache slot, -1 if never fed
    child_q: dict[int, torch.Tensor] = field(default_factory=dict)
    cache_start: int = 0

    def __len__(self) -> int:
        return len(self.tokens)

    def children(self) -> dict[int, list[int]]:
        """parent -> child node indices in proposal order (tree_drafter.py:63-70)."""
        out: dict[int, list[int]] = {}
        for i, p in enumerate(self.parents):
            out.setdefault(p, []).append(i)
        for kids in out.values():
            kids.sort(key=lambda i: self.ranks[i])
        return out

    def ancestors(self, i: int) -> list[int]:
        path = []
        while i != ROOT:
            path.append(i)
            i = self.parents[i]
        return path[::-1]

    def subset(self, keep: list[int]) -> "DraftTree":
        keep = sorted(keep)
        remap = {old: new for new, old in enumerate(keep)}
        remap[ROOT] = ROOT
        t = DraftTree(cache_start=self.cache_start)
        for old in keep:
            t.tokens.append(self.tokens[old])
            t.parents.append(remap[self.parents[old]])
            t.depths.append(self.depths[old])
            t.scores.append(self.scores[old])
            t.ranks.append(self.ranks[old])
            t.draft_pos.append(self.draft_pos[old])
        for p, q in self.child_q.items():
            if p in remap:
                t.child_q[remap[p]] = q
        return t


class TreeDrafter:
    def __init__(self, draft: SubnetworkDraftModel, cfg: DraftingConfig):
        cfg.validate()
        self.draft = draft
        self.cfg = cfg
        self.branch = cfg.per_depth(cfg.branch, "branch")
        self.width = cfg.per_depth(cfg.width, "width")
        self.greedy = cfg.temperature == 0
        self._engine = None

    def max_nodes_per_level(self) -> list[int]:
        n, out = 1, []
        for d in range(self.cfg.depth):
            n *= self.branch[d]
            if self.width[d] is not None:
                n = min(n, self.width[d])
            out.append(n)
        return out

    def max_tree_cache(self) -> int:
        """Draft-cache slots one round's tree uses (the last level is never fed)."""
        return sum(self.max_nodes_per_level()[:-1])

    def max_verify_nodes(self) -> int:
        total = sum(self.max_nodes_per_level())
        return min(total, self.cfg.max_nodes) if self.cfg.max_nodes else total

    @torch.no_grad()
    def build(self, cache: KVCache, pending: torch.Tensor, root_pos: int,
              generator: Optional[torch.Generator] = None) -> DraftTree:
        """``pending``: [1, n] committed tokens not yet in ``cache``; the last
        one is the root at absolute position ``root_pos`` (tree_drafter.py:147-208)."""
        if not self.greedy:
            from ssd.engine.sampling import sampled_tree_build

            return sampled_tree_build(self, cache, pending, root_pos, generator)
        from ssd.engine.round import GreedyRound, ROOT_TOK, SEQ

        draft = self.draft
        w = draft.weights
        pend = pending.reshape(-1)
        n_pend = int(pend.numel())
        if cache.get_seq_length() != root_pos - n_pend + 1:
            raise ValueError("pending tokens must directly follow the cache contents")
        if n_pend > 1:  # feed the earlier pending tokens as an ordinary causal chunk
            draft(pend[:-1].reshape(1, -1), position_ids=torch.arange(root_pos - n_pend + 1, root_pos).reshape(1, -1),
                  past_key_values=cache, compute_logits=False)
        cache.allocate(w.Hkv, w.hd, w.dtype, w.device)
        eng = self._engine
        if eng is None or eng.cache is not cache:
            eng = GreedyRound(draft, draft, self.cfg, cache, max_new=1)
            self._engine = eng
        eng.state[SEQ] = root_pos
        eng.state[ROOT_TOK] = int(pend[-1])
        eng.draft_phase()
        t = eng.read_tree()
        eng.ws.check_status()
        tree = DraftTree(tokens=t["tokens"], parents=t["parents"], depths=t["depths"], scores=t["scores"],
                         ranks=t["ranks"], draft_pos=t["draft_pos"], cache_start=root_pos + 1)
        cache.seq_len = root_pos + 1 + eng.plan.max_tree_cache
        return tree
