"""Tree drafting and verification restated for the oracle (plain Python).

Follows ssd/engine/tree_drafter.py (warp_probs :34-45, DraftTree :48-95,
TreeDrafter :98-208) and ssd/engine/verify.py (verify_inputs :32-42,
greedy_verify :45-57, sample_verify :60-95), and ssd/data/token_freq.py
(top_vocab :49-55). Random draws use a torch CPU generator with the same
calls as the reference so a seeded run consumes the same random stream.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from oracle.model import plan_bridges  # noqa: F401  (re-exported)

ROOT = -1


def log_softmax(x: np.ndarray) -> np.ndarray:
    m = x.max(axis=-1, keepdims=True)
    return x - m - np.log(np.exp(x - m).sum(axis=-1, keepdims=True))


def warp_probs(logits: np.ndarray, temperature: float, top_p: float) -> np.ndarray:
    """tree_drafter.py:34-45: softmax(logits / T), then nucleus filtering
    (keep the smallest prefix of the descending order with mass >= top_p)."""
    z = logits.astype(np.float64) / temperature
    z = z - z.max(axis=-1, keepdims=True)
    p = np.exp(z)
    p /= p.sum(axis=-1, keepdims=True)
    if top_p < 1.0:
        order = np.argsort(-p, axis=-1, kind="stable")
        sp = np.take_along_axis(p, order, -1)
        cum = np.cumsum(sp, axis=-1)
        sp = np.where(cum - sp > top_p, 0.0, sp)
        out = np.zeros_like(p)
        np.put_along_axis(out, order, sp, -1)
        p = out / out.sum(axis=-1, keepdims=True)
    return p


def top_k_warp(logits: np.ndarray, k: int, temperature: float, top_p: float) -> np.ndarray:
    """The distribution sample_next draws from at temperature > 0
    (ssd/data/generate_selfdistill.py:51-61): the k largest logits of the row,
    warp_probs over them, zero elsewhere. 1-D rows."""
    x = np.asarray(logits, dtype=np.float64)
    idx = np.argsort(-x, kind="stable")[:k]
    out = np.zeros_like(x)
    out[idx] = warp_probs(x[idx], temperature, top_p)
    return out


@dataclass
class DraftTree:
    """DraftTree (tree_drafter.py:48-95)."""

    tokens: list = field(default_factory=list)
    parents: list = field(default_factory=list)
    depths: list = field(default_factory=list)
    scores: list = field(default_factory=list)
    ranks: list = field(default_factory=list)
    draft_pos: list = field(default_factory=list)
    child_q: dict = field(default_factory=dict)
    cache_start: int = 0

    def __len__(self) -> int:
        return len(self.tokens)

    def children(self) -> dict:
        out: dict = {}
        for i, p in enumerate(self.parents):
            out.setdefault(p, []).append(i)
        for kids in out.values():
            kids.sort(key=lambda i: self.ranks[i])
        return out

    def ancestors(self, i: int) -> list:
        path = []
        while i != ROOT:
            path.append(i)
            i = self.parents[i]
        return path[::-1]

    def subset(self, keep) -> "DraftTree":
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


def per_depth(value, depth: int, name: str) -> list:
    """DraftingConfig.per_depth (ssd/config.py:111-116)."""
    if value is None or isinstance(value, int):
        return [value] * depth
    if len(value) != depth:
        raise ValueError(f"drafting.{name} has {len(value)} entries but depth={depth}")
    return list(value)


class OracleTreeDrafter:
    """TreeDrafter (tree_drafter.py:98-208) over an OracleModel draft."""

    def __init__(self, draft, depth: int, branch, width=None, max_nodes=None, temperature: float = 0.0,
                 top_p: float = 1.0):
        self.draft = draft
        self.depth = depth
        self.branch = per_depth(branch, depth, "branch")
        self.width = per_depth(width, depth, "width")
        self.max_nodes = max_nodes
        self.temperature = temperature
        self.top_p = top_p
        self.greedy = temperature == 0

    def max_nodes_per_level(self) -> list:
        n, out = 1, []
        for d in range(self.depth):
            n *= self.branch[d]
            if self.width[d] is not None:
                n = min(n, self.width[d])
            out.append(n)
        return out

    def max_tree_cache(self) -> int:
        return sum(self.max_nodes_per_level()[:-1])

    def max_verify_nodes(self) -> int:
        total = sum(self.max_nodes_per_level())
        return min(total, self.max_nodes) if self.max_nodes else total

    def propose(self, logits: np.ndarray, k: int, generator):
        """_propose (tree_drafter.py:124-145)."""
        import torch

        vocab_ids = self.draft.vocab_ids
        if self.greedy:
            lp = log_softmax(logits.astype(np.float64))
            out = []
            for row in lp:
                order = np.argsort(-row, kind="stable")[:k]
                toks = order if vocab_ids is None else vocab_ids[order]
                out.append(([int(t) for t in toks], [float(row[i]) for i in order], None))
            return out
        probs = warp_probs(logits, self.temperature, self.top_p)
        if vocab_ids is not None:
            full = np.zeros((probs.shape[0], self.draft.conf["vocab"]))
            full[:, vocab_ids] = probs
            probs = full
        out = []
        for q in probs:
            qt = torch.from_numpy(q.astype(np.float32))
            support = int((qt > 0).sum())
            gumbel = -torch.empty_like(qt).exponential_(generator=generator).log()
            keys = qt.log() + gumbel
            tok = keys.topk(min(k, support)).indices
            out.append((tok.tolist(), qt[tok].log().tolist(), qt))
        return out

    def build(self, cache, pending: list, root_pos: int, generator=None) -> DraftTree:
        """TreeDrafter.build (tree_drafter.py:147-208)."""
        n_pend = len(pending)
        pos = np.arange(root_pos - n_pend + 1, root_pos + 1)
        logits = self.draft.forward(pending, pos, cache, logits_to_keep=1)
        tree_start = cache.get_seq_length()
        tree = DraftTree(cache_start=tree_start)
        frontier, frontier_logits = [ROOT], logits[-1:]
        for d in range(self.depth):
            cands = []
            for parent, (toks, lps, q) in zip(frontier, self.propose(frontier_logits, self.branch[d], generator)):
                if q is not None:
                    tree.child_q[parent] = q
                base = tree.scores[parent] if parent != ROOT else 0.0
                cands += [(base + lp, parent, t, r) for r, (t, lp) in enumerate(zip(toks, lps))]
            cands.sort(key=lambda c: -c[0])
            if self.width[d] is not None:
                cands = cands[: self.width[d]]
            level = []
            for score, parent, tok, rank in cands:
                level.append(len(tree))
                tree.tokens.append(tok)
                tree.parents.append(parent)
                tree.depths.append(d + 1)
                tree.scores.append(score)
                tree.ranks.append(rank)
                tree.draft_pos.append(-1)
            if d == self.depth - 1 or not level:
                break
            past = cache.get_seq_length()
            for j, i in enumerate(level):
                tree.draft_pos[i] = past + j
            mask = np.zeros((len(level), past + len(level)), dtype=bool)
            mask[:, :tree_start] = True
            for j, i in enumerate(level):
                for a in tree.ancestors(i):
                    mask[j, tree.draft_pos[a]] = True
            ids = [tree.tokens[i] for i in level]
            pos = np.full(len(level), root_pos + d + 1)
            frontier = level
            frontier_logits = self.draft.forward(ids, pos, cache, tree_mask=mask)
        if self.max_nodes is not None and len(tree) > self.max_nodes:
            order = sorted(range(len(tree)), key=lambda i: (-tree.scores[i], tree.depths[i]))
            keep = set(order[: self.max_nodes])
            for i in list(keep):
                keep.update(tree.ancestors(i))
            tree = tree.subset(sorted(keep))
        return tree


def verify_inputs(tree: DraftTree, root_token: int, root_pos: int, past_len: int):
    """verify.py:32-42 -> (ids [n+1], positions [n+1], bool mask [n+1, past+n+1])."""
    n = len(tree)
    ids = [root_token] + list(tree.tokens)
    pos = [root_pos] + [root_pos + d for d in tree.depths]
    mask = np.zeros((n + 1, past_len + n + 1), dtype=bool)
    mask[:, : past_len + 1] = True
    for i in range(n):
        for a in tree.ancestors(i):
            mask[i + 1, past_len + 1 + a] = True
    return ids, pos, mask


def greedy_verify(tree: DraftTree, target_logits: np.ndarray):
    """verify.py:45-57 (argmax = first index of the maximum)."""
    argmax = [int(np.argmax(r)) for r in target_logits]
    kids = tree.children()
    accepted, cur = [], ROOT
    while True:
        want = argmax[cur + 1]
        nxt = next((c for c in kids.get(cur, []) if tree.tokens[c] == want), None)
        if nxt is None:
            return accepted, want
        accepted.append(nxt)
        cur = nxt


def sample_verify(tree: DraftTree, target_logits: np.ndarray, temperature: float, top_p: float, generator=None):
    """verify.py:60-95: multi-candidate speculative sampling without replacement."""
    import torch

    kids = tree.children()
    accepted, cur = [], ROOT
    while True:
        p = torch.from_numpy(warp_probs(target_logits[cur + 1], temperature, top_p).astype(np.float32))
        children = kids.get(cur, [])
        if children:
            q = tree.child_q[cur].clone()
            chosen = None
            for c in children:
                x = tree.tokens[c]
                if q[x] <= 0:
                    continue
                if torch.rand((), generator=generator).item() < min(1.0, (p[x] / q[x]).item()):
                    chosen = c
                    break
                residual = (p - q).clamp_min(0)
                if residual.sum() > 0:
                    p = residual / residual.sum()
                q[x] = 0
                if q.sum() <= 0:
                    break
                q = q / q.sum()
            if chosen is not None:
                accepted.append(chosen)
                cur = chosen
                continue
        bonus = torch.multinomial(p, 1, generator=generator).item()
        return accepted, bonus


def top_vocab(counts: np.ndarray, size: int, always=frozenset()) -> np.ndarray:
    """token_freq.py:49-55: the `size` most frequent ids (stable descending
    order, forced ids first), sorted ascending."""
    counts = np.asarray(counts)
    order = np.argsort(-counts, kind="stable")
    forced = [t for t in always if 0 <= t < counts.shape[0]]
    rest = order[~np.isin(order, forced)][: max(0, size - len(forced))]
    return np.sort(np.concatenate([np.asarray(forced, dtype=np.int64), rest.astype(np.int64)]))


def first_token(logits: np.ndarray, temperature: float, top_p: float, generator) -> int:
    """speculative.py:81-84."""
    if temperature == 0:
        return int(np.argmax(logits))
    import torch

    p = torch.from_numpy(warp_probs(logits, temperature, top_p).astype(np.float32))
    return int(torch.multinomial(p, 1, generator=generator))


def finish(tokens: list, eos_ids, max_new: int):
    """speculative.py:87-91."""
    for i, t in enumerate(tokens[:max_new]):
        if t in eos_ids:
            return tokens[: i + 1], True
    return tokens[:max_new], len(tokens) >= max_new
