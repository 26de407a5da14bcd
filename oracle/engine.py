"""Round loop and autoregressive baseline restated for the oracle.

Follows ssd/engine/speculative.py (autoregressive_generate :101-122,
SpeculativeGenerator.generate :132-174).
"""

from __future__ import annotations

from typing import Optional

import numpy as np

from oracle.tree import OracleTreeDrafter, finish, first_token, greedy_verify, sample_verify, verify_inputs


def _gen(seed):
    if seed is None:
        return None
    import torch

    return torch.Generator().manual_seed(seed)


def autoregressive_generate(target, ids, max_new_tokens: int, eos_ids=frozenset(), temperature: float = 0.0,
                            top_p: float = 1.0, seed: Optional[int] = None, record_logits: bool = False) -> dict:
    """speculative.py:101-122 -> {"tokens", "gaps"(, "logits")}: one target step per token."""
    gen = _gen(seed)
    ids = [int(t) for t in np.asarray(ids).reshape(-1)]
    cache = target.new_cache(len(ids) + max_new_tokens + 1)
    logits = target.forward(ids, None, cache, logits_to_keep=1)[-1]
    out = [first_token(logits, temperature, top_p, gen)]
    gaps = [_gap(logits)]
    rec = [logits] if record_logits else None
    while not finish(out, eos_ids, max_new_tokens)[1]:
        logits = target.forward([out[-1]], None, cache)[-1]
        out.append(first_token(logits, temperature, top_p, gen))
        gaps.append(_gap(logits))
        if record_logits:
            rec.append(logits)
    res = {"tokens": finish(out, eos_ids, max_new_tokens)[0], "gaps": gaps}
    if record_logits:
        res["logits"] = rec
    return res


def _gap(logits: np.ndarray) -> float:
    top = np.partition(logits, -2)[-2:]
    return float(top[1] - top[0])


def speculative_generate(target, draft, drafting: dict, ids, max_new_tokens: int, eos_ids=frozenset(),
                         seed: Optional[int] = None, keep_trees: bool = False) -> dict:
    """SpeculativeGenerator.generate (speculative.py:132-174).

    drafting: dict with depth, branch, width, max_nodes, temperature, top_p.
    Returns tokens, accepted_per_round, tree_sizes (and trees if keep_trees),
    and wall-clock seconds of the prefill and of the decode loop.
    """
    import time

    gen = _gen(seed)
    T = float(drafting.get("temperature", 0.0))
    P = float(drafting.get("top_p", 1.0))
    drafter = OracleTreeDrafter(draft, drafting["depth"], drafting.get("branch", 1), drafting.get("width"),
                                drafting.get("max_nodes"), T, P)
    ids = [int(t) for t in np.asarray(ids).reshape(-1)]
    n_prompt = len(ids)
    extra = max(drafter.max_verify_nodes(), drafter.max_tree_cache()) + 1
    cache = target.new_cache(n_prompt + max_new_tokens + drafting["depth"] + extra + 1)
    t0 = time.perf_counter()
    logits = target.forward(ids, None, cache, logits_to_keep=1)[-1]
    out = [first_token(logits, T, P, gen)]
    t1 = time.perf_counter()
    res = {"tokens": [], "accepted_per_round": [], "tree_sizes": [], "trees": [], "prefill_s": t1 - t0}
    while not finish(out, eos_ids, max_new_tokens)[1]:
        committed = cache.get_seq_length()
        tree = drafter.build(cache, [out[-1]], committed, gen)
        cache.crop(committed)
        vids, vpos, mask = verify_inputs(tree, out[-1], committed, committed)
        logits = target.forward(vids, vpos, cache, tree_mask=mask)
        if T == 0:
            accepted, bonus = greedy_verify(tree, logits)
        else:
            accepted, bonus = sample_verify(tree, logits, T, P, gen)
        cache.keep_positions(committed, [committed] + [committed + 1 + i for i in accepted])
        new = [tree.tokens[i] for i in accepted] + [bonus]
        out.extend(new)
        res["accepted_per_round"].append(len(new))
        res["tree_sizes"].append(len(tree))
        if keep_trees:
            res["trees"].append(dict(tokens=list(tree.tokens), parents=list(tree.parents), depths=list(tree.depths),
                                     ranks=list(tree.ranks), scores=list(tree.scores), accepted=list(accepted),
                                     bonus=bonus))
    res["tokens"] = finish(out, eos_ids, max_new_tokens)[0]
    res["decode_s"] = time.perf_counter() - t1
    return res
