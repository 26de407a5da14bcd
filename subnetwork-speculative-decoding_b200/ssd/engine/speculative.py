"""Speculative decoding loop and the autoregressive baseline (API of
ssd/engine/speculative.py:65-174).

One KV cache shared by target and draft (batch 1). Between rounds it holds
the target's KV for every layer of all committed tokens except the last one
(the root). A round drafts a tree through the draft sub-network, verifies
root + tree with the target in one forward, keeps the root and the accepted
path in the cache and commits accepted + bonus tokens.

Rounds run as CUDA graphs over device-resident state (ssd/engine/round.py,
greedy; ssd/engine/sampling.py, temperature > 0); the host reads the
committed tokens once per round.
The target-only baseline runs the same layer kernels one token per step.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn as nn

from ssd.config import DraftingConfig
from ssd.engine.round import GreedyRound, TargetStep, TreePlan, cache_capacity
from ssd.engine.kv_cache import KVCache
from ssd.models.subnetwork_draft import SubnetworkDraftModel


@dataclass
class GenerationResult:
    tokens: list[int]
    times: dict[str, float]  # seconds per phase
    accepted_per_round: list[int] = field(default_factory=list)  # committed per round (accepted + bonus)
    tree_sizes: list[int] = field(default_factory=list)

    @property
    def decode_time(self) -> float:
        return sum(v for k, v in self.times.items() if k != "prefill")

    @property
    def mean_accepted(self) -> float:
        return sum(self.accepted_per_round) / max(1, len(self.accepted_per_round))


def _finish(tokens: list[int], eos_ids: set[int], max_new: int) -> tuple[list[int], bool]:
    """speculative.py:87-91."""
    for i, t in enumerate(tokens[:max_new]):
        if t in eos_ids:
            return tokens[: i + 1], True
    return tokens[:max_new], len(tokens) >= max_new


class TargetRunner(SubnetworkDraftModel):
    """The full target through the same layer kernels (speculative.py:94-98)."""

    def __init__(self, base: nn.Module):
        super().__init__(base, list(range(base.config.num_hidden_layers)))


def _sync(dev) -> None:
    torch.cuda.synchronize(dev)


class PhaseClock:
    """Per-phase times of the round loop for GenerationResult.times (the
    reference's draft / verify / bookkeeping totals, speculative.py:149-171).
    Each round's phases are bracketed by CUDA events on the launching stream;
    they are read after the round's committed tokens (a stream-synchronising
    read), so the clock adds no synchronisation of its own. Host time of the
    loop not covered by device phases (token reads, the Python loop) is
    counted as bookkeeping, so the phases add up to the decode wall time."""

    def __init__(self, phases):
        self.phases = tuple(phases)
        self.events = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.phases) + 1)]
        self.totals = {p: 0.0 for p in self.phases}
        self.armed = False

    def collect(self) -> None:
        """Add the last round's phase times (its events have completed)."""
        if self.armed:
            for i, p in enumerate(self.phases):
                self.totals[p] += self.events[i].elapsed_time(self.events[i + 1]) / 1e3
        self.armed = False

    def round_events(self):
        self.armed = True
        return self.events

    def finish(self, times: dict, wall: float) -> None:
        self.collect()
        times.update(self.totals)
        rest = wall - sum(self.totals.values())
        if rest > 0 and "bookkeeping" in times:
            times["bookkeeping"] += rest


@torch.no_grad()
def autoregressive_generate(target: TargetRunner, input_ids: torch.Tensor, max_new_tokens: int, eos_ids: set[int],
                            temperature: float = 0.0, top_p: float = 1.0, seed: Optional[int] = None,
                            use_graph: bool = True, steps_per_sync: int = 4, max_cache: Optional[int] = None
                            ) -> GenerationResult:
    """Target-only decoding, one target step per token (speculative.py:101-122)."""
    if temperature != 0:
        from ssd.engine.sampling import sampled_autoregressive

        return sampled_autoregressive(target, input_ids, max_new_tokens, eos_ids, temperature, top_p, seed,
                                      use_graph=use_graph, steps_per_sync=steps_per_sync, max_cache=max_cache)
    dev = target.weights.device
    n_prompt = int(input_ids.shape[-1])
    cap = max_cache or cache_capacity(n_prompt, max_new_tokens)
    eng = _engine_cache(target, ("ar", n_prompt, max_new_tokens, cap),
                        lambda: TargetStep(target, target.new_cache(cap), max_new_tokens))
    times: dict[str, float] = {}
    _sync(dev)
    t0 = time.perf_counter()
    eng.prefill(input_ids.to(dev))
    _sync(dev)
    times["prefill"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    out = eng.tokens()
    while not _finish(out, eos_ids, max_new_tokens)[1]:
        left = max_new_tokens - len(out)
        eng.run(max(1, min(steps_per_sync, left)), use_graph)
        out = eng.tokens()
    _sync(dev)
    times["decode"] = time.perf_counter() - t0
    eng.ws.check_status()
    eng.cache.seq_len = int(eng.state[0].item())
    return GenerationResult(tokens=_finish(out, eos_ids, max_new_tokens)[0], times=times)


def _engine_cache(owner, key, make):
    """Keep the last engine (buffers + captured graph) per owner and key."""
    store = getattr(owner, "_ssd_engines", None)
    if store is None:
        store = {}
        object.__setattr__(owner, "_ssd_engines", store)
    eng = store.get(key)
    if eng is None:
        store.clear()
        torch.cuda.empty_cache()
        eng = make()
        store[key] = eng
    return eng


class SpeculativeGenerator:
    def __init__(self, base: nn.Module, draft: SubnetworkDraftModel, cfg: DraftingConfig,
                 target: Optional[TargetRunner] = None):
        cfg.validate()
        self.target = target or TargetRunner(base)
        self.draft = draft
        self.cfg = cfg
        self.plan = TreePlan(cfg)

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, eos_ids: set[int], seed: Optional[int] = None,
                 use_graph: bool = True, max_cache: Optional[int] = None) -> GenerationResult:
        """SpeculativeGenerator.generate (speculative.py:132-174)."""
        cfg = self.cfg
        if cfg.temperature != 0:
            from ssd.engine.sampling import sampled_speculative

            return sampled_speculative(self, input_ids, max_new_tokens, eos_ids, seed, use_graph=use_graph,
                                       max_cache=max_cache)
        dev = self.target.weights.device
        n_prompt = int(input_ids.shape[-1])
        cap = max_cache or cache_capacity(n_prompt, max_new_tokens, self.plan)
        key = ("sd", id(self.draft), n_prompt, max_new_tokens, cap, repr(cfg))
        eng = _engine_cache(self, key, lambda: GreedyRound(self.target, self.draft, cfg, self.target.new_cache(cap),
                                                           max_new_tokens))
        times: dict[str, float] = {}
        _sync(dev)
        t0 = time.perf_counter()
        eng.prefill(input_ids.to(dev))
        _sync(dev)
        times["prefill"] = time.perf_counter() - t0
        clock = PhaseClock(eng.PHASES)
        t0 = time.perf_counter()
        out = eng.tokens()
        while not _finish(out, eos_ids, max_new_tokens)[1]:
            eng.run_round(use_graph, clock.round_events())
            out = eng.tokens()
            clock.collect()
        _sync(dev)
        clock.finish(times, time.perf_counter() - t0)
        eng.ws.check_status()
        eng.cache.seq_len = int(eng.state[0].item())
        acc = eng.committed_per_round()
        return GenerationResult(tokens=_finish(out, eos_ids, max_new_tokens)[0], times=times,
                                accepted_per_round=acc, tree_sizes=[self.plan.n_verify] * len(acc))

    def engine(self):
        store = getattr(self, "_ssd_engines", {})
        return next(iter(store.values()), None)
