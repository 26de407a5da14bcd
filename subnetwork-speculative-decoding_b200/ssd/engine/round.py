"""Device-resident speculative-decoding round and target-only step.

The reference drives a round from Python with a host sync per tree level
(ssd/engine/tree_drafter.py:133,143-144; ssd/engine/verify.py:47). Here the
whole round is a fixed sequence of kernel launches that reads every dynamic
quantity (committed length, root token, tree) from device memory:

  draft root forward -> top-k -> for each level: level prune (+ the level's
  draft forward -> top-k) -> max_nodes prune -> verify inputs -> target
  forward over root + tree -> argmax -> tree walk -> KV compaction -> commit

so it is captured once in a CUDA graph and replayed; the host reads back the
committed tokens once per round. Every level has a static maximum size
(min(parents x branch, width)); a level with fewer candidates (sampling,
where a parent's nucleus can hold fewer than `branch` tokens) leaves empty
slots that the prune kernels skip, so the shapes stay static. The sampling
round (ssd/engine/sampling.py) overrides the two head hooks, `_propose` and
`_walk`, of the greedy round defined here.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from ssd import ops
from ssd.config import DraftingConfig
from ssd.models import runner as R

# state word indices
SEQ, ROOT_TOK, N_NODES, N_ACC, BONUS, N_KEEP, N_OUT, ZERO = range(8)


class TreePlan:
    """Static shape of a greedy tree (TreeDrafter.max_nodes_per_level and
    friends, ssd/engine/tree_drafter.py:107-122)."""

    def __init__(self, cfg: DraftingConfig):
        cfg.validate()
        self.cfg = cfg
        self.depth = cfg.depth
        self.branch = cfg.per_depth(cfg.branch, "branch")
        self.width = cfg.per_depth(cfg.width, "width")
        if max(self.branch) > 16:
            raise ValueError("branch entries above 16 are not supported by the device top-k")
        n, sizes = 1, []
        for d in range(self.depth):
            n *= self.branch[d]
            if self.width[d] is not None:
                n = min(n, self.width[d])
            sizes.append(n)
        self.level_sizes = sizes
        self.fed = [d < self.depth - 1 for d in range(self.depth)]
        offs, acc = [], 0
        for d in range(self.depth):
            offs.append(acc)
            if self.fed[d]:
                acc += sizes[d]
        self.slot_offsets = offs
        self.max_tree_cache = acc
        self.cap = sum(sizes)
        self.n_verify = min(self.cap, cfg.max_nodes) if cfg.max_nodes else self.cap
        self.rows = self.n_verify + 1
        self.mask_words = max(1, math.ceil(max(self.max_tree_cache, self.n_verify) / 64))
        if self.mask_words > 4:
            raise ValueError("tree too large for the 256-slot ancestor mask")
        self.max_fwd_rows = max([1, self.rows] + [sizes[d] for d in range(self.depth) if self.fed[d]])

    def max_verify_nodes(self) -> int:
        return self.n_verify


class DeviceTree:
    def __init__(self, cap: int, device):
        i32 = dict(dtype=torch.int32, device=device)
        self.cap = cap
        self.tokens = torch.zeros(cap, **i32)
        self.parents = torch.zeros(cap, **i32)
        self.depths = torch.zeros(cap, **i32)
        self.ranks = torch.zeros(cap, **i32)
        self.draft_pos = torch.zeros(cap, **i32)
        self.scores = torch.zeros(cap, dtype=torch.float64, device=device)
        self.n_nodes = torch.zeros(1, **i32)


def cache_capacity(n_prompt: int, max_new: int, plan: Optional[TreePlan] = None) -> int:
    """Cache length used by both the speculative and the target-only engine
    (one rule, so both see the same attention split layout)."""
    need = n_prompt + max_new + 2
    if plan is not None:
        need += plan.depth + max(plan.n_verify, plan.max_tree_cache) + 1
    slack = 64 + (0 if plan is None else plan.rows + plan.max_tree_cache)
    return int(math.ceil((n_prompt + max_new + max(slack, need - n_prompt - max_new)) / 256.0) * 256)


class _Decoder:
    """Shared state, buffers and prefill of the device engines."""

    def __init__(self, target, cache, max_new: int, fwd_rows: int, head_rows: int):
        self.target = target
        self.w: R.ModelWeights = target.weights
        w = self.w
        self.device = w.device
        self.cache = cache
        cache.allocate(w.Hkv, w.hd, w.dtype, w.device)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.state = torch.zeros(8, **i32)
        self.out_cap = max_new + 64
        self.out_tokens = torch.zeros(self.out_cap, **i32)
        self.round_log = torch.zeros(1 + self.out_cap, **i32)
        self.scratch = R.Scratch(w, max(fwd_rows, 1))
        self.ws = ops.Workspace(self.device, max_rows=max(fwd_rows, 64), vocab=w.V, max_head_rows=max(head_rows, 1))
        self.argmax = torch.zeros(max(head_rows, 1), **i32)
        self.amax = torch.zeros(max(head_rows, 1), dtype=torch.float32, device=self.device)
        self.gap = torch.zeros(max(head_rows, 1), dtype=torch.float32, device=self.device)
        self.fwd_root = R.ForwardInputs(1, self.device, mask_words=1)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self._prefill_bufs = None  # (rows, ForwardInputs, Scratch, Workspace) of the longest prompt so far

    def _prefill_buffers(self, P: int):
        """Inputs, activations and workspace for a prompt of P rows, kept for
        later prompts of up to the same length (the workspace is zeroed once
        at allocation; its split counters reset themselves)."""
        if self._prefill_bufs is None or self._prefill_bufs[0] < P:
            self._prefill_bufs = None  # release the smaller set first
            w = self.w
            self._prefill_bufs = (P, R.ForwardInputs(P, self.device, mask_words=1), R.Scratch(w, P),
                                  ops.Workspace(self.device, max_rows=P, vocab=w.V, max_head_rows=1))
        return self._prefill_bufs[1:]

    def prefill(self, prompt: torch.Tensor) -> None:
        """Target over the prompt (causal), first token = argmax of its last row
        (speculative.py:222-224 with temperature 0)."""
        w = self.w
        P = int(prompt.numel())
        self.cache.reset()
        self.cache.check_room(P)
        fwd, scratch, ws = self._prefill_buffers(P)
        fwd.fill(prompt.reshape(-1), torch.arange(P), 0, None)
        R.run_stack_auto(w, self.target.layer_indices, [None] * len(self.target.layer_indices), None, fwd, P,
                         self.cache, scratch, ws, self.cache.max_length)
        xn, rn = R.head_input(w, scratch, P - 1, P)
        self._first_token(xn, ws, rn)
        self.state.zero_()
        self.state[SEQ] = P
        self.state[ROOT_TOK:ROOT_TOK + 1].copy_(self.argmax[:1])
        self.out_tokens[:1].copy_(self.argmax[:1])
        self.state[N_OUT] = 1
        self.round_log.zero_()
        ws.check_status()
        self.cache.seq_len = P

    def _first_token(self, xn: torch.Tensor, ws: ops.Workspace, rn=None) -> None:
        """First generated token from the last prompt row into argmax[0]
        (_first_token, speculative.py:81-84; greedy here). rn: the folded
        final RMSNorm of xn, if any."""
        R.head_argmax(self.w, xn, self.w.lm_head, self.argmax[:1], ws, out_max=self.amax[:1], out_gap=self.gap[:1],
                      in_norm=rn)

    def _capture(self, fn) -> torch.cuda.CUDAGraph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.graph(g, stream=s):
            fn()
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g

    def n_out(self) -> int:
        return int(self.state[N_OUT].item())

    def tokens(self) -> list[int]:
        """Committed tokens so far (one small device->host read)."""
        n = min(self.n_out(), self.out_cap)
        self.d2h_bytes = getattr(self, "d2h_bytes", 0) + 4 + 4 * n
        return self.out_tokens[:n].tolist()


class TargetStep(_Decoder):
    """Target-only greedy decoding step (autoregressive_generate,
    ssd/engine/speculative.py:101-122) as one graph: prep -> target forward
    (T=1) -> argmax -> commit."""

    def __init__(self, target, cache, max_new: int):
        super().__init__(target, cache, max_new, fwd_rows=1, head_rows=1)

    def step(self) -> None:
        w = self.w
        st = self.state
        ops.causal_prep(st[SEQ:SEQ + 1], 1, st[ROOT_TOK:ROOT_TOK + 1], self.fwd_root)
        R.run_stack_auto(w, self.target.layer_indices, [None] * len(self.target.layer_indices), None, self.fwd_root,
                         1, self.cache, self.scratch, self.ws, self.cache.max_length)
        xn, rn = R.head_input(w, self.scratch, 0, 1)
        self._next_token(xn, rn)
        ops.round_commit(st[ZERO:ZERO + 1], self.argmax, self.out_tokens, self.argmax[:1], st[SEQ:SEQ + 1],
                         st[ROOT_TOK:ROOT_TOK + 1], self.out_tokens, st[N_OUT:N_OUT + 1], None, self.ws.status)

    def _next_token(self, xn: torch.Tensor, rn=None) -> None:
        """Next token into argmax[0]: lm_head fused with the argmax."""
        R.head_argmax(self.w, xn, self.w.lm_head, self.argmax[:1], self.ws, out_max=self.amax[:1],
                      out_gap=self.gap[:1], in_norm=rn)

    def run(self, n_steps: int, use_graph: bool = True) -> None:
        if use_graph:
            if self.graph is None:
                before = ops.launch_count()
                self.graph = self._capture(self.step)
                self.launches_per_round = ops.launch_count() - before
            for _ in range(n_steps):
                self.graph.replay()
        else:
            for _ in range(n_steps):
                self.step()


class GreedyRound(_Decoder):
    """One greedy speculative round over device-resident state."""

    def __init__(self, target, draft, cfg: DraftingConfig, cache, max_new: int):
        self.plan = TreePlan(cfg)
        p = self.plan
        super().__init__(target, cache, max_new, fwd_rows=p.max_fwd_rows, head_rows=p.rows)
        self.draft = draft
        dev = self.device
        self.tree = DeviceTree(p.cap, dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.root_frontier = torch.full((1,), -1, **i32)
        self.level_nodes = [torch.zeros(n, **i32) for n in p.level_sizes]
        self.fwd_level = [R.ForwardInputs(p.level_sizes[d], dev, p.mask_words) if p.fed[d] else None
                          for d in range(p.depth)]
        for f in self.fwd_level:
            if f is not None:
                f.use_mask = True
        self.fwd_verify = R.ForwardInputs(p.rows, dev, p.mask_words)
        self.fwd_verify.use_mask = True
        parents = [1] + p.level_sizes[:-1]
        self.topk_tok = [torch.zeros(parents[d], p.branch[d], **i32) for d in range(p.depth)]
        self.topk_lp = [torch.zeros(parents[d], p.branch[d], dtype=torch.float32, device=dev)
                        for d in range(p.depth)]
        self.accepted = torch.zeros(p.depth + 1, **i32)
        self.keep_slots = torch.zeros(p.depth + 2, **i32)
        self.scratch.reserve_bridges(list(draft.bridges.values()))
        self.head_w = draft.head_weight()
        self.vocab_ids = draft.vocab_ids
        for b in draft.bridges.values():
            if b.norm.weight.device != dev:
                raise ValueError("bridges must live on the model's device")

    # --------------------------------------------------------------- phases
    def _draft_forward(self, fwd, T: int):
        """Draft sub-network forward; returns the head input (x, folded norm or None)."""
        d = self.draft
        R.run_stack_auto(self.w, d.layer_indices, d.pre_layer_bridge_modules(), d.pre_norm_bridge_module(), fwd, T,
                         self.cache, self.scratch, self.ws, self.cache.max_length)
        return R.head_input(self.w, self.scratch, 0, T)

    def draft_phase(self) -> None:
        """TreeDrafter.build (tree_drafter.py:147-208) on the device."""
        p, st = self.plan, self.state
        ops.causal_prep(st[SEQ:SEQ + 1], 1, st[ROOT_TOK:ROOT_TOK + 1], self.fwd_root)
        xn, rn = self._draft_forward(self.fwd_root, 1)
        self._propose(xn, 0, 1, p.branch[0], self.topk_tok[0], self.topk_lp[0], rn)
        for d in range(p.depth):
            frontier = self.root_frontier if d == 0 else self.level_nodes[d - 1]
            n_front = 1 if d == 0 else p.level_sizes[d - 1]
            ops.level_prune(self.topk_tok[d], self.topk_lp[d], n_front, p.branch[d], p.width[d], d, frontier,
                            self.level_nodes[d], self.tree, st[SEQ:SEQ + 1], p.fed[d], p.slot_offsets[d],
                            self.fwd_level[d], self.ws.status)
            if p.fed[d]:
                xn, rn = self._draft_forward(self.fwd_level[d], p.level_sizes[d])
                self._propose(xn, 1 + p.slot_offsets[d], p.level_sizes[d], p.branch[d + 1], self.topk_tok[d + 1],
                              self.topk_lp[d + 1], rn)
        ops.tree_prune(self.tree, p.cfg.max_nodes)

    def _propose(self, xn: torch.Tensor, row0: int, T: int, k: int, out_tok: torch.Tensor,
                 out_lp: torch.Tensor, rn=None) -> None:
        """k children per draft row (TreeDrafter._propose, tree_drafter.py:124-132
        for greedy): the draft head fused with a log-softmax top-k. `row0` is
        the row's index among the round's draft rows (0 = root)."""
        R.head_topk(self.w, xn, self.head_w, k, out_tok, out_lp, self.ws, vocab_ids=self.vocab_ids, in_norm=rn)

    def verify_phase(self) -> None:
        """verify_inputs + target forward + greedy_verify (verify.py:32-57)."""
        p, st, w = self.plan, self.state, self.w
        ops.verify_prep(self.tree, p.rows, st[ROOT_TOK:ROOT_TOK + 1], st[SEQ:SEQ + 1], self.fwd_verify,
                        self.ws.status)
        R.run_stack_auto(w, self.target.layer_indices, [None] * len(self.target.layer_indices), None,
                         self.fwd_verify, p.rows, self.cache, self.scratch, self.ws, self.cache.max_length)
        xn, rn = R.head_input(w, self.scratch, 0, p.rows)
        self._walk(xn, rn)

    def _walk(self, xn: torch.Tensor, rn=None) -> None:
        """Target head over root + tree rows, then the acceptance walk
        (greedy_verify, verify.py:45-57): lm_head fused with the argmax."""
        p, st, w = self.plan, self.state, self.w
        R.head_argmax(w, xn, w.lm_head, self.argmax[: p.rows], self.ws, out_max=self.amax[: p.rows],
                      out_gap=self.gap[: p.rows], in_norm=rn)
        ops.tree_walk_greedy(self.tree, self.argmax, st[SEQ:SEQ + 1], self.accepted, st[N_ACC:N_ACC + 1],
                             st[BONUS:BONUS + 1], self.keep_slots, st[N_KEEP:N_KEEP + 1], p.n_verify)

    def commit_phase(self) -> None:
        """keep_positions + append accepted + bonus (speculative.py:165-172)."""
        st = self.state
        ops.kv_compact(self.cache.buf, st[SEQ:SEQ + 1], self.keep_slots, st[N_KEEP:N_KEEP + 1],
                       max_keep=self.plan.depth + 1, status=self.ws.status)
        ops.round_commit(st[N_ACC:N_ACC + 1], self.accepted, self.tree.tokens, st[BONUS:BONUS + 1], st[SEQ:SEQ + 1],
                         st[ROOT_TOK:ROOT_TOK + 1], self.out_tokens, st[N_OUT:N_OUT + 1], self.round_log,
                         self.ws.status)

    def round(self) -> None:
        self.draft_phase()
        self.verify_phase()
        self.commit_phase()

    PHASES = ("draft", "verify", "bookkeeping")

    def run_round(self, use_graph: bool = True, events: Optional[list] = None) -> None:
        """One round. With use_graph the three phases replay as captured CUDA
        graphs; `events` (4 CUDA events) are recorded between them so the
        caller can read per-phase device time without host syncs."""
        fns = (self.draft_phase, self.verify_phase, self.commit_phase)
        if use_graph and self.graph is None:
            self.graph = []
            for fn in fns:
                before = ops.launch_count()
                self.graph.append(self._capture(fn))
                self.launches_per_round = getattr(self, "launches_per_round", 0) + ops.launch_count() - before
        for i, fn in enumerate(fns):
            if events is not None:
                events[i].record()
            if use_graph:
                self.graph[i].replay()
            else:
                fn()
        if events is not None:
            events[3].record()

    def committed_per_round(self) -> list[int]:
        n = int(self.round_log[0].item())
        return self.round_log[1:1 + n].tolist()

    def read_tree(self):
        """The current device tree as host lists (for the API path / tests)."""
        n = int(self.tree.n_nodes.item())
        t = self.tree
        return dict(tokens=t.tokens[:n].tolist(), parents=t.parents[:n].tolist(), depths=t.depths[:n].tolist(),
                    ranks=t.ranks[:n].tolist(), scores=t.scores[:n].tolist(), draft_pos=t.draft_pos[:n].tolist())
