"""Sampling (temperature > 0) on the device: warped distributions, Gumbel
top-k drafting and multi-candidate speculative-sampling verification.

The reference samples on the host: ``warp_probs`` (ssd/engine/tree_drafter.py:
34-45) sorts each row, ``_propose`` (tree_drafter.py:134-145) draws Gumbel
top-k per parent on the CPU, ``sample_verify`` (ssd/engine/verify.py:60-95)
walks the tree with ``torch.rand`` / ``torch.multinomial``. Here:

* the draft head writes fp32 logits of every draft row of the round
  (root = row 0, the fed level d node in slot j = row 1 + offset_d + j), one
  kernel computes each row's warp parameters {max, 1/T, nucleus threshold,
  log Z} (exact top-p by radix select, no sort), and one kernel draws
  ``branch`` children per row by Gumbel top-k;
* the target head writes the verify rows' logits, their warp parameters are
  computed in parallel, and a single-CTA kernel runs the rejection walk,
  materialising p and q only along the accepted path;
* random numbers are Philox4x32-10, keyed by the generation seed, counter =
  (round, row, index, stream): stream 0 the draft draws, 1 the acceptance
  tests, 2 the bonus token, 3 the target-only / first-token draws. Nothing
  on the host draws, so the round stays one CUDA graph per phase.

The draws differ from the reference's torch.Generator streams; what matches
is the distribution (the output of an unpruned tree is distributed exactly as
target sampling, checked by a chi-square test).
"""

from __future__ import annotations

import time
from typing import Optional

import torch

from ssd import _lib as L
from ssd import ops
from ssd.models import runner as R
from ssd.engine.round import BONUS, N_ACC, N_KEEP, N_OUT, SEQ, DeviceTree, GreedyRound, TargetStep

STREAM_DRAFT, STREAM_ACCEPT, STREAM_BONUS, STREAM_TOKEN = 0, 1, 2, 3


def seed_from(seed: Optional[int] = None, generator: Optional[torch.Generator] = None) -> int:
    """The 64-bit Philox key: the caller's seed, else one draw from `generator`
    (or from torch's default generator when neither is given)."""
    if seed is not None:
        return int(seed) & 0xFFFFFFFFFFFFFFFF
    return int(torch.randint(0, 2**62, (1,), generator=generator).item())


def _as_i64(seed: int) -> int:
    return seed - (1 << 64) if seed >= (1 << 63) else seed


class _SamplingState:
    """Seed word, temperature / top-p and the single-row logits buffers shared
    by the sampling engines."""

    def _init_sampling(self, temperature: float, top_p: float, seed: int) -> None:
        if not temperature > 0:
            raise ValueError("sampling engines need temperature > 0")
        if not 0 < top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        if self.w.tp is not None:
            raise NotImplementedError("sampling (temperature > 0) is not supported with tensor parallelism")
        dev, V = self.device, self.w.V
        self.temperature, self.top_p = float(temperature), float(top_p)
        self.seed_buf = torch.zeros(1, dtype=torch.int64, device=dev)
        self.logits1 = torch.zeros(1, V, dtype=torch.float32, device=dev)
        self.p_scratch = torch.zeros(V, dtype=torch.float32, device=dev)
        self.set_seed(seed)

    def set_seed(self, seed: int) -> None:
        self.seed_buf.fill_(_as_i64(int(seed) & 0xFFFFFFFFFFFFFFFF))

    def _first_token(self, xn: torch.Tensor, ws: ops.Workspace, rn=None) -> None:
        """_first_token with temperature > 0 (speculative.py:81-84): lm_head
        logits of the last prompt row, then one warped draw (round 0)."""
        ops.linear(xn, [self.w.lm_head], ws, epilogue=L.EPI_STORE_F32, out=self.logits1, T=1, in_norm=rn)
        ops.sample_token(self.logits1[0], self.temperature, self.top_p, self.seed_buf, None, 0, STREAM_TOKEN,
                         self.p_scratch, self.argmax[:1])


class SampledTargetStep(_SamplingState, TargetStep):
    """Target-only sampled decoding step: prep -> target forward (T=1) ->
    lm_head logits -> warped draw -> commit, one CUDA graph. The draw's RNG
    round is the number of tokens generated so far."""

    def __init__(self, target, cache, max_new: int, temperature: float, top_p: float, seed: int):
        TargetStep.__init__(self, target, cache, max_new)
        self._init_sampling(temperature, top_p, seed)

    def _next_token(self, xn: torch.Tensor, rn=None) -> None:
        st = self.state
        ops.linear(xn, [self.w.lm_head], self.ws, epilogue=L.EPI_STORE_F32, out=self.logits1, T=1, in_norm=rn)
        ops.sample_token(self.logits1[0], self.temperature, self.top_p, self.seed_buf, st[N_OUT:N_OUT + 1], 0,
                         STREAM_TOKEN, self.p_scratch, self.argmax[:1])


class SampledRound(_SamplingState, GreedyRound):
    """One sampled speculative round over device-resident state: the greedy
    round's kernels with the two heads replaced (Gumbel top-k drafting,
    rejection-sampling walk). The RNG round is round_log[0], the number of
    rounds committed since prefill."""

    def __init__(self, target, draft, cfg, cache, max_new: int, seed: int):
        GreedyRound.__init__(self, target, draft, cfg, cache, max_new)
        self._init_sampling(cfg.temperature, cfg.top_p, seed)
        p, dev = self.plan, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        self.Vd = int(self.head_w.shape[0])
        self.draft_rows = 1 + p.max_tree_cache
        self.dlogits = torch.zeros(self.draft_rows, self.Vd, **f32)
        self.dparams = ops.warp_params_buffer(self.draft_rows, dev)
        self.tlogits = torch.zeros(p.rows, self.w.V, **f32)
        self.tparams = ops.warp_params_buffer(p.rows, dev)
        self.q_scratch = torch.zeros(self.w.V, **f32)

    def _propose(self, xn, row0, T, k, out_tok, out_lp, rn=None) -> None:
        """_propose with sampling (tree_drafter.py:134-145): draft logits ->
        warp parameters -> k draws without replacement per row."""
        rows = self.dlogits[row0:row0 + T]
        prm = self.dparams[row0:row0 + T]
        ops.linear(xn, [self.head_w], self.ws, epilogue=L.EPI_STORE_F32, out=rows, T=T, in_norm=rn)
        ops.warp_sample_topk(rows, self.temperature, self.top_p, prm, k, self.seed_buf, self.round_log[0:1], row0,
                             out_tok, out_lp, vocab_ids=self.vocab_ids)

    def _walk(self, xn, rn=None) -> None:
        """sample_verify (verify.py:60-95) on the device."""
        p, st = self.plan, self.state
        ops.linear(xn, [self.w.lm_head], self.ws, epilogue=L.EPI_STORE_F32, out=self.tlogits, T=p.rows, in_norm=rn)
        ops.warp_sample_topk(self.tlogits, self.temperature, self.top_p, self.tparams)
        ops.tree_walk_sample(self.tree, self.tlogits, self.tparams, self.dlogits, self.dparams, self.draft_rows,
                             self.seed_buf, self.round_log[0:1], self.p_scratch, self.q_scratch, st[SEQ:SEQ + 1],
                             self.accepted, st[N_ACC:N_ACC + 1], st[BONUS:BONUS + 1], self.keep_slots,
                             st[N_KEEP:N_KEEP + 1], p.n_verify, self.ws.status, vocab_ids=self.vocab_ids)

    def draft_probs(self, row: int) -> torch.Tensor:
        """Warped draft distribution of one draft row over the full vocabulary
        (the reference's DraftTree.child_q entry)."""
        out = torch.zeros(1, self.Vd, dtype=torch.float32, device=self.device)
        ops.warp_probs(self.dlogits[row:row + 1], self.dparams[row:row + 1], out)
        if self.vocab_ids is None:
            return out[0]
        full = torch.zeros(self.w.V, dtype=torch.float32, device=self.device)
        return full.index_copy_(0, self.vocab_ids.to(self.device), out[0])


# ---------------------------------------------------------------- host API
def warp_probs_device(logits: torch.Tensor, temperature: float, top_p: float) -> torch.Tensor:
    """warp_probs (tree_drafter.py:34-45): fp32 probabilities of softmax(l / T)
    restricted to the top-p nucleus, renormalised, over the last dimension.
    Computed on the GPU; the result is returned on the input's device."""
    if not torch.cuda.is_available():
        raise RuntimeError("warp_probs runs on the sm_100a kernels and needs a CUDA device")
    src_dev = logits.device
    V = logits.shape[-1]
    x = logits.detach().to(device="cuda" if not logits.is_cuda else logits.device, dtype=torch.float32)
    x = x.reshape(-1, V).contiguous()
    rows = x.shape[0]
    params = ops.warp_params_buffer(rows, x.device)
    ops.warp_params(x, temperature, top_p, params)
    out = torch.empty_like(x)
    ops.warp_probs(x, params, out)
    return out.reshape(logits.shape).to(src_dev)


def sampled_tree_build(drafter, cache, pending: torch.Tensor, root_pos: int, generator=None):
    """TreeDrafter.build with temperature > 0 (tree_drafter.py:147-208): the
    sampled round's draft phase on the device, read back as a DraftTree whose
    child_q holds each parent's warped draft distribution (full vocabulary)."""
    from ssd.engine.round import ROOT_TOK
    from ssd.engine.tree_drafter import DraftTree

    draft = drafter.draft
    w = draft.weights
    pend = pending.reshape(-1)
    n_pend = int(pend.numel())
    if cache.get_seq_length() != root_pos - n_pend + 1:
        raise ValueError("pending tokens must directly follow the cache contents")
    if n_pend > 1:
        draft(pend[:-1].reshape(1, -1), position_ids=torch.arange(root_pos - n_pend + 1, root_pos).reshape(1, -1),
              past_key_values=cache, compute_logits=False)
    cache.allocate(w.Hkv, w.hd, w.dtype, w.device)
    eng = drafter._engine
    if not isinstance(eng, SampledRound) or eng.cache is not cache:
        eng = SampledRound(draft, draft, drafter.cfg, cache, max_new=1, seed=0)
        drafter._engine = eng
    eng.set_seed(seed_from(None, generator))
    eng.state[SEQ] = root_pos
    eng.state[ROOT_TOK] = int(pend[-1])
    eng.draft_phase()
    t = eng.read_tree()
    eng.ws.check_status()
    tree = DraftTree(tokens=t["tokens"], parents=t["parents"], depths=t["depths"], scores=t["scores"],
                     ranks=t["ranks"], draft_pos=t["draft_pos"], cache_start=root_pos + 1)
    parents = set(tree.parents)
    for par in parents:
        row = 0 if par == -1 else tree.draft_pos[par] - root_pos
        tree.child_q[par] = eng.draft_probs(row).cpu()
    cache.seq_len = root_pos + 1 + eng.plan.max_tree_cache
    return tree


def sample_verify_device(tree, target_logits: torch.Tensor, temperature: float, top_p: float,
                         generator=None) -> tuple[list[int], int]:
    """sample_verify (verify.py:60-95) for a host DraftTree: the tree and its
    child_q go to the device, the walk runs in one kernel."""
    if not torch.cuda.is_available():
        raise RuntimeError("sample_verify runs on the sm_100a kernels and needs a CUDA device")
    dev = target_logits.device if target_logits.is_cuda else torch.device("cuda")
    n = len(tree)
    V = int(target_logits.shape[-1])
    t = DeviceTree(max(n, 1), dev)
    draft_pos = [0] * n
    rows = {-1: 0}
    for par in sorted(k for k in tree.child_q if k != -1):
        rows[par] = len(rows)
        draft_pos[par] = rows[par]
    if n:
        i32 = dict(dtype=torch.int32)
        t.tokens[:n].copy_(torch.tensor(tree.tokens, **i32))
        t.parents[:n].copy_(torch.tensor(tree.parents, **i32))
        t.ranks[:n].copy_(torch.tensor(tree.ranks, **i32))
        t.draft_pos[:n].copy_(torch.tensor(draft_pos, **i32))
    t.n_nodes.fill_(n)
    # q rows as log-probabilities with identity warp parameters {0, 1, -inf, 0}
    qlog = torch.full((len(rows), V), float("-inf"), dtype=torch.float32, device=dev)
    for par, r in rows.items():
        if par in tree.child_q:
            qlog[r] = tree.child_q[par].to(dev, torch.float32).log()
    dparams = torch.tensor([[0.0, 1.0, float("-inf"), 0.0]] * len(rows), dtype=torch.float32, device=dev)
    tl = target_logits.detach().to(dev, torch.float32).reshape(-1, V).contiguous()
    tparams = ops.warp_params_buffer(tl.shape[0], dev)
    ops.warp_params(tl, temperature, top_p, tparams)
    i32 = dict(dtype=torch.int32, device=dev)
    seed = torch.tensor([_as_i64(seed_from(None, generator))], dtype=torch.int64, device=dev)
    accepted = torch.zeros(max(n, 1) + 1, **i32)
    n_acc, bonus, n_keep = (torch.zeros(1, **i32) for _ in range(3))
    keep = torch.zeros(max(n, 1) + 2, **i32)
    zero = torch.zeros(1, **i32)
    status = torch.zeros(1, **i32)
    ops.tree_walk_sample(t, tl, tparams, qlog, dparams, len(rows), seed, None,
                         torch.empty(V, dtype=torch.float32, device=dev),
                         torch.empty(V, dtype=torch.float32, device=dev), zero, accepted, n_acc, bonus, keep, n_keep,
                         n, status)
    if int(status.item()):
        raise RuntimeError("sample_verify: device walk reported an index error")
    na = int(n_acc.item())
    return accepted[:na].tolist(), int(bonus.item())


def _timed_decode(eng, dev, input_ids, run, done, clock=None):
    """Prefill, then `run` until `done`; times {prefill, decode}, or with a
    PhaseClock {prefill, draft, verify, bookkeeping}."""
    times: dict[str, float] = {}
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    eng.prefill(input_ids.to(dev))
    torch.cuda.synchronize(dev)
    times["prefill"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    out = eng.tokens()
    while not done(out):
        run(len(out))
        out = eng.tokens()
        if clock is not None:
            clock.collect()
    torch.cuda.synchronize(dev)
    if clock is None:
        times["decode"] = time.perf_counter() - t0
    else:
        clock.finish(times, time.perf_counter() - t0)
    eng.ws.check_status()
    eng.cache.seq_len = int(eng.state[SEQ].item())
    return out, times


def sampled_autoregressive(target, input_ids: torch.Tensor, max_new_tokens: int, eos_ids: set[int],
                           temperature: float, top_p: float, seed: Optional[int] = None, use_graph: bool = True,
                           steps_per_sync: int = 4, max_cache: Optional[int] = None):
    """autoregressive_generate with temperature > 0 (speculative.py:101-122)."""
    from ssd.engine.round import cache_capacity
    from ssd.engine.speculative import GenerationResult, _engine_cache, _finish

    dev = target.weights.device
    n_prompt = int(input_ids.shape[-1])
    cap = max_cache or cache_capacity(n_prompt, max_new_tokens)
    key = ("ar_sample", n_prompt, max_new_tokens, cap, float(temperature), float(top_p))
    eng = _engine_cache(target, key, lambda: SampledTargetStep(target, target.new_cache(cap), max_new_tokens,
                                                               temperature, top_p, 0))
    eng.set_seed(seed_from(seed))
    out, times = _timed_decode(
        eng, dev, input_ids,
        lambda n: eng.run(max(1, min(steps_per_sync, max_new_tokens - n)), use_graph),
        lambda out: _finish(out, eos_ids, max_new_tokens)[1])
    return GenerationResult(tokens=_finish(out, eos_ids, max_new_tokens)[0], times=times)


def sampled_speculative(gen, input_ids: torch.Tensor, max_new_tokens: int, eos_ids: set[int],
                        seed: Optional[int] = None, use_graph: bool = True, max_cache: Optional[int] = None):
    """SpeculativeGenerator.generate with temperature > 0 (speculative.py:132-174)."""
    from ssd.engine.round import cache_capacity
    from ssd.engine.speculative import GenerationResult, PhaseClock, _engine_cache, _finish

    cfg = gen.cfg
    dev = gen.target.weights.device
    n_prompt = int(input_ids.shape[-1])
    cap = max_cache or cache_capacity(n_prompt, max_new_tokens, gen.plan)
    key = ("sd_sample", id(gen.draft), n_prompt, max_new_tokens, cap, repr(cfg))
    eng = _engine_cache(gen, key, lambda: SampledRound(gen.target, gen.draft, cfg, gen.target.new_cache(cap),
                                                       max_new_tokens, 0))
    eng.set_seed(seed_from(seed))
    clock = PhaseClock(eng.PHASES)
    out, times = _timed_decode(eng, dev, input_ids, lambda n: eng.run_round(use_graph, clock.round_events()),
                               lambda out: _finish(out, eos_ids, max_new_tokens)[1], clock)
    acc = eng.committed_per_round()
    return GenerationResult(tokens=_finish(out, eos_ids, max_new_tokens)[0], times=times, accepted_per_round=acc,
                            tree_sizes=[gen.plan.n_verify] * len(acc))
