"""Batched decoding of independent sequences on the device kernels (the
cached generation of generate_batch, ssd/data/generate_selfdistill.py:64-108).

The reference left-pads a batch to one length and masks the padding out of
every row. Here each sequence owns a range of `region` cache slots; a row of
sequence b sees only the slots of its own range (ssd_tree_attention's
prefix_start / prefix_len), so no padding is stored or read and every row's
positions count from its own first token, exactly the positions the
reference derives from its padding mask. Each step runs one forward over the
B sequences' newest tokens (the GEMMs read every weight once for all B
rows), then one head: the lm_head fused with the argmax (greedy), or fp32
logits and one Gumbel draw per row from the keep_top-largest logits under
temperature and top_p (sample_next, generate_selfdistill.py:51-61), RNG
counter (step, row, token, 0) under the caller's seed.
"""

from __future__ import annotations

from typing import Optional

import torch

from ssd import _lib as L
from ssd import ops
from ssd.models import runner as R


class BatchDecoder:
    def __init__(self, target, batch: int, region: int, max_rows: int):
        self.target = target
        self.w = target.weights
        w = self.w
        if w.tp is not None:
            raise NotImplementedError("batched decoding runs on one GPU")
        self.device = w.device
        self.B, self.region = batch, region
        self.cache = target.new_cache(batch * region)
        self.cache.allocate(w.Hkv, w.hd, w.dtype, w.device)
        self.scratch = R.Scratch(w, max(max_rows, batch))
        self.ws = ops.Workspace(self.device, max_rows=max(max_rows, 64), vocab=w.V, max_head_rows=max(batch, 1))
        self.fwd = R.ForwardInputs(max(max_rows, batch), self.device, mask_words=1)
        self.starts = torch.zeros(max(max_rows, batch), dtype=torch.int32, device=self.device)
        self.fwd.prefix_start = self.starts
        i32 = dict(dtype=torch.int32, device=self.device)
        self.next_tok = torch.zeros(batch, **i32)
        self.logits = None
        self.params = None

    def _forward(self, ids: list, seqs: list, positions: list) -> None:
        """One forward over rows (sequence seqs[i], token ids[i] at position
        positions[i]); row i writes slot seqs[i] * region + positions[i] and sees
        its sequence's slots up to and including that one."""
        T = len(ids)
        reg = self.region
        slots = [s * reg + p for s, p in zip(seqs, positions)]
        f = self.fwd
        host = torch.tensor([ids, positions, slots, [x + 1 for x in slots], [s * reg for s in seqs]],
                            dtype=torch.int32)
        f.ids[:T].copy_(host[0])
        f.positions[:T].copy_(host[1])
        f.slots[:T].copy_(host[2])
        f.prefix_len[:T].copy_(host[3])
        self.starts[:T].copy_(host[4])
        f.use_mask = False
        R.run_stack_auto(self.w, self.target.layer_indices, [None] * len(self.target.layer_indices), None, f, T,
                         self.cache, self.scratch, self.ws, self.cache.max_length)

    def _head(self, r0: int, temperature: float, top_p: float, keep_top: int, seed, step: int) -> list[int]:
        """Next token of each sequence from forward rows r0 .. r0 + B."""
        w, B = self.w, self.B
        xn, rn = R.head_input(w, self.scratch, r0, r0 + B)
        if temperature == 0:
            R.head_argmax(w, xn, w.lm_head, self.next_tok, self.ws, in_norm=rn)
        else:
            if self.logits is None:
                self.logits = torch.zeros(B, w.V, dtype=torch.float32, device=self.device)
                self.params = ops.warp_params_buffer(B, self.device)
            ops.linear(xn, [w.lm_head], self.ws, epilogue=L.EPI_STORE_F32, out=self.logits, T=B, in_norm=rn)
            rnd = torch.tensor([step], dtype=torch.int32, device=self.device)
            ops.warp_sample_topk(self.logits, temperature, top_p, self.params, 1, seed, rnd, 0,
                                 self.next_tok.view(B, 1), None, keep_top=keep_top)
        return self.next_tok.tolist()

    @torch.no_grad()
    def generate(self, prompts: list[list[int]], max_new: int, eos_ids: set[int], temperature: float = 0.0,
                 top_p: float = 1.0, keep_top: int = 64, seed: Optional[int] = None) -> list[list[int]]:
        """New tokens per sequence (uncut; the caller cuts after EOS). The
        loop ends when every sequence has produced an EOS or max_new tokens."""
        B = len(prompts)
        if B != self.B:
            raise ValueError(f"decoder built for {self.B} sequences, got {B}")
        lens = [len(p) for p in prompts]
        if max(lens) + max_new > self.region:
            raise RuntimeError("prompt + new tokens exceed the sequence's cache range")
        seed_t = None
        if temperature > 0:
            from ssd.engine.sampling import _as_i64, seed_from

            seed_t = torch.tensor([_as_i64(seed_from(seed))], dtype=torch.int64, device=self.device)
        self.cache.reset()
        # prefill: every prompt token but each sequence's last, then the B last
        # tokens, whose rows feed the head
        ids, seqs, pos = [], [], []
        for b, p in enumerate(prompts):
            ids += p[:-1]
            seqs += [b] * (len(p) - 1)
            pos += list(range(len(p) - 1))
        r0 = len(ids)
        ids += [p[-1] for p in prompts]
        seqs += list(range(B))
        pos += [n - 1 for n in lens]
        self._forward(ids, seqs, pos)
        out = [[t] for t in self._head(r0, temperature, top_p, keep_top, seed_t, 0)]
        done = [t in eos_ids for t in (o[0] for o in out)]
        for step in range(1, max_new):
            if all(done):
                break
            self._forward([o[-1] for o in out], list(range(B)), [n - 1 + step for n in lens])
            nxt = self._head(0, temperature, top_p, keep_top, seed_t, step)
            for b in range(B):
                out[b].append(nxt[b])
                done[b] = done[b] or nxt[b] in eos_ids
        self.ws.check_status()
        return out
