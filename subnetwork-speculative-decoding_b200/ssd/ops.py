"""Tensor-level wrappers over the C ABI (include/ssd_b200.h).

Each function takes torch CUDA tensors, checks shapes/dtypes, and launches
on the current torch stream. Nothing here computes on the host: a missing
library or a non-CUDA tensor is an error.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from ssd import _lib as L

_DT = {torch.float32: L.SSD_F32, torch.bfloat16: L.SSD_BF16}


def dtype_code(dt: torch.dtype) -> int:
    if dt not in _DT:
        raise ValueError(f"unsupported dtype {dt} (float32 or bfloat16)")
    return _DT[dt]


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("SSD B200 ops take CUDA tensors only (no CPU fallback)")
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def launch_count() -> int:
    return L.launch_count()


class Workspace:
    """Scratch for the GEMM / attention / head kernels plus a device status word.

    The buffer is zeroed once; the kernels' split counters reset themselves.
    One workspace per stream.
    """

    def __init__(self, device: torch.device, max_rows: int, vocab: int, max_head_rows: Optional[int] = None):
        L.load()
        head_rows = max_rows if max_head_rows is None else max_head_rows
        nbytes = int(L.load().ssd_workspace_bytes(max(1, max_rows), max(1, head_rows), max(1, vocab)))
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.nbytes = nbytes

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def check_status(self) -> None:
        """Raise if any kernel recorded a device-side error (bad index, timeout)."""
        v = int(self.status.item())
        if v:
            self.status.zero_()
            what = []
            if v & 1:
                what.append("a pipeline wait timed out")
            if v & 2:
                what.append("an index was out of range")
            raise RuntimeError("SSD device error: " + ", ".join(what))


class NormOut:
    """Next RMSNorm input produced by a residual-updating kernel (SsdNormOut):
    out[t, n] = resid[t, n] * weight[n] (bf16) and ssq[t, i] = sum of squares
    of resid[t, :] over the i-th 128-feature tile."""

    def __init__(self, weight: torch.Tensor, out: torch.Tensor, ssq: torch.Tensor):
        self.weight, self.out, self.ssq = weight, out, ssq

    def c(self):
        return C.byref(L.SsdNormOut(_p(self.weight), _p(self.out), self.out.stride(0), _p(self.ssq),
                                    self.ssq.stride(0)))


class RowNorm:
    """RMSNorm completed inside a GEMM (SsdRowNorm): output column t is scaled
    by rsqrt(sum(ssq[t, :parts]) / d + eps)."""

    def __init__(self, ssq: torch.Tensor, parts: int, d: int, eps: float):
        self.ssq, self.parts, self.d, self.eps = ssq, parts, d, float(eps)

    def rows(self, r0: int, r1: int) -> "RowNorm":
        return RowNorm(self.ssq[r0:r1], self.parts, self.d, self.eps)

    def c(self):
        return C.byref(L.SsdRowNorm(_p(self.ssq), self.ssq.stride(0), self.parts, self.d, self.eps))


def _c(x):
    return None if x is None else x.c()


def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor, ws: Workspace,
          norm_out: Optional[NormOut] = None) -> None:
    T = ids.numel()
    L.call("ssd_embed", _p(ids), T, _p(table), table.shape[0], table.shape[1], dtype_code(table.dtype), _p(out),
           _c(norm_out), _p(ws.status), _stream())


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor) -> None:
    T, d = x.shape
    L.call("ssd_rmsnorm", _p(x), T, d, x.stride(0), _p(weight), float(eps), _p(out), out.stride(0),
           dtype_code(out.dtype), _stream())


def linear(x: torch.Tensor, weights: Sequence[torch.Tensor], ws: Workspace, *, biases: Sequence = (),
           epilogue: int = L.EPI_STORE, act: str = "none", layout: int = L.SEG_CONCAT,
           out: Optional[torch.Tensor] = None, resid: Optional[torch.Tensor] = None, T: Optional[int] = None,
           in_norm: Optional[RowNorm] = None, norm_out: Optional[NormOut] = None) -> None:
    """out/resid <- epilogue(x @ cat(weights)^T + bias). x: [T, K] in the weights' dtype."""
    T = x.shape[0] if T is None else T
    K = weights[0].shape[1]
    n = len(weights)
    for w in weights:
        if w.shape[1] != K or not w.is_contiguous():
            raise ValueError("weight segments must be contiguous [rows, K]")
    wp = (C.c_void_p * 3)(*[w.data_ptr() for w in weights], *([None] * (3 - n)))
    rows = (C.c_int64 * 3)(*[w.shape[0] for w in weights], *([0] * (3 - n)))
    bl = list(biases) + [None] * (3 - len(biases))
    bp = (C.c_void_p * 3)(*[(b.data_ptr() if b is not None else None) for b in bl[:3]])
    L.call("ssd_linear", _p(x), x.stride(0), T, K, n, wp, rows, bp, layout, epilogue, L.ACT[act],
           _p(out), out.stride(0) if out is not None else 0, _p(resid), resid.stride(0) if resid is not None else 0,
           dtype_code(weights[0].dtype), ws.ptr, ws.nbytes, _c(in_norm), _c(norm_out), _p(ws.status), _stream())


def _norm_fields(a, in_norm: Optional[RowNorm], norm_out: Optional[NormOut]) -> None:
    if in_norm is not None:
        a.in_norm = L.SsdRowNorm(_p(in_norm.ssq), in_norm.ssq.stride(0), in_norm.parts, in_norm.d, in_norm.eps)
    if norm_out is not None:
        a.norm_out = L.SsdNormOut(_p(norm_out.weight), _p(norm_out.out), norm_out.out.stride(0), _p(norm_out.ssq),
                                  norm_out.ssq.stride(0))


def linear_args(x: torch.Tensor, weights: Sequence[torch.Tensor], *, biases: Sequence = (),
                epilogue: int = L.EPI_STORE, act: str = "none", layout: int = L.SEG_CONCAT,
                out: Optional[torch.Tensor] = None, resid: Optional[torch.Tensor] = None,
                in_norm: Optional[RowNorm] = None, norm_out: Optional[NormOut] = None) -> L.SsdLinearArgs:
    """One ssd_linear_chain link with linear()'s arguments."""
    K = weights[0].shape[1]
    for w in weights:
        if w.shape[1] != K or not w.is_contiguous():
            raise ValueError("weight segments must be contiguous [rows, K]")
    a = L.SsdLinearArgs()
    a.x, a.ldx, a.K, a.n_seg, a.seg_layout = _p(x), x.stride(0), K, len(weights), layout
    for i, w in enumerate(weights):
        a.w[i], a.rows[i] = w.data_ptr(), w.shape[0]
    for i, b in enumerate(list(biases)[:3]):
        a.bias[i] = b.data_ptr() if b is not None else None
    a.epilogue, a.act = epilogue, L.ACT[act]
    if out is not None:
        a.out, a.ldo = _p(out), out.stride(0)
    if resid is not None:
        a.resid, a.ldr = _p(resid), resid.stride(0)
    _norm_fields(a, in_norm, norm_out)
    return a


def qkv_args(x, wq, wk, wv, n_heads, n_kv, head_dim, cos, sin, positions, slots, k_cache, v_cache, q_out,
             in_norm: Optional[RowNorm] = None) -> L.SsdLinearArgs:
    """One ssd_linear_chain link with qkv_rope()'s arguments."""
    a = L.SsdLinearArgs()
    a.x, a.ldx, a.K, a.epilogue = _p(x), x.stride(0), wq.shape[1], L.EPI_QKV
    for i, w in enumerate((wq, wk, wv)):
        a.w[i] = _p(w)
    a.out, a.ldo = _p(q_out), q_out.stride(0)
    a.n_heads, a.n_kv_heads, a.head_dim = n_heads, n_kv, head_dim
    a.rope_cos, a.rope_sin, a.max_pos = _p(cos), _p(sin), cos.shape[0]
    a.positions, a.slots = _p(positions), _p(slots)
    a.k_cache, a.v_cache, a.cache_head_stride, a.max_slots = _p(k_cache), _p(v_cache), k_cache.stride(0), \
        k_cache.shape[1]
    _norm_fields(a, in_norm, None)
    return a


def linear_chain(links: Sequence[L.SsdLinearArgs], T: int, ws: Workspace) -> None:
    """Run up to CHAIN_MAX dependent GEMM links over T <= 64 rows in one
    persistent launch (ssd_linear_chain)."""
    n = len(links)
    arr = (L.SsdLinearArgs * n)(*links)
    L.call("ssd_linear_chain", n, C.cast(arr, C.c_void_p), T, L.SSD_BF16, ws.ptr, ws.nbytes, _p(ws.status),
           _stream())


class GemmChain:
    """Collects the GEMMs between two non-GEMM kernels of a bf16 decode
    forward and launches them as ssd_linear_chain links (at most CHAIN_MAX
    per launch); with `enabled` False every call launches on its own."""

    def __init__(self, ws: Workspace, T: int, enabled: bool):
        self.ws, self.T, self.enabled = ws, T, enabled and 1 <= T <= 64
        self.links: list = []

    def linear(self, x, weights, **kw) -> None:
        if not self.enabled:
            linear(x, weights, self.ws, T=self.T, **kw)
            return
        self._add(linear_args(x, weights, **kw))

    def qkv(self, x, wq, wk, wv, n_heads, n_kv, head_dim, cos, sin, positions, slots, k_cache, v_cache, q_out,
            in_norm=None) -> None:
        if not self.enabled:
            qkv_rope(x, wq, wk, wv, n_heads, n_kv, head_dim, cos, sin, positions, slots, k_cache, v_cache, q_out,
                     self.ws, T=self.T, in_norm=in_norm)
            return
        self._add(qkv_args(x, wq, wk, wv, n_heads, n_kv, head_dim, cos, sin, positions, slots, k_cache, v_cache,
                           q_out, in_norm=in_norm))

    def _add(self, a) -> None:
        self.links.append(a)
        if len(self.links) == L.CHAIN_MAX:
            self.flush()

    def flush(self) -> None:
        if self.links:
            linear_chain(self.links, self.T, self.ws)
            self.links = []


def qkv_rope(x, wq, wk, wv, n_heads, n_kv, head_dim, cos, sin, positions, slots, k_cache, v_cache, q_out,
             ws: Workspace, T: Optional[int] = None, in_norm: Optional[RowNorm] = None) -> None:
    """k_cache/v_cache: [n_kv, max_slots, head_dim] views of one layer."""
    T = x.shape[0] if T is None else T
    L.call("ssd_qkv_rope", _p(x), x.stride(0), T, wq.shape[1], _p(wq), _p(wk), _p(wv), n_heads, n_kv, head_dim,
           _p(cos), _p(sin), cos.shape[0], _p(positions), _p(slots), _p(k_cache), _p(v_cache), k_cache.stride(0),
           k_cache.shape[1], _p(q_out), q_out.stride(0), dtype_code(wq.dtype), ws.ptr, ws.nbytes, _c(in_norm),
           _p(ws.status), _stream())


def tree_attention(q, k_cache, v_cache, n_heads, n_kv, head_dim, prefix_len, out, ws: Workspace, *,
                   spec_base=None, spec_mask=None, kv_bound: int = 0, T: Optional[int] = None,
                   prefix_start=None) -> None:
    """Row t attends slots [prefix_start[t] (0 if None), prefix_len[t]) plus its
    speculative mask bits (ssd_tree_attention)."""
    T = q.shape[0] if T is None else T
    mw = spec_mask.shape[-1] if spec_mask is not None else 0
    L.call("ssd_tree_attention", _p(q), q.stride(0), T, n_heads, n_kv, head_dim, _p(k_cache), _p(v_cache),
           k_cache.stride(0), k_cache.shape[1], _p(prefix_len), _p(prefix_start), _p(spec_base), _p(spec_mask), mw,
           kv_bound, _p(out), out.stride(0), dtype_code(q.dtype), ws.ptr, ws.nbytes, _p(ws.status), _stream())


def head_argmax(x, w, out_idx, ws: Workspace, out_max=None, out_gap=None, T: Optional[int] = None,
                in_norm: Optional[RowNorm] = None) -> None:
    T = x.shape[0] if T is None else T
    L.call("ssd_head_argmax", _p(x), x.stride(0), T, w.shape[1], _p(w), w.shape[0], _p(out_idx), _p(out_max),
           _p(out_gap), dtype_code(w.dtype), ws.ptr, ws.nbytes, _c(in_norm), _p(ws.status), _stream())


def head_topk(x, w, k: int, out_tok, out_lp, ws: Workspace, vocab_ids=None, T: Optional[int] = None,
              in_norm: Optional[RowNorm] = None) -> None:
    T = x.shape[0] if T is None else T
    L.call("ssd_head_topk", _p(x), x.stride(0), T, w.shape[1], _p(w), w.shape[0], _p(vocab_ids), k, _p(out_tok),
           _p(out_lp), dtype_code(w.dtype), ws.ptr, ws.nbytes, _c(in_norm), _p(ws.status), _stream())


def level_prune(topk_tok, topk_lp, n_frontier, k, width, level, frontier, next_frontier, tree, root_pos, fed,
                level_slot_offset, fwd, status) -> None:
    """tree: DeviceTree; fwd: ForwardInputs (or None when not fed)."""
    L.call("ssd_level_prune", _p(topk_tok), _p(topk_lp), n_frontier, k, width if width else 0, level, _p(frontier),
           _p(next_frontier), _p(tree.n_nodes), _p(tree.tokens), _p(tree.parents), _p(tree.depths), _p(tree.ranks),
           _p(tree.scores), _p(tree.draft_pos), tree.cap, _p(root_pos), 1 if fed else 0, level_slot_offset,
           _p(fwd.ids) if fed else None, _p(fwd.positions) if fed else None, _p(fwd.slots) if fed else None,
           _p(fwd.prefix_len) if fed else None, _p(fwd.spec_base) if fed else None, _p(fwd.mask) if fed else None,
           fwd.mask_words if fed else 0, _p(status), _stream())


def tree_prune(tree, max_nodes: Optional[int]) -> None:
    L.call("ssd_tree_prune", _p(tree.n_nodes), max_nodes or 0, _p(tree.tokens), _p(tree.parents), _p(tree.depths),
           _p(tree.ranks), _p(tree.scores), _p(tree.draft_pos), tree.cap, _stream())


def verify_prep(tree, rows_cap, root_token, root_pos, fwd, status) -> None:
    L.call("ssd_verify_prep", _p(tree.n_nodes), rows_cap, _p(root_token), _p(root_pos), _p(tree.tokens),
           _p(tree.parents), _p(tree.depths), _p(fwd.ids), _p(fwd.positions), _p(fwd.slots), _p(fwd.prefix_len),
           _p(fwd.spec_base), _p(fwd.mask), fwd.mask_words, _p(status), _stream())


def tree_walk_greedy(tree, argmax, root_pos, accepted, n_accepted, bonus, keep_slots, n_keep, max_nodes) -> None:
    L.call("ssd_tree_walk_greedy", _p(tree.n_nodes), max_nodes, _p(argmax), _p(tree.tokens), _p(tree.parents), _p(tree.ranks),
           _p(root_pos), _p(accepted), _p(n_accepted), _p(bonus), _p(keep_slots), _p(n_keep), _stream())


def kv_compact(cache: torch.Tensor, start, keep_slots, n_keep, max_keep: int, status=None) -> None:
    """cache: [L, 2, n_kv, max_slots, head_dim]. A keep list that does not fit
    sets the bad-index bit of `status` (a workspace's status word)."""
    Ln, _, n_kv, _, hd = cache.shape
    L.call("ssd_kv_compact", _p(cache), Ln, cache.stride(0), cache.stride(1), n_kv, cache.stride(2), hd, _p(start),
           _p(keep_slots), _p(n_keep), max_keep, dtype_code(cache.dtype), _p(status), _stream())


def round_commit(n_accepted, accepted, tokens, bonus, seq_len, root_token, out_tokens, n_out, round_log,
                 status) -> None:
    L.call("ssd_round_commit", _p(n_accepted), _p(accepted), _p(tokens), _p(bonus), _p(seq_len), _p(root_token),
           _p(out_tokens), _p(n_out), out_tokens.numel(), _p(round_log), _p(status), _stream())


def causal_prep(base, T: int, src_ids, fwd) -> None:
    L.call("ssd_causal_prep", _p(base), T, _p(src_ids), _p(fwd.ids), _p(fwd.positions), _p(fwd.slots),
           _p(fwd.prefix_len), _stream())


# ------------------------------------------------------------------ sampling
def warp_params_buffer(rows: int, device) -> torch.Tensor:
    """Storage for `rows` warp-parameter records {max, 1/T, lambda, log Z}."""
    return torch.zeros(max(1, rows), 4, dtype=torch.float32, device=device)


def warp_params(logits: torch.Tensor, temperature: float, top_p: float, out: torch.Tensor,
                rows: Optional[int] = None, V: Optional[int] = None) -> None:
    """Warp parameters of fp32 logit rows [rows, V] (warp_probs, tree_drafter.py:34-45)."""
    rows = logits.shape[0] if rows is None else rows
    V = logits.shape[1] if V is None else V
    if logits.dtype != torch.float32 or out.shape[0] < rows:
        raise ValueError("warp_params: fp32 logits and a params buffer of >= rows records")
    L.call("ssd_warp_params", _p(logits), logits.stride(0), rows, V, float(temperature), float(top_p), _p(out),
           _stream())


def warp_probs(logits: torch.Tensor, params: torch.Tensor, out: torch.Tensor, rows: Optional[int] = None) -> None:
    """Warped probabilities (warp_probs, tree_drafter.py:34-45) from warp parameters."""
    rows = logits.shape[0] if rows is None else rows
    L.call("ssd_warp_probs", _p(logits), logits.stride(0), rows, logits.shape[1], _p(params), _p(out), out.stride(0),
           _stream())


def gumbel_topk(logits: torch.Tensor, params: torch.Tensor, k: int, seed: torch.Tensor, round_: Optional[torch.Tensor],
                row_base: int, out_tok: torch.Tensor, out_lp: torch.Tensor, vocab_ids=None,
                rows: Optional[int] = None) -> None:
    """k draws without replacement per row, in draw order (tree_drafter.py:134-145)."""
    rows = logits.shape[0] if rows is None else rows
    L.call("ssd_gumbel_topk", _p(logits), logits.stride(0), rows, logits.shape[1], _p(params), k, _p(vocab_ids),
           _p(seed), _p(round_), row_base, _p(out_tok), _p(out_lp), _stream())


def warp_sample_topk(logits: torch.Tensor, temperature: float, top_p: float, params_out: Optional[torch.Tensor],
                     k: int = 0, seed: Optional[torch.Tensor] = None, round_: Optional[torch.Tensor] = None,
                     row_base: int = 0, out_tok: Optional[torch.Tensor] = None, out_lp: Optional[torch.Tensor] = None,
                     vocab_ids=None, rows: Optional[int] = None, keep_top: int = 0) -> None:
    """Fused warp parameters + k Gumbel draws per row on one cluster per row
    (ssd_warp_sample_topk; k = 0: parameters only; keep_top > 0: only the
    keep_top largest logits of a row take part)."""
    rows = logits.shape[0] if rows is None else rows
    if logits.dtype != torch.float32 or (params_out is not None and params_out.shape[0] < rows):
        raise ValueError("warp_sample_topk: fp32 logits and a params buffer of >= rows records")
    L.call("ssd_warp_sample_topk", _p(logits), logits.stride(0), rows, logits.shape[1], float(temperature),
           float(top_p), keep_top, k, _p(vocab_ids), _p(seed), _p(round_), row_base, _p(params_out), _p(out_tok), _p(out_lp),
           _stream())


def sample_token(logits: torch.Tensor, temperature: float, top_p: float, seed: torch.Tensor,
                 round_: Optional[torch.Tensor], row_id: int, stream_id: int, scratch: torch.Tensor,
                 out: torch.Tensor) -> None:
    """out[0] ~ warp(logits) (_first_token, speculative.py:81-84)."""
    L.call("ssd_sample_token", _p(logits), logits.shape[-1], float(temperature), float(top_p), _p(seed), _p(round_),
           row_id, stream_id, _p(scratch), _p(out), _stream())


def tree_walk_sample(tree, tlogits, tparams, dlogits, dparams, draft_rows: int, seed, round_, p_scratch, q_scratch,
                     root_pos, accepted, n_accepted, bonus, keep_slots, n_keep, max_nodes: int, status,
                     vocab_ids=None) -> None:
    """sample_verify (verify.py:60-95) over the device tree."""
    L.call("ssd_tree_walk_sample", _p(tree.n_nodes), max_nodes, _p(tree.tokens), _p(tree.parents), _p(tree.ranks),
           _p(tree.draft_pos), _p(root_pos), _p(tlogits), tlogits.stride(0), _p(tparams), tlogits.shape[1],
           _p(dlogits), dlogits.stride(0), _p(dparams), draft_rows, dlogits.shape[1], _p(vocab_ids), _p(seed),
           _p(round_), _p(p_scratch), _p(q_scratch), _p(accepted), _p(n_accepted), _p(bonus), _p(keep_slots),
           _p(n_keep), _p(status), _stream())


# ------------------------------------------------------------ tensor parallel
def fill_normal(out: torch.Tensor, row0: int, col0: int, full_cols: int, seed: int, stream_id: int, std: float,
                scale: float = 1.0) -> None:
    """out (2-D, contiguous rows) <- block [row0:, col0:] of a seeded N(0, std^2) * scale global matrix."""
    t = out if out.dim() == 2 else out.view(1, -1)
    L.call("ssd_fill_normal", _p(t), t.shape[0], t.shape[1], t.stride(0), row0, col0, full_cols,
           seed & (2 ** 64 - 1), stream_id & (2 ** 64 - 1), float(std), float(scale), dtype_code(t.dtype), _stream())


def tp_allreduce_residual(group, parity: int, T: int, resid: torch.Tensor, ws: Workspace,
                          norm_out: Optional[NormOut] = None, dtype: torch.dtype = torch.bfloat16) -> None:
    """resid[:T] += all-reduced partials (buffer `parity`) of the group (see ssd_tp_allreduce_residual)."""
    L.call("ssd_tp_allreduce_residual", group.ref(), parity, T, _p(resid), resid.stride(0), _c(norm_out),
           dtype_code(dtype), _p(ws.status), _stream())


def tp_head_argmax(group, x, w_shard, vocab_offset: int, out_idx, ws: Workspace, out_max=None, out_gap=None,
                   T: Optional[int] = None, in_norm: Optional[RowNorm] = None) -> None:
    T = x.shape[0] if T is None else T
    L.call("ssd_tp_head_argmax", group.ref(), _p(x), x.stride(0), T, w_shard.shape[1], _p(w_shard), w_shard.shape[0],
           vocab_offset, _p(out_idx), _p(out_max), _p(out_gap), dtype_code(w_shard.dtype), ws.ptr, ws.nbytes,
           _c(in_norm), _p(ws.status), _stream())


def tp_head_topk(group, x, w_shard, vocab_offset: int, k: int, out_tok, out_lp, ws: Workspace, vocab_ids=None,
                 T: Optional[int] = None, in_norm: Optional[RowNorm] = None) -> None:
    T = x.shape[0] if T is None else T
    L.call("ssd_tp_head_topk", group.ref(), _p(x), x.stride(0), T, w_shard.shape[1], _p(w_shard), w_shard.shape[0],
           vocab_offset, _p(vocab_ids), k, _p(out_tok), _p(out_lp), dtype_code(w_shard.dtype), ws.ptr, ws.nbytes,
           _c(in_norm), _p(ws.status), _stream())
