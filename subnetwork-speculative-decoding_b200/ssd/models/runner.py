"""Kernel-driven forward of a base-layer subset plus bridges over the shared
KV cache: the B200 replacement of SubnetworkDraftModel.forward's cache branch
(ssd/models/subnetwork_draft.py:249-357, _layer_forward :193-246).

Per layer (all launches on the current stream, no host syncs):
  rmsnorm -> QKV GEMM (+RoPE, K/V written into the cache) -> tree attention
  -> o_proj GEMM (+residual) -> rmsnorm -> gate/up GEMM (+SwiGLU)
  -> down GEMM (+residual)
The residual stream is fp32; GEMM operands use the weights' dtype (bf16:
tcgen05 tensor cores, fp32: CUDA cores). Every buffer is allocated once and
reused, so a forward can be captured in a CUDA graph.
"""

from __future__ import annotations

import os

from dataclasses import dataclass
from typing import Optional

import torch

from ssd import _lib as L
from ssd import ops


@dataclass
class LayerW:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    o: torch.Tensor
    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    ln1: torch.Tensor
    ln2: torch.Tensor
    eps1: float
    eps2: float


class ModelWeights:
    """References (never copies) the base model's tensors; builds the RoPE
    tables once. Cached on the base module."""

    def __init__(self, base):
        cfg = base.config
        inner = base.model
        self.config = cfg
        self.d = cfg.hidden_size
        self.H = cfg.num_attention_heads
        self.Hkv = cfg.num_key_value_heads
        self.hd = getattr(cfg, "head_dim", None) or self.d // self.H
        self.F = cfg.intermediate_size
        self.V = cfg.vocab_size
        self.L = cfg.num_hidden_layers
        self.tp = None  # tensor-parallel group (ssd.engine.tp.attach)
        self.vocab_offset = 0  # first lm_head row of this rank's shard
        self.embed = inner.embed_tokens.weight
        self.lm_head = base.lm_head.weight
        self.norm = inner.norm.weight
        self.norm_eps = float(getattr(inner.norm, "variance_epsilon", cfg.rms_norm_eps))
        self.dtype = self.embed.dtype
        self.device = self.embed.device
        if self.device.type != "cuda":
            raise ValueError("the B200 path needs the base model on a CUDA device (no CPU fallback)")
        self.layers = []
        for lyr in inner.layers:
            at, mlp = lyr.self_attn, lyr.mlp
            for lin in (at.q_proj, at.k_proj, at.v_proj, at.o_proj, mlp.gate_proj, mlp.up_proj, mlp.down_proj):
                if getattr(lin, "bias", None) is not None:
                    raise ValueError("attention/MLP biases are not supported by the B200 layer kernels")
            self.layers.append(LayerW(
                at.q_proj.weight, at.k_proj.weight, at.v_proj.weight, at.o_proj.weight, mlp.gate_proj.weight,
                mlp.up_proj.weight, mlp.down_proj.weight, lyr.input_layernorm.weight,
                lyr.post_attention_layernorm.weight,
                float(getattr(lyr.input_layernorm, "variance_epsilon", cfg.rms_norm_eps)),
                float(getattr(lyr.post_attention_layernorm, "variance_epsilon", cfg.rms_norm_eps))))
        for t in [self.embed, self.lm_head, self.norm] + [x for lw in self.layers for x in
                                                          (lw.q, lw.k, lw.v, lw.o, lw.gate, lw.up, lw.down)]:
            if t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError("base weights must share one dtype and be contiguous")
        self._rope(base)

    def _rope(self, base) -> None:
        """cos/sin tables [max_pos, head_dim/2] in fp32, computed on the CPU the
        way HF's rotary embedding does (fp32 inv_freq x position)."""
        rot = getattr(base.model, "rotary_emb", None)
        if rot is not None and hasattr(rot, "inv_freq"):
            inv = rot.inv_freq.detach().float().cpu()
            scale = float(getattr(rot, "attention_scaling", 1.0))
        else:
            from ssd.synthetic import rope_theta

            theta = rope_theta(self.config)
            inv = 1.0 / (theta ** (torch.arange(0, self.hd, 2, dtype=torch.int64).float() / self.hd))
            scale = 1.0
        max_pos = int(min(getattr(self.config, "max_position_embeddings", 8192), 131072))
        self.max_pos = max_pos
        f = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
        self.rope_cos = (f.cos() * scale).to(self.device)
        self.rope_sin = (f.sin() * scale).to(self.device)

    @staticmethod
    def of(base) -> "ModelWeights":
        w = getattr(base, "_ssd_b200_weights", None)
        if w is None:
            w = ModelWeights(base)
            object.__setattr__(base, "_ssd_b200_weights", w)
        return w


class ForwardInputs:
    """Device-side inputs of one forward over up to `cap` rows: token ids,
    RoPE positions, cache slots written, contiguous prefix length per row and
    the ancestor bitmask over speculative slots starting at spec_base; for
    batched forwards (several sequences, each in its own slot range) also the
    first visible slot per row (prefix_start, else None: slot 0)."""

    def __init__(self, cap: int, device, mask_words: int = 2):
        self.cap = cap
        self.mask_words = mask_words
        i32 = dict(dtype=torch.int32, device=device)
        self.ids = torch.zeros(cap, **i32)
        self.positions = torch.zeros(cap, **i32)
        self.slots = torch.zeros(cap, **i32)
        self.prefix_len = torch.ones(cap, **i32)
        self.spec_base = torch.zeros(1, **i32)
        self.mask = torch.zeros(cap, mask_words, dtype=torch.int64, device=device)
        self.use_mask = False
        self.prefix_start = None

    def fill(self, ids, positions, past: int, tree_mask: Optional[torch.Tensor]) -> None:
        """Host-side fill for the API path (reference mask semantics of
        subnetwork_draft.py:165-191): causal when tree_mask is None, else the
        mask's all-True leading columns become the prefix and the remaining
        columns the per-row bitmask."""
        T = int(ids.numel())
        if T > self.cap:
            raise ValueError(f"forward of {T} rows exceeds the buffer capacity {self.cap}")
        dev = self.ids.device
        self.ids[:T].copy_(ids.reshape(-1).to(dev, torch.int32), non_blocking=True)
        self.positions[:T].copy_(positions.reshape(-1).to(dev, torch.int32), non_blocking=True)
        self.slots[:T].copy_(torch.arange(past, past + T, dtype=torch.int32), non_blocking=False)
        if tree_mask is None:
            self.prefix_len[:T].copy_(torch.arange(past + 1, past + T + 1, dtype=torch.int32) if T > 1 else
                                      torch.tensor([past + 1], dtype=torch.int32))
            self.use_mask = False
            return
        m = tree_mask.to("cpu", torch.bool)
        while m.dim() > 2:
            if m.shape[0] != 1:
                raise ValueError("tree_attention_mask must describe batch size 1")
            m = m[0]
        S = past + T
        if m.shape[-1] == S and past > 0:
            full = m
        elif m.shape[-2:] == (T, T):
            full = torch.cat([torch.ones(T, past, dtype=torch.bool), m], dim=-1)
        else:
            raise ValueError(f"tree_attention_mask must be [.., {T}, {T}] or [.., {T}, {S}], got {tuple(m.shape)}")
        allcols = full.all(dim=0)
        P = int(allcols.long().cumprod(0).sum())
        width = S - P
        if width > 64 * self.mask_words:
            raise ValueError(f"tree mask spans {width} speculative slots (max {64 * self.mask_words})")
        bits = torch.zeros(T, self.mask_words, dtype=torch.int64)
        sub = full[:, P:]
        for j in range(width):
            col = sub[:, j].to(torch.int64)
            w, b = divmod(j, 64)
            val = (col << b) if b < 63 else torch.where(col.bool(), torch.tensor(-(1 << 63)), torch.tensor(0))
            bits[:, w] |= val
        self.prefix_len[:T].fill_(P)
        self.spec_base.fill_(P)
        self.mask[:T].copy_(bits)
        self.use_mask = width > 0


def norm_parts(w) -> int:
    """Partial sums of squares per row (one per 128-feature tile)."""
    return (w.d + 127) // 128


def folds_norms(w) -> bool:
    """bf16 forwards fold every RMSNorm into the GEMMs next to it: the
    residual-updating epilogue writes resid * w_norm and per-tile sums of
    squares, the consuming GEMM scales each token by rsqrt(mean + eps). The
    fp32 tier keeps the standalone RMSNorm kernel, whose rounding follows the
    reference's exactly."""
    return w.dtype == torch.bfloat16


class Scratch:
    """Persistent activation buffers for forwards of up to `rows` rows."""

    def __init__(self, w: ModelWeights, rows: int):
        self.w = w
        self.rows = rows
        dev = w.device
        self.resid = torch.zeros(rows, w.d, dtype=torch.float32, device=dev)
        # per-row partial sums of squares (one per 128 features) for the
        # RMSNorms folded into the GEMMs
        self.ssq = torch.zeros(rows, norm_parts(w), dtype=torch.float32, device=dev)
        self.q = torch.zeros(rows, w.H * w.hd, dtype=w.dtype, device=dev)
        self.attn = torch.zeros(rows, w.H * w.hd, dtype=w.dtype, device=dev)
        self._xn: dict = {}
        self._hid: dict = {}
        self.width = max(w.d, w.F)

    def xn(self, dtype: torch.dtype, cols: int) -> torch.Tensor:
        t = self._xn.get(dtype)
        if t is None or t.shape[1] < cols:
            t = torch.zeros(self.rows, max(cols, self.w.d), dtype=dtype, device=self.w.device)
            self._xn[dtype] = t
        return t

    def hid(self, dtype: torch.dtype, cols: int, which: int = 0) -> torch.Tensor:
        key = (dtype, which)
        t = self._hid.get(key)
        if t is None or t.shape[1] < cols:
            t = torch.zeros(self.rows, max(cols, self.w.F), dtype=dtype, device=self.w.device)
            self._hid[key] = t
        return t

    def reserve_bridges(self, bridges) -> None:
        """Allocate bridge buffers up front (before any graph capture)."""
        for b in bridges:
            dt = b.norm.weight.dtype
            self.xn(dt, self.w.d)
            self.hid(dt, b.hidden, 0)
            self.hid(dt, b.hidden, 1)


def _seg_linear(x, weights, ws, **kw):
    ops.linear(x, weights, ws, **kw)


def run_bridge(bridge, scratch: Scratch, T: int, ws: ops.Workspace) -> None:
    """TransitionBridge forward x + MLP(RMSNorm(x)) on the fp32 residual
    stream (ssd/models/bridges.py:131-135) in the bridge's parameter dtype."""
    dt = bridge.norm.weight.dtype
    xn = scratch.xn(dt, scratch.w.d)[:T]
    ops.rmsnorm(scratch.resid[:T], bridge.norm.weight, bridge.norm.eps, xn)
    mlp = bridge.mlp
    if bridge.mlp_type == "swiglu":
        h = scratch.hid(dt, bridge.hidden, 0)[:T, : bridge.hidden]
        ops.linear(xn, [mlp.gate_proj.weight, mlp.up_proj.weight], ws,
                   biases=[mlp.gate_proj.bias, mlp.up_proj.bias], epilogue=L.EPI_SWIGLU, layout=L.SEG_PAIRS, out=h)
    else:
        h = xn
        for i, lin in enumerate(mlp.linears()):
            nxt = scratch.hid(dt, bridge.hidden, i % 2)[:T, : lin.weight.shape[0]]
            ops.linear(h, [lin.weight], ws, biases=[lin.bias], act=bridge.activation, out=nxt)
            h = nxt
    ops.linear(h, [mlp.out_proj.weight], ws, biases=[mlp.out_proj.bias], epilogue=L.EPI_RESIDUAL,
               resid=scratch.resid[:T])


def run_layer(w: ModelWeights, li: int, fwd: ForwardInputs, T: int, cache, scratch: Scratch, ws: ops.Workspace,
              kv_bound: int) -> None:
    """One decoder layer (subnetwork_draft.py:193-246) through the kernels."""
    lw = w.layers[li]
    kc, vc = cache.layer(li)
    xn = scratch.xn(w.dtype, w.d)[:T, : w.d]
    resid = scratch.resid[:T]
    ops.rmsnorm(resid, lw.ln1, lw.eps1, xn)
    ops.qkv_rope(xn, lw.q, lw.k, lw.v, w.H, w.Hkv, w.hd, w.rope_cos, w.rope_sin, fwd.positions, fwd.slots, kc, vc,
                 scratch.q[:T], ws, T=T)
    ops.tree_attention(scratch.q[:T], kc, vc, w.H, w.Hkv, w.hd, fwd.prefix_len, scratch.attn[:T], ws,
                       spec_base=fwd.spec_base if fwd.use_mask else None, spec_mask=fwd.mask if fwd.use_mask else None,
                       kv_bound=kv_bound, T=T, prefix_start=fwd.prefix_start)
    ops.linear(scratch.attn[:T], [lw.o], ws, epilogue=L.EPI_RESIDUAL, resid=resid)
    ops.rmsnorm(resid, lw.ln2, lw.eps2, xn)
    hid = scratch.hid(w.dtype, w.F, 0)[:T, : w.F]
    ops.linear(xn, [lw.gate, lw.up], ws, epilogue=L.EPI_SWIGLU, layout=L.SEG_PAIRS, out=hid)
    ops.linear(hid, [lw.down], ws, epilogue=L.EPI_RESIDUAL, resid=resid)


def run_stack(w: ModelWeights, layer_indices, pre_layer_bridges, pre_norm_bridge, fwd: ForwardInputs, T: int, cache,
              scratch: Scratch, ws: ops.Workspace, kv_bound: int, embeds: Optional[torch.Tensor] = None) -> None:
    """Embedding -> [bridge] -> layer ... -> [bridge]; leaves the pre-norm
    hidden state in scratch.resid[:T]."""
    if T > scratch.rows:
        raise ValueError(f"forward of {T} rows exceeds the scratch capacity {scratch.rows}")
    if embeds is None:
        ops.embed(fwd.ids[:T], w.embed, scratch.resid[:T], ws)
    else:
        scratch.resid[:T].copy_(embeds.reshape(T, w.d))
    for slot, li in enumerate(layer_indices):
        b = pre_layer_bridges[slot]
        if b is not None:
            run_bridge(b, scratch, T, ws)
        run_layer(w, li, fwd, T, cache, scratch, ws, kv_bound)
    if pre_norm_bridge is not None:
        run_bridge(pre_norm_bridge, scratch, T, ws)


def _norm_chain(w: ModelWeights, layer_indices, pre_layer_bridges, pre_norm_bridge) -> list:
    """(weight, eps) of every RMSNorm of a forward, in execution order; the
    last one is the final norm before the head."""
    out = []
    for slot, li in enumerate(layer_indices):
        b = pre_layer_bridges[slot]
        if b is not None:
            out.append((b.norm.weight, float(b.norm.eps)))
        lw = w.layers[li]
        out.append((lw.ln1, lw.eps1))
        out.append((lw.ln2, lw.eps2))
    if pre_norm_bridge is not None:
        out.append((pre_norm_bridge.norm.weight, float(pre_norm_bridge.norm.eps)))
    out.append((w.norm, w.norm_eps))
    return out


def chain_enabled(w: ModelWeights, T: int) -> bool:
    """Whether a bf16 forward of T rows runs its GEMMs as ssd_linear_chain
    launches (decode-sized, single GPU; SSD_CHAIN=1 turns it on, SSD_CHAIN=0
    off; off by default while the separate launches measure faster)."""
    return (w.dtype == torch.bfloat16 and w.tp is None and 1 <= T <= 64
            and os.environ.get("SSD_CHAIN", "0") == "1")


def run_stack_folded(w: ModelWeights, layer_indices, pre_layer_bridges, pre_norm_bridge, fwd: ForwardInputs, T: int,
                     cache, scratch: Scratch, ws: ops.Workspace, kv_bound: int) -> None:
    """run_stack with every RMSNorm folded into the neighbouring kernels (bf16).
    Leaves resid (pre-norm hidden state), and xn / ssq holding the final
    norm's folded input for final_norm_folded. Decode-sized forwards run the
    GEMMs between two attention launches (o_proj, gate/up, down, bridges, the
    next layer's q/k/v) as one chained launch."""
    norms = _norm_chain(w, layer_indices, pre_layer_bridges, pre_norm_bridge)
    parts, d = norm_parts(w), w.d
    xg = scratch.xn(w.dtype, d)[:T, :d]
    ssq = scratch.ssq[:T]
    resid = scratch.resid[:T]
    out_for = lambda k: ops.NormOut(norms[k][0], xg, ssq)
    in_for = lambda k: ops.RowNorm(ssq, parts, d, norms[k][1])
    chain = ops.GemmChain(ws, T, chain_enabled(w, T))
    ops.embed(fwd.ids[:T], w.embed, resid, ws, norm_out=out_for(0))
    if w.tp is not None:
        w.tp.begin()
    k = 0
    for slot, li in enumerate(layer_indices):
        b = pre_layer_bridges[slot]
        if b is not None:
            _bridge_folded(b, scratch, T, chain, xg, in_for(k), out_for(k + 1))
            k += 1
        lw = w.layers[li]
        kc, vc = cache.layer(li)
        chain.qkv(xg, lw.q, lw.k, lw.v, w.H, w.Hkv, w.hd, w.rope_cos, w.rope_sin, fwd.positions, fwd.slots, kc, vc,
                  scratch.q[:T], in_norm=in_for(k))
        chain.flush()
        ops.tree_attention(scratch.q[:T], kc, vc, w.H, w.Hkv, w.hd, fwd.prefix_len, scratch.attn[:T], ws,
                           spec_base=fwd.spec_base if fwd.use_mask else None,
                           spec_mask=fwd.mask if fwd.use_mask else None, kv_bound=kv_bound, T=T,
                           prefix_start=fwd.prefix_start)
        _residual_linear(w, scratch.attn[:T], lw.o, chain, resid, out_for(k + 1), T)
        hid = scratch.hid(w.dtype, w.F, 0)[:T, : w.F]
        chain.linear(xg, [lw.gate, lw.up], epilogue=L.EPI_SWIGLU, layout=L.SEG_PAIRS, out=hid, in_norm=in_for(k + 1))
        _residual_linear(w, hid, lw.down, chain, resid, out_for(k + 2), T)
        k += 2
    if pre_norm_bridge is not None:
        _bridge_folded(pre_norm_bridge, scratch, T, chain, xg, in_for(k), out_for(k + 1))
        k += 1
    chain.flush()
    assert k == len(norms) - 1
    if w.tp is not None:
        w.tp.end()


def _residual_linear(w: ModelWeights, x, weight, chain: ops.GemmChain, resid, norm_out, T: int) -> None:
    """resid += x @ weight^T (+ the next folded norm input). Tensor parallel:
    weight is this rank's input-feature slice; its partial goes to the
    group's exchange buffer and ssd_tp_allreduce_residual sums the ranks'."""
    if w.tp is None:
        chain.linear(x, [weight], epilogue=L.EPI_RESIDUAL, resid=resid, norm_out=norm_out)
        return
    w.tp.check_rows(T)
    parity = w.tp.next_parity()
    ops.linear(x, [weight], chain.ws, epilogue=L.EPI_STORE_F32, out=w.tp.partials[parity][:T])
    ops.tp_allreduce_residual(w.tp, parity, T, resid, chain.ws, norm_out=norm_out, dtype=w.dtype)


def head_argmax(w: ModelWeights, x, weight, out_idx, ws: ops.Workspace, out_max=None, out_gap=None,
                in_norm=None) -> None:
    """lm_head fused with the per-row argmax (vocabulary-parallel when w.tp)."""
    if w.tp is None:
        ops.head_argmax(x, weight, out_idx, ws, out_max=out_max, out_gap=out_gap, in_norm=in_norm)
    else:
        ops.tp_head_argmax(w.tp, x, weight, w.vocab_offset, out_idx, ws, out_max=out_max, out_gap=out_gap,
                           in_norm=in_norm)


def head_topk(w: ModelWeights, x, weight, k: int, out_tok, out_lp, ws: ops.Workspace, vocab_ids=None,
              in_norm=None) -> None:
    """lm_head fused with the per-row log-softmax top-k (vocabulary-parallel when w.tp)."""
    if w.tp is None:
        ops.head_topk(x, weight, k, out_tok, out_lp, ws, vocab_ids=vocab_ids, in_norm=in_norm)
    else:
        ops.tp_head_topk(w.tp, x, weight, w.vocab_offset, k, out_tok, out_lp, ws, vocab_ids=vocab_ids,
                         in_norm=in_norm)


def _bridge_folded(bridge, scratch: Scratch, T: int, chain: ops.GemmChain, xg, rn, nout) -> None:
    """TransitionBridge x + MLP(RMSNorm(x)) with its RMSNorm folded: xg / rn
    carry the folded input, the out-projection produces the next norm's."""
    dt = bridge.norm.weight.dtype
    mlp = bridge.mlp
    if bridge.mlp_type == "swiglu":
        h = scratch.hid(dt, bridge.hidden, 0)[:T, : bridge.hidden]
        chain.linear(xg, [mlp.gate_proj.weight, mlp.up_proj.weight], biases=[mlp.gate_proj.bias, mlp.up_proj.bias],
                     epilogue=L.EPI_SWIGLU, layout=L.SEG_PAIRS, out=h, in_norm=rn)
    else:
        h = xg
        for i, lin in enumerate(mlp.linears()):
            nxt = scratch.hid(dt, bridge.hidden, i % 2)[:T, : lin.weight.shape[0]]
            chain.linear(h, [lin.weight], biases=[lin.bias], act=bridge.activation, out=nxt,
                         in_norm=rn if i == 0 else None)
            h = nxt
    chain.linear(h, [mlp.out_proj.weight], biases=[mlp.out_proj.bias], epilogue=L.EPI_RESIDUAL,
                 resid=scratch.resid[:T], norm_out=nout)


def final_norm_folded(w: ModelWeights, scratch: Scratch, r0: int, r1: int):
    """Head input of a folded forward: (resid * w_norm rows, their RowNorm)."""
    x = scratch.xn(w.dtype, w.d)[r0:r1, : w.d]
    return x, ops.RowNorm(scratch.ssq[r0:r1], norm_parts(w), w.d, w.norm_eps)


def head_input(w: ModelWeights, scratch: Scratch, r0: int, r1: int):
    """(x, in_norm) for the lm_head of rows r0..r1 after run_stack_auto."""
    if folds_norms(w):
        return final_norm_folded(w, scratch, r0, r1)
    return final_norm(w, scratch, r0, r1), None


def run_stack_auto(w: ModelWeights, layer_indices, pre_layer_bridges, pre_norm_bridge, fwd: ForwardInputs, T: int,
                   cache, scratch: Scratch, ws: ops.Workspace, kv_bound: int) -> None:
    """The engines' forward: folded norms for bf16, standalone ones for fp32."""
    if folds_norms(w):
        run_stack_folded(w, layer_indices, pre_layer_bridges, pre_norm_bridge, fwd, T, cache, scratch, ws, kv_bound)
    elif w.tp is not None:
        raise NotImplementedError("tensor parallelism runs the bf16 path only")
    else:
        run_stack(w, layer_indices, pre_layer_bridges, pre_norm_bridge, fwd, T, cache, scratch, ws, kv_bound)


def final_norm(w: ModelWeights, scratch: Scratch, r0: int, r1: int) -> torch.Tensor:
    xn = scratch.xn(w.dtype, w.d)[r0:r1, : w.d]
    ops.rmsnorm(scratch.resid[r0:r1], w.norm, w.norm_eps, xn)
    return xn
