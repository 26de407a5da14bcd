"""Draft model = a referenced subset of the target's own layers plus bridges
(API of ssd/models/subnetwork_draft.py:44-472), computed by the B200 kernels.

    embed -> [bridge] -> layer a0 -> [bridge] -> layer a1 -> ... -> [bridge] -> norm -> lm_head

Base modules are referenced, never copied (only the draft-vocab head slice
is a copy, as in the reference), so ``parameters()``/``state_dict()`` hold
only the bridges. The KV cache is keyed by base layer index, so the draft
shares the target's cache. With every layer selected and no bridges the
model is the target itself (``TargetRunner``).

Batch size: the cached path serves one sequence (as the reference's decode
engine); the cache-less path loops over batch rows.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn as nn

from ssd import _lib as L
from ssd import ops
from ssd.config import BridgeConfig, validate_layer_indices
from ssd.engine.kv_cache import KVCache
from ssd.models.bridges import TransitionBridge
from ssd.models import runner as R


@dataclass
class BridgeSpec:
    name: str
    src_boundary: int
    tgt_boundary: int


@dataclass
class DraftOutput:
    logits: Optional[torch.Tensor]
    hidden_states: torch.Tensor
    past_key_values: Optional[KVCache]
    bridge_states: dict = field(default_factory=dict)
    vocab_ids: Optional[torch.Tensor] = None
    layer_inputs: dict = field(default_factory=dict)


def plan_bridges(layer_indices: list[int], num_base_layers: int) -> list[BridgeSpec]:
    """A bridge wherever the draft skips base layers: before each selected
    layer that does not follow the previous one, and before the final norm
    if the last base layer is skipped (subnetwork_draft.py:61-73)."""
    specs: list[BridgeSpec] = []
    have = 0
    for idx in layer_indices:
        if have != idx:
            specs.append(BridgeSpec(f"into_{idx}", have, idx))
        have = idx + 1
    if have != num_base_layers:
        specs.append(BridgeSpec("into_norm", have, num_base_layers))
    return specs


def required_boundaries(layer_indices: list[int], num_base_layers: int) -> set[int]:
    return {b for s in plan_bridges(layer_indices, num_base_layers) for b in (s.src_boundary, s.tgt_boundary)}


class _BaseRefs:
    """Plain holder so base modules are not registered as draft submodules."""

    def __init__(self, base_model: nn.Module, layer_indices: list[int]):
        inner = base_model.model
        self.embed_tokens = inner.embed_tokens
        self.layers = [inner.layers[i] for i in layer_indices]
        self.norm = inner.norm
        self.rotary_emb = getattr(inner, "rotary_emb", None)
        self.lm_head = base_model.lm_head


def _module_device(m: nn.Module) -> torch.device:
    return next(m.parameters()).device


class SubnetworkDraftModel(nn.Module):
    def __init__(self, base_model: nn.Module, layer_indices: list[int], bridge_config: Optional[BridgeConfig] = None,
                 freeze_base: bool = True):
        super().__init__()
        cfg = base_model.config
        self.num_base_layers = cfg.num_hidden_layers
        self.layer_indices = validate_layer_indices(layer_indices, self.num_base_layers)
        self.d_model = cfg.hidden_size
        self.num_heads = cfg.num_attention_heads
        self.num_kv_heads = cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", None) or self.d_model // self.num_heads
        self.bridge_config = bridge_config or BridgeConfig()
        if freeze_base:
            base_model.requires_grad_(False)
        object.__setattr__(self, "_base_model", base_model)
        self.base = _BaseRefs(base_model, self.layer_indices)
        self.bridge_specs = plan_bridges(self.layer_indices, self.num_base_layers)
        by_target = {s.tgt_boundary: s.name for s in self.bridge_specs}
        self._pre_layer_bridge = [by_target.get(idx) for idx in self.layer_indices]
        self._pre_norm_bridge = by_target.get(self.num_base_layers)
        self.bridges = nn.ModuleDict(
            {s.name: TransitionBridge.from_config(self.d_model, self.bridge_config) for s in self.bridge_specs})
        self.place_bridges()
        self.vocab_ids: Optional[torch.Tensor] = None
        self._sub_head: Optional[torch.Tensor] = None
        self._scratch: Optional[R.Scratch] = None
        self._ws: Optional[ops.Workspace] = None

    # ------------------------------------------------------------- set-up
    def set_vocab_subset(self, token_ids: Optional[torch.Tensor]) -> None:
        """Score only ``token_ids`` in the draft head: keeps a contiguous copy
        of those lm_head rows (subnetwork_draft.py:136-144)."""
        if token_ids is None:
            self.vocab_ids = self._sub_head = None
            return
        if getattr(self._base_model, "_ssd_tp_shard", None) is not None:
            raise NotImplementedError("a draft vocabulary subset is not supported on a tensor-parallel shard")
        w = self.base.lm_head.weight
        self.vocab_ids = token_ids.to(device=w.device, dtype=torch.int64)
        self._sub_head = w.detach().index_select(0, self.vocab_ids).contiguous()

    def place_bridges(self) -> None:
        """Each bridge on the device of the base module consuming its output."""
        for spec in self.bridge_specs:
            if spec.tgt_boundary == self.num_base_layers:
                consumer = self.base.norm
            else:
                consumer = self.base.layers[self.layer_indices.index(spec.tgt_boundary)]
            self.bridges[spec.name].to(_module_device(consumer))

    @property
    def num_layers(self) -> int:
        return len(self.layer_indices)

    @property
    def weights(self) -> R.ModelWeights:
        return R.ModelWeights.of(self._base_model)

    def head_weight(self) -> torch.Tensor:
        return self._sub_head if self._sub_head is not None else self.base.lm_head.weight

    def new_cache(self, max_length: int) -> KVCache:
        """One slot per base layer, so the cache is shared with the target."""
        return KVCache(self.num_base_layers, max_length)

    def pre_layer_bridge_modules(self) -> list:
        return [self.bridges[n] if n is not None else None for n in self._pre_layer_bridge]

    def pre_norm_bridge_module(self):
        return self.bridges[self._pre_norm_bridge] if self._pre_norm_bridge is not None else None

    def check_bridge_dtypes(self) -> None:
        for b in self.bridges.values():
            if b.norm.weight.dtype not in (torch.float32, torch.bfloat16):
                raise ValueError("bridges must be float32 or bfloat16")

    def _resources(self, rows: int):
        w = self.weights
        if self._scratch is None or self._scratch.rows < rows:
            self._scratch = R.Scratch(w, max(rows, 64))
            self._scratch.reserve_bridges(list(self.bridges.values()))
            self._ws = ops.Workspace(w.device, max_rows=self._scratch.rows, vocab=w.V, max_head_rows=64)
        return w, self._scratch, self._ws

    # ------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, input_ids: Optional[torch.Tensor] = None, position_ids: Optional[torch.Tensor] = None,
                past_key_values: Optional[KVCache] = None, tree_attention_mask: Optional[torch.Tensor] = None,
                inputs_embeds: Optional[torch.Tensor] = None, logits_to_keep: int = 0, compute_logits: bool = True,
                output_bridge_states: bool = False, true_layer_inputs: Optional[dict] = None,
                output_layer_inputs: Optional[set] = None) -> DraftOutput:
        """Run the sub-network (subnetwork_draft.py:249-357) on the kernels.

        input_ids [B, q]; position_ids [B, q] (default past + arange(q));
        past_key_values: a KVCache, updated in place and advanced by q;
        tree_attention_mask: bool [.., q, q] or [.., q, past + q] (None ->
        causal); logits_to_keep: logits only for the last N rows.
        """
        if true_layer_inputs is not None:
            if past_key_values is not None:
                raise ValueError("true_layer_inputs is for training without a cache")
            raise NotImplementedError("training-mode forwards (true_layer_inputs) are not part of the B200 path")
        if output_layer_inputs:
            raise NotImplementedError("output_layer_inputs is a training tap, not part of the B200 path")
        if input_ids is None and inputs_embeds is None:
            raise ValueError("pass input_ids or inputs_embeds")
        if self.weights.tp is not None:
            raise NotImplementedError("tensor-parallel shards run through the decode engines "
                                      "(SpeculativeGenerator.generate / autoregressive_generate)")
        bsz, q_len = (input_ids.shape if input_ids is not None else inputs_embeds.shape[:2])
        if past_key_values is not None and bsz != 1:
            raise ValueError("the cached B200 path serves batch size 1")
        if bsz > 1:
            outs = [self.forward(input_ids[b:b + 1] if input_ids is not None else None,
                                 position_ids[b:b + 1] if position_ids is not None and position_ids.shape[0] > 1
                                 else position_ids, None, tree_attention_mask,
                                 inputs_embeds[b:b + 1] if inputs_embeds is not None else None, logits_to_keep,
                                 compute_logits, output_bridge_states) for b in range(bsz)]
            return DraftOutput(
                logits=None if outs[0].logits is None else torch.cat([o.logits for o in outs]),
                hidden_states=torch.cat([o.hidden_states for o in outs]), past_key_values=None,
                bridge_states={k: torch.cat([o.bridge_states[k] for o in outs]) for k in outs[0].bridge_states},
                vocab_ids=outs[0].vocab_ids)
        w, scratch, ws = self._resources(q_len)
        cache = past_key_values if past_key_values is not None else KVCache(self.num_base_layers, q_len)
        past = cache.get_seq_length()
        cache.check_room(q_len)
        cache.allocate(w.Hkv, w.hd, w.dtype, w.device)
        if position_ids is None:
            position_ids = torch.arange(past, past + q_len)
        if position_ids.reshape(-1).max().item() >= w.max_pos:
            raise ValueError(f"position beyond the RoPE table ({w.max_pos})")
        fwd = getattr(self, "_fwd", None)
        if fwd is None or fwd.cap < q_len:
            fwd = R.ForwardInputs(max(q_len, 64), w.device, mask_words=4)
            self._fwd = fwd
        ids = input_ids if input_ids is not None else torch.zeros(1, q_len, dtype=torch.int64)
        fwd.fill(ids, position_ids, past, tree_attention_mask)
        bridge_states: dict = {}
        pre = self.pre_layer_bridge_modules()
        embeds = inputs_embeds[0].to(w.device).float() if inputs_embeds is not None else None
        if output_bridge_states:
            # run layer by layer to tap each bridge output
            if embeds is None:
                ops.embed(fwd.ids[:q_len], w.embed, scratch.resid[:q_len], ws)
            else:
                scratch.resid[:q_len].copy_(embeds)
            for slot, li in enumerate(self.layer_indices):
                b = pre[slot]
                if b is not None:
                    R.run_bridge(b, scratch, q_len, ws)
                    bridge_states[self._pre_layer_bridge[slot]] = scratch.resid[:q_len].to(w.dtype).unsqueeze(0)
                R.run_layer(w, li, fwd, q_len, cache, scratch, ws, cache.max_length)
            if self._pre_norm_bridge is not None:
                R.run_bridge(self.pre_norm_bridge_module(), scratch, q_len, ws)
                bridge_states[self._pre_norm_bridge] = scratch.resid[:q_len].to(w.dtype).unsqueeze(0)
        else:
            R.run_stack(w, self.layer_indices, pre, self.pre_norm_bridge_module(), fwd, q_len, cache, scratch, ws,
                        cache.max_length, embeds=embeds)
        cache.advance(q_len)
        hidden = R.final_norm(w, scratch, 0, q_len).clone().unsqueeze(0)
        logits = None
        if compute_logits:
            keep = q_len if logits_to_keep <= 0 else min(logits_to_keep, q_len)
            head = self.head_weight()
            xk = scratch.xn(w.dtype, w.d)[q_len - keep:q_len, : w.d]
            logits = torch.empty(keep, head.shape[0], dtype=w.dtype, device=w.device)
            ops.linear(xk, [head], ws, out=logits)
            logits = logits.unsqueeze(0)
        ws.check_status()
        return DraftOutput(logits=logits, hidden_states=hidden,
                           past_key_values=past_key_values, bridge_states=bridge_states,
                           vocab_ids=self.vocab_ids if compute_logits else None)

    # ------------------------------------------------------- persistence
    def save_bridges(self, path: str, **meta) -> None:
        """Same checkpoint format as the reference (subnetwork_draft.py:455-466)."""
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        torch.save({"layer_indices": self.layer_indices, "bridge_config": vars(self.bridge_config),
                    "state_dict": self.bridges.state_dict(), "meta": meta}, path)

    def load_bridges(self, path: str, strict: bool = True) -> None:
        """subnetwork_draft.py:468-472."""
        ckpt = torch.load(path, map_location="cpu", weights_only=True)
        if list(ckpt["layer_indices"]) != self.layer_indices:
            raise ValueError(f"checkpoint layer_indices {ckpt['layer_indices']} != {self.layer_indices}")
        self.bridges.load_state_dict(ckpt["state_dict"], strict=strict)
