"""numpy restatement of the shared-cache layer implementation (test oracle).

Follows ssd/models/subnetwork_draft.py (SubnetworkDraftModel.forward
:249-357, _layer_forward :193-246, _build_attn_mask :165-191, plan_bridges
:61-73), ssd/models/bridges.py (RMSNorm :27-37, _PlainMLP :40-54, _SwiGLU
:57-65, TransitionBridge.forward :131-135) and ssd/engine/kv_cache.py
(KVCache :21-73), batch size 1.
"""

from __future__ import annotations

from typing import Optional

import numpy as np


def weights_from_hf(model, dtype=np.float64) -> tuple[dict, dict]:
    """(base weights, config) as numpy arrays from a HF LlamaForCausalLM."""
    cfg = model.config
    inner = model.model

    def a(t):
        return t.detach().float().cpu().numpy().astype(dtype, copy=False)

    rp = getattr(cfg, "rope_parameters", None)
    theta = float(rp["rope_theta"]) if isinstance(rp, dict) and "rope_theta" in rp else float(cfg.rope_theta)
    conf = dict(
        vocab=cfg.vocab_size,
        hidden=cfg.hidden_size,
        layers=cfg.num_hidden_layers,
        heads=cfg.num_attention_heads,
        kv_heads=cfg.num_key_value_heads,
        head_dim=getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads,
        eps=float(cfg.rms_norm_eps),
        theta=theta,
    )
    layers = []
    for lyr in inner.layers:
        at, mlp = lyr.self_attn, lyr.mlp
        layers.append(dict(q=a(at.q_proj.weight), k=a(at.k_proj.weight), v=a(at.v_proj.weight),
                           o=a(at.o_proj.weight), gate=a(mlp.gate_proj.weight), up=a(mlp.up_proj.weight),
                           down=a(mlp.down_proj.weight), ln1=a(lyr.input_layernorm.weight),
                           ln2=a(lyr.post_attention_layernorm.weight)))
    base = dict(embed=a(inner.embed_tokens.weight), lm_head=a(model.lm_head.weight), norm=a(inner.norm.weight),
                layers=layers)
    return base, conf


def bridges_from_module(bridges, bridge_cfg: dict, dtype=np.float64) -> dict:
    """numpy copy of a ModuleDict of TransitionBridge (reference or product)."""
    out = {}
    for name, b in bridges.items():
        sd = {k: v.detach().float().cpu().numpy().astype(dtype) for k, v in b.state_dict().items()}
        out[name] = dict(sd=sd, mlp_type=bridge_cfg.get("mlp_type", "mlp"),
                         activation=bridge_cfg.get("activation", "silu"),
                         num_layers=bridge_cfg.get("num_layers", 2), eps=bridge_cfg.get("norm_eps", 1e-5))
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """LlamaRMSNorm / bridges.RMSNorm (bridges.py:33-37)."""
    var = np.mean(x * x, axis=-1, keepdims=True)
    return w * (x / np.sqrt(var + eps))


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _gelu(x):
    from math import erf, sqrt

    verf = np.vectorize(erf)
    return 0.5 * x * (1.0 + verf(x / sqrt(2.0)))


_ACTS = {"silu": _silu, "gelu": _gelu, "relu": lambda x: np.maximum(x, 0.0)}


def bridge_forward(b: dict, x: np.ndarray) -> np.ndarray:
    """TransitionBridge.forward (bridges.py:131-135): x + MLP(RMSNorm(x))."""
    sd = b["sd"]
    h = rms_norm(x, sd["norm.weight"], b["eps"])

    def lin(name, v):
        y = v @ sd[f"{name}.weight"].T
        if f"{name}.bias" in sd:
            y = y + sd[f"{name}.bias"]
        return y

    if b["mlp_type"] == "swiglu":  # _SwiGLU (bridges.py:64-65)
        y = lin("mlp.out_proj", _silu(lin("mlp.gate_proj", h)) * lin("mlp.up_proj", h))
    else:  # _PlainMLP (bridges.py:53-54): body = [Linear, act] * (num_layers - 1)
        act = _ACTS[b["activation"]]
        for i in range(b["num_layers"] - 1):
            h = act(lin(f"mlp.body.{2 * i}", h))
        y = lin("mlp.out_proj", h)
    return x + y


def plan_bridges(layer_indices: list[int], num_base_layers: int) -> list[tuple[str, int, int]]:
    """(name, src_boundary, tgt_boundary) per bridge (subnetwork_draft.py:61-73)."""
    specs, have = [], 0
    for idx in layer_indices:
        if have != idx:
            specs.append((f"into_{idx}", have, idx))
        have = idx + 1
    if have != num_base_layers:
        specs.append(("into_norm", have, num_base_layers))
    return specs


class OracleKVCache:
    """KVCache (kv_cache.py:21-73) for batch 1: per base layer [n_kv, max_len, hd]."""

    def __init__(self, num_slots: int, max_length: int):
        self.num_slots = num_slots
        self.max_length = max_length
        self.seq_len = 0
        self.k: list[Optional[np.ndarray]] = [None] * num_slots
        self.v: list[Optional[np.ndarray]] = [None] * num_slots

    def get_seq_length(self) -> int:
        return self.seq_len

    def update(self, slot: int, k: np.ndarray, v: np.ndarray):
        """kv_cache.py:32-43: write [len, len+q) and return the [0, len+q) views."""
        n_kv, q_len, hd = k.shape
        end = self.seq_len + q_len
        if end > self.max_length:
            raise RuntimeError(f"KVCache overflow: {end} > max_length={self.max_length}")
        if self.k[slot] is None:
            self.k[slot] = np.zeros((n_kv, self.max_length, hd), dtype=k.dtype)
            self.v[slot] = np.zeros((n_kv, self.max_length, hd), dtype=v.dtype)
        self.k[slot][:, self.seq_len:end] = k
        self.v[slot][:, self.seq_len:end] = v
        return self.k[slot][:, :end], self.v[slot][:, :end]

    def advance(self, n: int) -> None:
        self.seq_len += n

    def crop(self, length: int) -> None:
        """kv_cache.py:48-52."""
        if length > self.seq_len:
            raise ValueError(f"cannot crop to {length} > current length {self.seq_len}")
        self.seq_len = length

    def keep_positions(self, start: int, positions: list[int]) -> None:
        """kv_cache.py:54-70: gather `positions` into [start, start+n)."""
        n = len(positions)
        if n == 0 or list(positions) == list(range(start, start + n)):
            self.seq_len = start + n
            return
        idx = np.asarray(positions)
        for s in range(self.num_slots):
            if self.k[s] is None:
                continue
            self.k[s][:, start:start + n] = self.k[s][:, idx].copy()
            self.v[s][:, start:start + n] = self.v[s][:, idx].copy()
        self.seq_len = start + n

    def reset(self) -> None:
        self.seq_len = 0


def rope_cos_sin(positions: np.ndarray, head_dim: int, theta: float):
    """HF Llama default RoPE: fp32 inv_freq and angles; cos/sin of emb=cat(f,f)."""
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) /
                                        np.float32(head_dim)))).astype(np.float32)
    ang = positions.astype(np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([ang, ang], axis=-1).astype(np.float64)
    return np.cos(emb), np.sin(emb)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


class OracleModel:
    """SubnetworkDraftModel restated (subnetwork_draft.py:101-357), B=1.

    With layer_indices == all layers and no bridges it is the reference's
    TargetRunner (ssd/engine/speculative.py:94-98).
    """

    def __init__(self, base: dict, conf: dict, layer_indices: list[int], bridges: Optional[dict] = None,
                 dtype=np.float64):
        self.base = base
        self.conf = conf
        self.layer_indices = list(layer_indices)
        self.dtype = dtype
        specs = plan_bridges(self.layer_indices, conf["layers"])
        by_tgt = {t: name for name, _, t in specs}
        self.bridge_specs = specs
        self.pre_layer_bridge = [by_tgt.get(i) for i in self.layer_indices]
        self.pre_norm_bridge = by_tgt.get(conf["layers"])
        self.bridges = bridges or {}
        missing = [name for name, _, _ in specs if name not in self.bridges]
        if missing:
            raise ValueError(f"missing bridge weights for {missing}")
        self.vocab_ids: Optional[np.ndarray] = None
        self.sub_head: Optional[np.ndarray] = None

    def set_vocab_subset(self, ids) -> None:
        """subnetwork_draft.py:136-144."""
        if ids is None:
            self.vocab_ids = self.sub_head = None
            return
        self.vocab_ids = np.asarray(ids, dtype=np.int64)
        self.sub_head = self.base["lm_head"][self.vocab_ids]

    def new_cache(self, max_length: int) -> OracleKVCache:
        return OracleKVCache(self.conf["layers"], max_length)

    @staticmethod
    def build_attn_mask(q_len: int, past_len: int, tree_mask: Optional[np.ndarray]) -> Optional[np.ndarray]:
        """_build_attn_mask (subnetwork_draft.py:165-191), 2-D [q, past+q]."""
        if tree_mask is not None and tree_mask.shape[-1] == past_len + q_len and past_len > 0:
            return tree_mask.astype(bool)
        if tree_mask is None:
            if q_len == 1:
                return None
            causal = np.tril(np.ones((q_len, q_len), dtype=bool))
        else:
            causal = tree_mask.astype(bool)
            if causal.shape[-2:] != (q_len, q_len):
                raise ValueError(f"tree_attention_mask must be [.., {q_len}, {q_len}], got {causal.shape}")
        return np.concatenate([np.ones((q_len, past_len), dtype=bool), causal], axis=-1)

    def _layer(self, li: int, h: np.ndarray, cos, sin, mask, cache: Optional[OracleKVCache]) -> np.ndarray:
        """_layer_forward (subnetwork_draft.py:193-246)."""
        c = self.conf
        W = self.base["layers"][li]
        T = h.shape[0]
        H, Hkv, hd = c["heads"], c["kv_heads"], c["head_dim"]
        x = rms_norm(h, W["ln1"], c["eps"])
        q = (x @ W["q"].T).reshape(T, H, hd).transpose(1, 0, 2)
        k = (x @ W["k"].T).reshape(T, Hkv, hd).transpose(1, 0, 2)
        v = (x @ W["v"].T).reshape(T, Hkv, hd).transpose(1, 0, 2)
        q = q * cos[None] + _rotate_half(q) * sin[None]
        k = k * cos[None] + _rotate_half(k) * sin[None]
        if cache is not None:
            k, v = cache.update(li, k, v)
        S = k.shape[1]
        if mask is None:
            if cache is None and T > 1:
                mask = np.tril(np.ones((T, S), dtype=bool))
            else:
                mask = np.ones((T, S), dtype=bool)
        G = H // Hkv
        out = np.empty((H, T, hd), dtype=h.dtype)
        scale = 1.0 / np.sqrt(hd)
        for hh in range(H):
            s = (q[hh] @ k[hh // G].T) * scale
            s = np.where(mask, s, -np.inf)
            s = s - s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=-1, keepdims=True)
            out[hh] = p @ v[hh // G]
        o = out.transpose(1, 0, 2).reshape(T, H * hd)
        h = h + o @ W["o"].T
        x2 = rms_norm(h, W["ln2"], c["eps"])
        return h + (_silu(x2 @ W["gate"].T) * (x2 @ W["up"].T)) @ W["down"].T

    def forward(self, ids, position_ids=None, cache: Optional[OracleKVCache] = None, tree_mask=None,
                logits_to_keep: int = 0, compute_logits: bool = True) -> Optional[np.ndarray]:
        """SubnetworkDraftModel.forward cache branch (subnetwork_draft.py:249-357).
        Returns logits [T', V or V'] (T' = logits_to_keep or T)."""
        c = self.conf
        ids = np.asarray(ids, dtype=np.int64).reshape(-1)
        T = ids.shape[0]
        past = cache.get_seq_length() if cache is not None else 0
        if position_ids is None:
            position_ids = np.arange(past, past + T)
        position_ids = np.asarray(position_ids).reshape(-1)
        cos, sin = rope_cos_sin(position_ids, c["head_dim"], c["theta"])
        mask = None
        if not (cache is None and tree_mask is None):
            mask = self.build_attn_mask(T, past, None if tree_mask is None else np.asarray(tree_mask))
        h = self.base["embed"][ids].astype(self.dtype)
        for slot, li in enumerate(self.layer_indices):
            name = self.pre_layer_bridge[slot]
            if name is not None:
                h = bridge_forward(self.bridges[name], h)
            h = self._layer(li, h, cos, sin, mask, cache)
        if self.pre_norm_bridge is not None:
            h = bridge_forward(self.bridges[self.pre_norm_bridge], h)
        if cache is not None:
            cache.advance(T)
        h = rms_norm(h, self.base["norm"], c["eps"])
        if not compute_logits:
            return None
        hs = h[-logits_to_keep:] if logits_to_keep > 0 else h
        head = self.sub_head if self.sub_head is not None else self.base["lm_head"]
        return hs @ head.T
