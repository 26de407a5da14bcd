"""Seeded synthetic models, prompts and draft vocabularies for the benchmark
configurations (random weights: the real Llama checkpoints are gated and
there is no network).

Weights: every >= 2-D parameter ~ N(0, init_std) and every norm weight = 1,
drawn in ``named_parameters()`` order from one generator seeded with the
config's seed. "Planted acceptance" scales o_proj and down_proj of every
non-draft layer by ``plant_scale`` so the draft sub-network approximates the
target. Bridges: in-projections ~ N(0, bridge_in_std), out-projection ~
N(0, bridge_out_std), biases 0, norm 1.

This module depends only on torch and transformers so the golden-fixture
script can load it next to the reference implementation.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from typing import Optional

import torch

# name -> LlamaConfig kwargs
SPECS: dict[str, dict] = {
    "tiny": dict(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=6, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=16, tie_word_embeddings=False),
    "tiny_v8": dict(vocab_size=8, hidden_size=64, intermediate_size=128, num_hidden_layers=6, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=16, tie_word_embeddings=False),
    "llama32_1b": dict(vocab_size=128256, hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=64, tie_word_embeddings=True),
    "llama3_8b": dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, tie_word_embeddings=False),
    "llama3_70b": dict(vocab_size=128256, hidden_size=8192, intermediate_size=28672, num_hidden_layers=80,
                       num_attention_heads=64, num_key_value_heads=8, head_dim=128, tie_word_embeddings=False),
}


@dataclass
class SyntheticSpec:
    """One benchmark configuration (see BASELINE configs C1-C5)."""

    model: str
    seed: int
    dtype: torch.dtype
    draft_layers: list[int]
    bridge_hidden: Optional[int]
    plant_scale: Optional[float] = None  # None -> no planting
    init_std: float = 0.02
    bridge_in_std: float = 0.02
    bridge_out_std: float = 1e-4
    prompt_len: int = 128
    max_new_tokens: int = 64
    drafting: dict = field(default_factory=dict)
    draft_vocab: Optional[int] = None


CONFIGS: dict[str, SyntheticSpec] = {
    # a seconds-long configuration for smoke runs of the command line
    "tiny": SyntheticSpec("tiny", 0, torch.float32, [0, 3, 5], None, prompt_len=16, max_new_tokens=16,
                          drafting=dict(depth=3, branch=[2, 2, 1])),
    "c1": SyntheticSpec("llama32_1b", 0, torch.float32, [0, 7, 15], 4096, None, prompt_len=128, max_new_tokens=64,
                        drafting=dict(depth=4, branch=1)),
    "c2": SyntheticSpec("llama32_1b", 1, torch.bfloat16, [0, 7, 15], 4096, 0.05, prompt_len=512, max_new_tokens=256,
                        drafting=dict(depth=4, branch=[3, 2, 2, 1], width=8, max_nodes=24), draft_vocab=32768),
    "c3": SyntheticSpec("llama3_8b", 2, torch.bfloat16, [0, 15, 31], None, 0.05, prompt_len=2048, max_new_tokens=256,
                        drafting=dict(depth=6, branch=[4, 2, 2, 1, 1, 1], max_nodes=32)),
    "c3_sample": SyntheticSpec("llama3_8b", 2, torch.bfloat16, [0, 15, 31], None, 0.05, prompt_len=2048,
                               max_new_tokens=256,
                               drafting=dict(depth=6, branch=[4, 2, 2, 1, 1, 1], max_nodes=32, temperature=0.7,
                                             top_p=0.9)),
    "c4": SyntheticSpec("llama3_70b", 3, torch.bfloat16, [0, 39, 79], 8192, 0.05, prompt_len=4096, max_new_tokens=128,
                        drafting=dict(depth=4, branch=[3, 2, 2, 1], width=8, max_nodes=24)),
}


def llama_config(name: str, **overrides):
    from transformers import LlamaConfig

    kw = dict(SPECS[name])
    kw.update(overrides)
    kw.setdefault("rope_theta", 500000.0)
    kw.setdefault("rms_norm_eps", 1e-5)
    kw.setdefault("max_position_embeddings", 8192)
    return LlamaConfig(**kw)


def rope_theta(config) -> float:
    rp = getattr(config, "rope_parameters", None)
    if isinstance(rp, dict) and "rope_theta" in rp:
        return float(rp["rope_theta"])
    return float(getattr(config, "rope_theta", 10000.0))


@torch.no_grad()
def init_model_(model, seed: int, init_std: float = 0.02, gen_device: str = "cpu") -> None:
    """Seeded N(0, init_std) weights, unit norms, in named_parameters order."""
    g = torch.Generator(device=gen_device).manual_seed(seed)
    for _, p in model.named_parameters():
        if p.dim() >= 2:
            if p.device.type == gen_device:
                p.normal_(0.0, init_std, generator=g)
            else:
                p.copy_(torch.empty(p.shape, device=gen_device, dtype=torch.float32).normal_(0.0, init_std,
                                                                                              generator=g))
        else:
            p.fill_(1.0)


@torch.no_grad()
def plant_(model, draft_layers: list[int], scale: float) -> None:
    """Scale o_proj and down_proj of every non-draft layer (planted acceptance)."""
    keep = set(draft_layers)
    for i, layer in enumerate(model.model.layers):
        if i not in keep:
            layer.self_attn.o_proj.weight.mul_(scale)
            layer.mlp.down_proj.weight.mul_(scale)


def build_base_model(name: str, seed: int, dtype: torch.dtype = torch.float32, device="cpu", *,
                     init_std: float = 0.02, plant_layers: Optional[list[int]] = None,
                     plant_scale: Optional[float] = None, gen_device: Optional[str] = None, **config_overrides):
    """A LlamaForCausalLM with seeded synthetic weights.

    gen_device: where the random numbers are drawn ("cpu" reproduces across
    machines; "cuda" is fast for 8B/70B). Defaults to "cpu" when the model is
    built on the CPU, else the model's device.
    """
    from transformers import LlamaForCausalLM
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    cfg = llama_config(name, **config_overrides)
    device = torch.device(device)
    if gen_device is None:
        gen_device = "cpu" if device.type == "cpu" else device.type
    with torch.device("meta"):
        model = LlamaForCausalLM(cfg)
    if gen_device == "cpu" and device.type != "cpu" and dtype != torch.float32:
        # draw in fp32 on the CPU for reproducibility, then move
        model.to_empty(device="cpu")
        model.tie_weights()
        init_model_(model, seed, init_std, "cpu")
        if plant_scale is not None:
            plant_(model, plant_layers or [], plant_scale)
        model.to(dtype=dtype).to(device)
    else:
        model.to_empty(device=device)
        model.tie_weights()
        if dtype != torch.float32:
            model.to(dtype=dtype)
        init_model_(model, seed, init_std, gen_device)
        if plant_scale is not None:
            plant_(model, plant_layers or [], plant_scale)
    model.model.rotary_emb = LlamaRotaryEmbedding(config=cfg, device=device)
    model.eval().requires_grad_(False)
    return model


@torch.no_grad()
def init_bridges_(bridges, seed: int, in_std: float = 0.02, out_std: float = 1e-4) -> None:
    """Deterministic bridge weights (works for the reference's and this
    package's TransitionBridge: same parameter names)."""
    g = torch.Generator().manual_seed(seed * 1000003 + 17)
    for name in sorted(bridges.keys()):
        for pname, p in bridges[name].named_parameters():
            if pname.startswith("norm"):
                p.fill_(1.0)
            elif pname.endswith("bias"):
                p.zero_()
            else:
                std = out_std if "out_proj" in pname else in_std
                p.copy_(torch.empty(p.shape, dtype=torch.float32).normal_(0.0, std, generator=g))


def make_prompt(seed: int, length: int, vocab: int) -> torch.Tensor:
    return torch.randint(0, vocab, (1, length), generator=torch.Generator().manual_seed(seed))


def zipf_counts(vocab: int, seed: int, s: float = 1.1) -> torch.Tensor:
    """Token counts round(1e9 * (r+1)^-s) for rank r of a seeded permutation."""
    perm = torch.randperm(vocab, generator=torch.Generator().manual_seed(seed))
    ranks = torch.arange(vocab, dtype=torch.float64)
    counts = torch.zeros(vocab, dtype=torch.int64)
    counts[perm] = torch.round(1e9 * (ranks + 1.0) ** (-s)).to(torch.int64)
    return counts


def weights_checksum(model) -> str:
    """Hash of all parameters (fp32 bytes) to detect RNG drift between hosts."""
    h = hashlib.sha256()
    for name, p in model.named_parameters():
        h.update(name.encode())
        h.update(p.detach().float().cpu().contiguous().numpy().tobytes())
    return h.hexdigest()[:24]
