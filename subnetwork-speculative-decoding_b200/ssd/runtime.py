"""Model loading, device selection and bridge-checkpoint layout (API of
ssd/runtime.py).

Checkpoints live at ``{training.output_dir}/{profile}/stage{1,2}.pt`` or
``online.pt`` (profile = layer subset, e.g. ``L0-7-15``), in the reference's
format. ``load_base_model`` loads a HF checkpoint when one is available;
``synthetic_base_model`` builds the seeded random-weight models of the
benchmark configurations (ssd.synthetic).
"""

from __future__ import annotations

import logging
from pathlib import Path
from typing import Optional

import torch
import torch.nn as nn

from ssd.config import SSDConfig, profile_name
from ssd.models.subnetwork_draft import SubnetworkDraftModel

log = logging.getLogger("ssd")


def setup_env(level: int = logging.INFO) -> None:
    """Load ``.env`` if python-dotenv is installed, and configure logging."""
    try:
        from dotenv import load_dotenv

        load_dotenv(Path.cwd() / ".env")
    except ImportError:
        pass
    logging.basicConfig(level=level, format="%(asctime)s %(levelname)s %(message)s", datefmt="%H:%M:%S")


def resolve_device(name: str = "auto") -> torch.device:
    """The B200 path runs on CUDA only; "auto" picks cuda."""
    if name != "auto":
        dev = torch.device(name)
    else:
        dev = torch.device("cuda")
    if dev.type != "cuda":
        raise ValueError("the B200 SSD path runs on CUDA devices only (no CPU/MPS fallback)")
    return dev


def free_device_memory() -> None:
    import gc

    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()


def device_memory_gb(device: torch.device) -> float:
    if device.type == "cuda":
        return torch.cuda.memory_reserved(device) / 2**30
    return 0.0


def load_tokenizer(cfg: SSDConfig):
    from transformers import AutoTokenizer

    return AutoTokenizer.from_pretrained(cfg.model.base_model)


def load_base_model(cfg: SSDConfig, device: Optional[torch.device] = None) -> nn.Module:
    """HF checkpoint -> LlamaForCausalLM on one CUDA device (runtime.py:69-80).
    Multi-device ``device_map`` placement is replaced by tensor parallelism."""
    from transformers import AutoModelForCausalLM

    if cfg.model.device_map is not None:
        raise NotImplementedError("device_map placement is not used by the B200 path")
    base = AutoModelForCausalLM.from_pretrained(cfg.model.base_model, dtype=getattr(torch, cfg.model.torch_dtype))
    base.to(device or resolve_device(cfg.model.device))
    base.eval().requires_grad_(False)
    cfg.validate_against(base.config.num_hidden_layers)
    return base


def synthetic_base_model(name: str, device=None):
    """Seeded random-weight model of a benchmark configuration (c1..c4)."""
    from ssd import synthetic as S

    spec = S.CONFIGS[name]
    dev = device or resolve_device()
    gen = "cpu" if spec.dtype == torch.float32 else "cuda"
    base = S.build_base_model(spec.model, spec.seed, spec.dtype, dev, plant_layers=spec.draft_layers,
                              plant_scale=spec.plant_scale, gen_device=gen)
    return base, spec


def input_device(base: nn.Module) -> torch.device:
    return base.model.embed_tokens.weight.device


def checkpoint_path(cfg: SSDConfig, stage) -> Path:
    """stage: 1, 2 or "online" (runtime.py:87-90)."""
    name = f"stage{stage}.pt" if isinstance(stage, int) else f"{stage}.pt"
    return Path(cfg.training.output_dir) / profile_name(cfg.draft_layers) / name


def latest_checkpoint(cfg: SSDConfig) -> Optional[Path]:
    """online > stage2 > stage1 (runtime.py:93-98)."""
    for stage in ("online", 2, 1):
        p = checkpoint_path(cfg, stage)
        if p.exists():
            return p
    return None


def build_draft(cfg: SSDConfig, base: nn.Module, checkpoint="latest", inference: bool = False,
                vocab_counts: Optional[torch.Tensor] = None) -> SubnetworkDraftModel:
    """Draft for ``cfg.draft_layers`` (runtime.py:101-138). ``inference``:
    cast bridges to the base dtype and apply ``drafting.draft_vocab`` (from
    ``draft_vocab.pt`` / ``token_freq.pt`` under output_dir, or from
    ``vocab_counts`` when given)."""
    draft = SubnetworkDraftModel(base, cfg.draft_layers, cfg.bridge)
    name = profile_name(cfg.draft_layers)
    if checkpoint == "latest":
        checkpoint = latest_checkpoint(cfg)
        if checkpoint is None and draft.bridge_specs:
            log.warning("no trained bridges for %s under %s; using untrained bridges", name, cfg.training.output_dir)
    if checkpoint is not None:
        draft.load_bridges(str(checkpoint))
        log.info("loaded bridges for %s from %s", name, checkpoint)
    if inference:
        draft.bridges.to(base.model.embed_tokens.weight.dtype)
    if inference and cfg.drafting.draft_vocab:
        from ssd.data.token_freq import token_freq_path, top_vocab

        eos = getattr(getattr(base, "generation_config", None), "eos_token_id", None)
        eos = set(eos if isinstance(eos, list) else ([] if eos is None else [eos]))
        explicit = Path(cfg.training.output_dir) / "draft_vocab.pt"
        if vocab_counts is not None:
            draft.set_vocab_subset(top_vocab(vocab_counts, cfg.drafting.draft_vocab, eos))
        elif explicit.exists():
            ids = torch.load(explicit)[: cfg.drafting.draft_vocab]
            draft.set_vocab_subset(ids.sort().values)
        else:
            path = token_freq_path(cfg)
            if not path.exists():
                raise FileNotFoundError(f"{path} missing: provide token counts for drafting.draft_vocab")
            draft.set_vocab_subset(top_vocab(torch.load(path), cfg.drafting.draft_vocab, eos))
    return draft
