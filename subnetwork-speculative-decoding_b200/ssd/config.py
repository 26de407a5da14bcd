"""YAML configuration, drop-in compatible with the reference's ssd/config.py.

Same sections, field names, defaults and validation errors (ssd/config.py:
BridgeConfig :17-26, ModelConfig :29-35, DataConfig :38-47, Stage1Config
:50-63, Stage2Config :66-82, DraftingConfig :88-130, OnlineConfig :133-157,
TrainingConfig :160-168, SSDConfig :171-228, validate_layer_indices
:232-243). The training/data sections are parsed so existing YAML files
load, but training itself is not part of this package.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field, fields
from pathlib import Path
from typing import Any, Optional, Union

import yaml


@dataclass
class BridgeConfig:
    mlp_type: str = "mlp"  # "mlp" | "swiglu"
    num_layers: int = 2  # linear layers ("mlp": 2-3; "swiglu": 2)
    hidden_dim: Optional[int] = None  # None -> d_model
    activation: str = "silu"  # "silu" | "gelu" | "relu"
    bias: bool = True
    init_std: float = 1e-3  # std of the output projection (near-identity start)
    norm_eps: float = 1e-5
    dtype: str = "float32"  # bridge parameter dtype; inputs are cast in/out


@dataclass
class ModelConfig:
    base_model: str = "meta-llama/Meta-Llama-3-8B-Instruct"
    torch_dtype: str = "bfloat16"
    device_map: Optional[str] = None
    device: str = "auto"
    attn_implementation: str = "sdpa"


@dataclass
class DataConfig:
    dataset: str = "HuggingFaceH4/ultrachat_200k"
    split: str = "train_sft"
    messages_field: str = "messages"
    local_path: Optional[str] = None
    format: str = "packed"
    max_len: int = 2048
    seq_len: int = 1024
    skip_samples: int = 0


@dataclass
class Stage1Config:
    steps: int = 2000
    batch_size: int = 8
    lr: float = 1e-4
    weight_decay: float = 0.0
    warmup_steps: int = 100
    grad_clip: float = 1.0
    alpha_mse: float = 1.0
    beta_cos: float = 1.0
    mode: str = "teacher"
    skip_first_positions: int = 1
    activation_cache: Optional[str] = None


@dataclass
class Stage2Config:
    steps: int = 2000
    batch_size: int = 4
    lr: float = 3e-5
    weight_decay: float = 0.0
    warmup_steps: int = 100
    grad_clip: float = 1.0
    temperature: float = 2.0
    kd_weight: float = 1.0
    ce_weight: float = 0.1
    ttt_steps: int = 1
    ttt_decay: float = 1.0
    micro_batch: Optional[int] = None


IntOrList = Union[int, list[int]]


@dataclass
class DraftingConfig:
    """Speculation tree. Per-depth values take an int (all depths) or a list
    of length ``depth``. Level d: every kept node of level d-1 proposes
    ``branch[d]`` children; the ``width[d]`` best by cumulative draft
    log-prob are kept; finally the best ``max_nodes`` go to verification."""

    depth: int = 4
    branch: IntOrList = 1
    width: Optional[IntOrList] = None
    max_nodes: Optional[int] = None
    temperature: float = 0.0
    top_p: float = 1.0
    draft_vocab: Optional[int] = None

    def per_depth(self, value: Optional[IntOrList], name: str) -> list[Optional[int]]:
        """One entry per tree level: a scalar (or None) repeats, a list must
        name every level."""
        if isinstance(value, (list, tuple)):
            if len(value) != self.depth:
                raise ValueError(f"drafting.{name}: {len(value)} values given for depth {self.depth}")
            return list(value)
        return [value for _ in range(self.depth)]

    def validate(self) -> None:
        """Reject trees the drafter cannot build (ValueError, as the reference)."""

        def at_least_one(v) -> bool:
            return isinstance(v, int) and v >= 1

        if not at_least_one(self.depth):
            raise ValueError(f"drafting.depth must be at least 1, got {self.depth!r}")
        problems = []
        if not all(at_least_one(b) for b in self.per_depth(self.branch, "branch")):
            problems.append(f"every branch entry must be at least 1 (branch={self.branch!r})")
        if not all(x is None or at_least_one(x) for x in self.per_depth(self.width, "width")):
            problems.append(f"every width entry must be at least 1 or null (width={self.width!r})")
        for name in ("max_nodes", "draft_vocab"):
            v = getattr(self, name)
            if v is not None and not at_least_one(v):
                problems.append(f"{name} must be at least 1 or null ({name}={v!r})")
        if self.temperature < 0:
            problems.append(f"temperature must be >= 0 (temperature={self.temperature!r})")
        if not 0.0 < self.top_p <= 1.0:
            problems.append(f"top_p must lie in (0, 1] (top_p={self.top_p!r})")
        if problems:
            raise ValueError("drafting: " + "; ".join(problems))


@dataclass
class OnlineConfig:
    prompt: str = "Tell me about something you find fascinating, in detail."
    streams: int = 32
    temperature: float = 0.8
    top_p: float = 0.95
    chunk: int = 128
    context: int = 384
    max_context: int = 1024
    keep_on_slide: int = 256
    loop_window: int = 64
    loop_min_distinct: float = 0.25
    micro_batch: int = 8
    lr: float = 5e-5
    weight_decay: float = 0.0
    warmup_steps: int = 50
    grad_clip: float = 1.0
    temperature_kd: float = 2.0
    kd_weight: float = 1.0
    ce_weight: float = 0.1
    save_every: int = 200


@dataclass
class TrainingConfig:
    output_dir: str = "outputs/default"
    seed: int = 0
    log_every: int = 20
    save_every: int = 500
    stage1: Stage1Config = field(default_factory=Stage1Config)
    stage2: Stage2Config = field(default_factory=Stage2Config)
    online: OnlineConfig = field(default_factory=OnlineConfig)


# Nested sections: (parent dataclass, field) -> the dataclass its mapping builds.
_NESTED: dict = {}


def _section(cls, raw: Any, path: str):
    """Build dataclass `cls` from a YAML mapping. Keys the schema does not
    define are an error (a typo must not silently fall back to a default);
    nested sections are built the same way, recursively."""
    if raw is None:
        raw = {}
    if not isinstance(raw, dict):
        raise ValueError(f"{path}: expected a mapping, got {type(raw).__name__}")
    names = {f.name for f in fields(cls)}
    extra = sorted(k for k in raw if k not in names)
    if extra:
        raise ValueError(f"{path}: unknown key(s) {extra}")
    kwargs = {}
    for key, value in raw.items():
        sub = _NESTED.get((cls, key))
        kwargs[key] = _section(sub, value, f"{path}.{key}") if sub is not None else value
    return cls(**kwargs)


def profile_name(layers: list[int]) -> str:
    """Name of a layer profile, e.g. [0, 7, 15] -> "L0-7-15"."""
    return "L" + "-".join(map(str, layers))


@dataclass
class SSDConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    draft_layers: list[int] = field(default_factory=lambda: [0, 15, 31])
    bridge: BridgeConfig = field(default_factory=BridgeConfig)
    drafting: DraftingConfig = field(default_factory=DraftingConfig)
    data: DataConfig = field(default_factory=DataConfig)
    training: TrainingConfig = field(default_factory=TrainingConfig)

    @classmethod
    def from_yaml(cls, path: str | Path) -> "SSDConfig":
        return cls.from_dict(yaml.safe_load(Path(path).read_text()) or {})

    @classmethod
    def from_dict(cls, raw: dict) -> "SSDConfig":
        """Parse a whole config. draft_layers is required (0-based indices);
        the drafting section is validated on load."""
        layers = raw.get("draft_layers") if isinstance(raw, dict) else None
        if not (isinstance(layers, list) and all(isinstance(i, int) and not isinstance(i, bool) for i in layers)):
            raise ValueError(f"draft_layers must be a list of 0-based layer indices such as [0, 7, 15], "
                             f"got {layers!r}")
        cfg = _section(cls, raw, "config")
        cfg.drafting.validate()
        return cfg

    def validate_against(self, num_hidden_layers: int) -> None:
        """Check draft_layers against the base model's depth."""
        validate_layer_indices(self.draft_layers, num_hidden_layers)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


_NESTED.update({
    (SSDConfig, "model"): ModelConfig, (SSDConfig, "bridge"): BridgeConfig,
    (SSDConfig, "drafting"): DraftingConfig, (SSDConfig, "data"): DataConfig,
    (SSDConfig, "training"): TrainingConfig, (TrainingConfig, "stage1"): Stage1Config,
    (TrainingConfig, "stage2"): Stage2Config, (TrainingConfig, "online"): OnlineConfig,
})


def validate_layer_indices(layer_indices: list[int], num_hidden_layers: int) -> list[int]:
    """The selected base layers as ints: non-empty, strictly increasing and
    inside 0..num_hidden_layers-1 (ValueError otherwise)."""
    idx = [int(i) for i in layer_indices]
    if len(idx) == 0:
        raise ValueError("layer_indices is empty: select at least one base layer")
    for prev, cur in zip(idx, idx[1:]):
        if cur <= prev:
            raise ValueError(f"layer_indices must increase strictly: {prev} is followed by {cur} in {idx}")
    outside = [i for i in idx if not 0 <= i < num_hidden_layers]
    if outside:
        raise ValueError(f"layer_indices {outside} lie outside 0..{num_hidden_layers - 1} "
                         f"(0-based indices into a model of {num_hidden_layers} layers)")
    return idx
