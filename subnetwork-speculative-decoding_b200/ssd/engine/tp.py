"""Tensor parallelism for the 70B configuration: one process per GPU, the
layer weights split over the ranks, activations exchanged over NVLink peer
memory by the library's own kernels (no NCCL call on the decode path).

Split (Megatron-style, as the 70B configuration prescribes):
  * q/k/v by heads, gate/up by FFN columns (column-parallel): each rank owns
    H/world query heads, Hkv/world KV heads (its slice of the KV cache) and
    F/world FFN columns;
  * o_proj and down_proj by input features (row-parallel): each rank's GEMM
    gives a partial sum of the [T, d] output; ssd_tp_allreduce_residual adds
    the ranks' partials to the replicated residual stream;
  * lm_head by vocabulary rows: ssd_tp_head_argmax / ssd_tp_head_topk merge
    the ranks' per-row winners (lowest global index on ties);
  * embedding, norms and bridges replicated.
Every rank runs the same round on the same inputs; all exchanged results are
bit-identical on every rank (fixed rank-order sums), so the tree bookkeeping
runs replicated with no broadcast.

A rank's model is an ordinary LlamaForCausalLM of the shard's shape (H/world
heads, Hkv/world KV heads, F/world FFN width, the full model width and
vocabulary) whose lm_head holds the rank's V/world rows, so the draft model,
runner and engines use it unchanged; ``ModelWeights.tp`` carries the group.
Synthetic weights are drawn per shard on the device (ssd_fill_normal): the
value of a global matrix element depends only on (seed, parameter name,
element index), so every world size sees the same global model.
"""

from __future__ import annotations

import ctypes as C
import hashlib
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from ssd import _lib as L
from ssd import ops


class TPGroup:
    """A tensor-parallel group's exchange regions (SsdTpGroup).

    group: a torch.distributed process group; "default" (the default)
    selects the default group if torch.distributed is initialised, else a
    single-rank group; None selects a single-rank group. Each rank's region
    comes from torch symmetric memory and is mapped into every rank.
    """

    def __init__(self, d: int, max_rows: int, device, group="default"):
        import torch.distributed as dist

        if isinstance(group, str):
            group = dist.group.WORLD if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if self.world > L.TP_MAX_RANKS:
            raise ValueError(f"tensor parallelism supports at most {L.TP_MAX_RANKS} ranks")
        if d % 128:
            raise ValueError(f"model width {d} is not a multiple of 128")
        self.d, self.max_rows = int(d), int(max_rows)
        self.device = torch.device(device)
        lib = L.load()
        nbytes = int(lib.ssd_tp_region_bytes(self.max_rows, self.d))
        self._handle = None
        if self.world == 1:
            region = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            ptrs = [region.data_ptr()]
        else:
            # plain peer mappings: the kernels use no multicast object
            os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
            import torch.distributed._symmetric_memory as symm_mem

            region = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
            region.zero_()
            self._handle = symm_mem.rendezvous(region, group)
            ptrs = [int(self._handle.buffer_ptrs[p]) for p in range(self.world)]
            torch.cuda.synchronize(self.device)
            dist.barrier(group)  # every region is zeroed before any rank writes a flag into it
        self.region = region
        n = self.max_rows * self.d * 4
        self.partials = []
        for parity in (0, 1):
            off = int(lib.ssd_tp_partial_offset(self.max_rows, self.d, parity))
            self.partials.append(region[off:off + n].view(torch.float32).view(self.max_rows, self.d))
        self._calls = 0  # all-reduce calls issued since begin()
        arr = (C.c_void_p * L.TP_MAX_RANKS)(*ptrs, *([None] * (L.TP_MAX_RANKS - len(ptrs))))
        self._struct = L.SsdTpGroup(self.rank, self.world, self.max_rows, self.d, arr)

    def ref(self):
        return C.byref(self._struct)

    def check_rows(self, T: int) -> None:
        if T > self.max_rows:
            raise RuntimeError(f"tensor-parallel exchange holds {self.max_rows} rows, the forward has {T}")

    # Consecutive all-reduce calls must alternate the partial buffers, in the
    # order the GPU runs them, across forwards and CUDA graphs alike: every
    # forward starts at parity 0 (begin) and issues an even number of calls
    # (two per layer), so any concatenation of forwards alternates.
    def begin(self) -> None:
        self._calls = 0

    def next_parity(self) -> int:
        p = self._calls & 1
        self._calls += 1
        return p

    def end(self) -> None:
        if self._calls & 1:
            raise RuntimeError("a tensor-parallel forward issued an odd number of all-reduce calls")


# ------------------------------------------------------------ shard layout
@dataclass(frozen=True)
class ShardBlock:
    """Where a rank's tensor sits in its global matrix."""

    global_rows: int
    global_cols: int
    row0: int
    col0: int
    rows: int
    cols: int


def shard_block(name: str, shape_global: tuple, rank: int, world: int) -> ShardBlock:
    """Block of global parameter `name` (HF Llama naming) owned by `rank`."""
    if len(shape_global) == 1:
        return ShardBlock(1, shape_global[0], 0, 0, 1, shape_global[0])
    R, Cc = shape_global
    col_par = name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight", "gate_proj.weight", "up_proj.weight",
                             "lm_head.weight"))
    row_par = name.endswith(("o_proj.weight", "down_proj.weight"))
    if col_par:  # split the output features (rows of the [out, in] weight)
        if R % world:
            raise ValueError(f"{name}: {R} rows do not split over {world} ranks")
        r = R // world
        return ShardBlock(R, Cc, rank * r, 0, r, Cc)
    if row_par:  # split the input features (columns)
        if Cc % world:
            raise ValueError(f"{name}: {Cc} columns do not split over {world} ranks")
        c = Cc // world
        return ShardBlock(R, Cc, 0, rank * c, R, c)
    return ShardBlock(R, Cc, 0, 0, R, Cc)


def stream_id(name: str) -> int:
    """64-bit random-stream id of a global parameter name."""
    return int.from_bytes(hashlib.sha256(name.encode()).digest()[:8], "little")


def global_shapes(cfg) -> dict[str, tuple]:
    """Global (unsharded) shape of every parameter of a Llama config."""
    d, V, F = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size
    H, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    hd = getattr(cfg, "head_dim", None) or d // H
    out = {"model.embed_tokens.weight": (V, d), "model.norm.weight": (d,), "lm_head.weight": (V, d)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        out.update({p + "self_attn.q_proj.weight": (H * hd, d), p + "self_attn.k_proj.weight": (Hkv * hd, d),
                    p + "self_attn.v_proj.weight": (Hkv * hd, d), p + "self_attn.o_proj.weight": (d, H * hd),
                    p + "mlp.gate_proj.weight": (F, d), p + "mlp.up_proj.weight": (F, d),
                    p + "mlp.down_proj.weight": (d, F), p + "input_layernorm.weight": (d,),
                    p + "post_attention_layernorm.weight": (d,)})
    return out


def shard_config(cfg, world: int):
    """LlamaConfig of one rank's shard (same width and vocabulary)."""
    import copy

    H, Hkv, F = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    for what, n in (("attention heads", H), ("KV heads", Hkv), ("FFN width", F), ("vocabulary", cfg.vocab_size)):
        if n % world:
            raise ValueError(f"{what} ({n}) do not split over {world} ranks")
    sc = copy.deepcopy(cfg)
    sc.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // H
    sc.num_attention_heads = H // world
    sc.num_key_value_heads = Hkv // world
    sc.intermediate_size = F // world
    return sc


@torch.no_grad()
def build_tp_base(name: str, seed: int, dtype: torch.dtype, device, rank: int, world: int, *,
                  init_std: float = 0.02, plant_layers: Optional[list[int]] = None,
                  plant_scale: Optional[float] = None, **config_overrides):
    """This rank's shard of a synthetic Llama: weights N(0, init_std) drawn per
    element from (seed, parameter name, global index), norms 1, o_proj and
    down_proj of layers outside plant_layers scaled by plant_scale."""
    from transformers import LlamaForCausalLM
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from ssd.synthetic import llama_config

    cfg = llama_config(name, **config_overrides)
    shapes = global_shapes(cfg)
    scfg = shard_config(cfg, world)
    device = torch.device(device)
    with torch.device("meta"):
        model = LlamaForCausalLM(scfg)
        model.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size // world, bias=False)
    model.to(dtype=dtype)
    model.to_empty(device=device)
    keep = set(plant_layers or [])
    for pname, p in model.named_parameters():
        if pname not in shapes:
            raise ValueError(f"unexpected parameter {pname}")
        if p.dim() == 1:
            p.fill_(1.0)
            continue
        blk = shard_block(pname, shapes[pname], rank, world)
        if tuple(p.shape) != (blk.rows, blk.cols):
            raise ValueError(f"{pname}: shard shape {tuple(p.shape)} != {(blk.rows, blk.cols)}")
        scale = 1.0
        if plant_scale is not None and (".o_proj." in pname or ".down_proj." in pname):
            layer = int(pname.split(".")[2])
            if layer not in keep:
                scale = float(plant_scale)
        ops.fill_normal(p.data, blk.row0, blk.col0, blk.global_cols, seed, stream_id(pname), init_std, scale)
    model.config = scfg
    model.model.rotary_emb = LlamaRotaryEmbedding(config=scfg, device=device)
    model.eval().requires_grad_(False)
    object.__setattr__(model, "_ssd_tp_shard", (rank, world, cfg))
    return model


@torch.no_grad()
def init_bridges_device_(bridges, seed: int, in_std: float = 0.02, out_std: float = 1e-4) -> None:
    """Bridge weights drawn on their device per element (replicated on every
    rank): in-projections N(0, in_std), out-projection N(0, out_std), biases
    0, norm 1."""
    for bname in sorted(bridges.keys()):
        for pname, p in bridges[bname].named_parameters():
            if pname.startswith("norm"):
                p.fill_(1.0)
            elif pname.endswith("bias"):
                p.zero_()
            else:
                std = out_std if "out_proj" in pname else in_std
                ops.fill_normal(p.data, 0, 0, p.shape[1], seed, stream_id(f"bridges.{bname}.{pname}"), std)


def attach(base, group: TPGroup) -> None:
    """Make the runner and the engines of `base` (a build_tp_base shard) use
    the group: row-parallel outputs are all-reduced, the heads merged."""
    from ssd.models.runner import ModelWeights

    info = getattr(base, "_ssd_tp_shard", None)
    if info is None:
        raise ValueError("attach: base is not a tensor-parallel shard (build_tp_base)")
    rank, world, cfg = info
    if (group.rank, group.world) != (rank, world):
        raise ValueError(f"shard of rank {rank}/{world} attached to group rank {group.rank}/{group.world}")
    w = ModelWeights.of(base)
    w.tp = group
    w.V = cfg.vocab_size
    w.vocab_offset = rank * (cfg.vocab_size // world)
