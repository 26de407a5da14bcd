"""CPU tests: the C-ABI library loads and exports every symbol the header
declares; host-side logic (config schema and validation, bridge planning,
static tree plans, mask conversion) matches the reference's behaviour."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from ssd import _lib as L
from ssd.config import DraftingConfig, SSDConfig, profile_name, validate_layer_indices
from ssd.engine.round import TreePlan, cache_capacity
from ssd.models.subnetwork_draft import plan_bridges

HEADER = Path(__file__).resolve().parent.parent / "include" / "ssd_b200.h"


def header_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(ssd_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = header_symbols()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), f"{n} declared in ssd_b200.h but not exported"
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"
    assert set(L.SIGNATURES) <= set(names)
    assert lib.ssd_version() == 1


def test_library_rejects_bad_arguments_without_gpu():
    """Argument validation happens on the host, before any launch."""
    with pytest.raises(ValueError):
        L.call("ssd_tree_attention", None, 0, 1, 3, 2, 16, None, None, 0, 0, None, None, None, None, 0, 0, None, 0,
               0, None, 0, None, None)
    with pytest.raises(L.SSDError):
        L.call("ssd_kv_compact", None, 1, 1, 1, 1, 1, 64, None, None, None, 99, 1, None, None)
    # GEMM chains: link count, dtype and row limits are checked before any CUDA call
    links = (L.SsdLinearArgs * 1)()
    with pytest.raises(ValueError):
        L.call("ssd_linear_chain", 0, ctypes.cast(links, ctypes.c_void_p), 4, L.SSD_BF16, None, 0, None, None)
    with pytest.raises(L.SSDError):
        L.call("ssd_linear_chain", 1, ctypes.cast(links, ctypes.c_void_p), 4, L.SSD_F32, None, 0, None, None)
    with pytest.raises(ValueError):
        L.call("ssd_linear_chain", 1, ctypes.cast(links, ctypes.c_void_p), 4, L.SSD_BF16, None, 0, None, None)  # no x


def _call_with(name: str, **at):
    """Call entry point `name` with zeros / NULL / 1.0 in every argument
    except the positions given as a<index>=value."""
    res, types = L.SIGNATURES[name]
    args = []
    for i, t in enumerate(types):
        if f"a{i}" in at:
            args.append(at[f"a{i}"])
        elif t is ctypes.c_void_p:
            args.append(None)
        elif t is ctypes.c_float:
            args.append(1.0)
        else:
            args.append(0)
    L.call(name, *args)


# (entry point, arguments that break its first host-side check, exception):
# each is rejected before any pointer is read or any CUDA call is made
BAD_CALLS = [
    ("ssd_warp_params", dict(a2=0, a3=10), ValueError),  # no rows
    ("ssd_warp_params", dict(a2=1, a3=10, a4=0.0), ValueError),  # temperature 0
    ("ssd_warp_params", dict(a2=1, a3=10, a5=1.5), ValueError),  # top_p > 1
    ("ssd_warp_probs", dict(a2=0, a3=10), ValueError),
    ("ssd_gumbel_topk", dict(a2=1, a3=10, a5=17), L.SSDError),  # k beyond 16
    ("ssd_warp_sample_topk", dict(a2=1, a3=10, a6=0, a7=-1), ValueError),  # negative keep_top
    ("ssd_warp_sample_topk", dict(a2=0, a3=10), ValueError),  # no rows
    ("ssd_sample_token", dict(a1=0), ValueError),  # empty vocabulary
    ("ssd_tree_walk_sample", dict(a1=5000), ValueError),  # more nodes than a tree holds
    ("ssd_level_prune", dict(a2=0, a3=2), ValueError),  # empty frontier
    ("ssd_level_prune", dict(a2=1000, a3=16), ValueError),  # 16 000 candidates
    ("ssd_tree_prune", dict(a8=0), ValueError),  # no capacity
    ("ssd_verify_prep", dict(a1=130, a13=2), ValueError),  # 129 nodes over a 128-slot mask
    ("ssd_tree_walk_greedy", dict(a1=-1), ValueError),
    ("ssd_causal_prep", dict(a1=0), ValueError),
    ("ssd_linear_noalloc", dict(a2=65, a3=4096, a4=1), L.SSDError),  # beyond its fixed scratch
    ("ssd_linear_noalloc", dict(a2=0, a3=4096, a4=1), L.SSDError),
]


@pytest.mark.parametrize("name,bad,exc", BAD_CALLS, ids=[f"{c[0]}-{i}" for i, c in enumerate(BAD_CALLS)])
def test_entry_points_reject_bad_shapes_before_any_launch(name, bad, exc):
    """Status codes map to the reference's exception types (invalid argument:
    ValueError; unsupported size: the library's RuntimeError subclass), with
    the failing entry point named in the message."""
    with pytest.raises(exc, match=name):
        _call_with(name, **bad)


YAML = """
model:
  base_model: meta-llama/Llama-3.2-1B-Instruct
  torch_dtype: bfloat16
draft_layers: [0, 7, 15]
bridge:
  hidden_dim: 4096
drafting:
  depth: 4
  branch: [3, 2, 2, 1]
  width: 8
  max_nodes: 24
  draft_vocab: 32768
training:
  output_dir: outputs/l1b
  stage1: {steps: 10}
"""


def test_config_roundtrip(tmp_path):
    p = tmp_path / "c.yaml"
    p.write_text(YAML)
    cfg = SSDConfig.from_yaml(p)
    assert cfg.draft_layers == [0, 7, 15] and cfg.bridge.hidden_dim == 4096
    assert cfg.drafting.per_depth(cfg.drafting.branch, "branch") == [3, 2, 2, 1]
    assert cfg.training.stage1.steps == 10
    assert profile_name(cfg.draft_layers) == "L0-7-15"


@pytest.mark.parametrize("bad", ["drafting: {depth: 0}\ndraft_layers: [0]", "draft_layers: 3",
                                 "draft_layers: [0]\nbogus: 1", "draft_layers: [0]\ndrafting: {nope: 1}",
                                 "draft_layers: [0]\ndrafting: {depth: 2, branch: [1, 2, 3]}",
                                 "draft_layers: [0]\ndrafting: {top_p: 0}"])
def test_config_rejects(tmp_path, bad):
    p = tmp_path / "bad.yaml"
    p.write_text(bad)
    with pytest.raises(ValueError):
        SSDConfig.from_yaml(p)


@pytest.mark.parametrize("bad", [[0, 6], [3, 3], [4, 2], []])
def test_invalid_layer_indices(bad):
    with pytest.raises(ValueError):
        validate_layer_indices(bad, 6)


def test_plan_bridges_matches_reference_naming():
    assert [(s.name, s.src_boundary, s.tgt_boundary) for s in plan_bridges([0, 2, 5], 6)] == [
        ("into_2", 1, 2), ("into_5", 3, 5)]
    assert [s.name for s in plan_bridges([1, 2, 4], 6)] == ["into_1", "into_4", "into_norm"]
    assert [s.name for s in plan_bridges([0, 15, 31], 32)] == ["into_15", "into_31"]


@pytest.mark.parametrize("cfg,levels,verify,cache", [
    (dict(depth=4, branch=[3, 2, 2, 1], width=8, max_nodes=24), [3, 6, 8, 8], 24, 17),
    (dict(depth=6, branch=[4, 2, 2, 1, 1, 1], max_nodes=32), [4, 8, 16, 16, 16, 16], 32, 60),
    (dict(depth=4, branch=1), [1, 1, 1, 1], 4, 3),
    (dict(depth=5, branch=[4, 3, 2, 2, 1], width=[4, 6, 6, 4, 4], max_nodes=12), [4, 6, 6, 4, 4], 12, 20),
])
def test_tree_plan_static_sizes(cfg, levels, verify, cache):
    """Same level sizes / verify nodes / tree cache as the reference's
    TreeDrafter.max_nodes_per_level, max_verify_nodes, max_tree_cache."""
    p = TreePlan(DraftingConfig(**cfg))
    assert p.level_sizes == levels and p.n_verify == verify and p.max_tree_cache == cache
    assert p.rows == verify + 1
    assert cache_capacity(2048, 256, p) >= 2048 + 256 + cfg["depth"] + max(verify, cache) + 2


def test_forward_inputs_mask_conversion():
    """A dense [q, past+q] tree mask becomes prefix length + bitmask."""
    from ssd.models.runner import ForwardInputs

    class _Dev:
        pass

    fi = ForwardInputs.__new__(ForwardInputs)
    fi.cap, fi.mask_words = 8, 2
    fi.ids = torch.zeros(8, dtype=torch.int32)
    fi.positions = torch.zeros(8, dtype=torch.int32)
    fi.slots = torch.zeros(8, dtype=torch.int32)
    fi.prefix_len = torch.zeros(8, dtype=torch.int32)
    fi.spec_base = torch.zeros(1, dtype=torch.int32)
    fi.mask = torch.zeros(8, 2, dtype=torch.int64)
    past, T = 6, 4
    parents = [-1, 0, 0, 1]
    m = torch.zeros(T, past + T, dtype=torch.bool)
    m[:, :past] = True
    for i in range(T):
        j = i
        while j != -1:
            m[i, past + j] = True
            j = parents[j]
    fi.fill(torch.tensor([1, 2, 3, 4]), torch.tensor([6, 7, 7, 8]), past, m)
    # node 0 is an ancestor of every row -> it joins the prefix
    assert fi.prefix_len[:T].tolist() == [past + 1] * T and int(fi.spec_base) == past + 1
    assert fi.mask[:T, 0].tolist() == [0, 0b001, 0b010, 0b101]
    fi.fill(torch.tensor([5, 6]), torch.tensor([6, 7]), past, None)
    assert fi.prefix_len[:2].tolist() == [past + 1, past + 2] and not fi.use_mask


def _random_tree(seed: int, n: int, vocab: int = 50):
    """A random draft tree in the drafter's storage order (parents first),
    siblings ranked in proposal order."""
    import random

    from ssd.engine.tree_drafter import ROOT, DraftTree

    rng = random.Random(seed)
    t = DraftTree()
    n_kids: dict = {}
    for i in range(n):
        parent = rng.choice([ROOT] + list(range(i))) if i else ROOT
        t.tokens.append(rng.randrange(vocab))
        t.parents.append(parent)
        t.depths.append(1 if parent == ROOT else t.depths[parent] + 1)
        t.scores.append(-rng.random())
        t.ranks.append(n_kids.get(parent, 0))
        t.draft_pos.append(i)
        n_kids[parent] = n_kids.get(parent, 0) + 1
    return t


@pytest.mark.parametrize("seed,n,past", [(0, 1, 0), (1, 7, 5), (2, 24, 13), (3, 32, 100)])
def test_verify_inputs_match_oracle(seed, n, past):
    """verify_inputs (verify.py:32-42): ids, positions and the bool mask equal
    the oracle's ancestor-walk restatement on random trees."""
    import numpy as np

    from oracle import tree as OT
    from ssd.engine.verify import verify_inputs

    t = _random_tree(seed, n)
    ot = OT.DraftTree(tokens=list(t.tokens), parents=list(t.parents), depths=list(t.depths), scores=list(t.scores),
                      ranks=list(t.ranks), draft_pos=list(t.draft_pos))
    ids, pos, mask = verify_inputs(t, 9, past, past, "cpu")
    rids, rpos, rmask = OT.verify_inputs(ot, 9, past, past)
    assert ids[0].tolist() == rids and pos[0].tolist() == rpos
    assert np.array_equal(mask.numpy(), rmask)


def test_kv_cache_protocol_on_the_host():
    """KVCache's host protocol (ssd/engine/kv_cache.py:21-73 of the reference):
    update writes at [len, len + q) and returns the views up to len + q;
    advance moves the length; crop discards the tail (a longer crop is a
    ValueError); overflow is a RuntimeError; keep_positions of positions
    already in place only sets the length (no kernel)."""
    import torch

    from ssd.engine.kv_cache import KVCache

    c = KVCache(2, 6)
    k1, v1 = torch.arange(12.0).view(1, 2, 3, 2), -torch.arange(12.0).view(1, 2, 3, 2)
    k, v = c.update(1, k1, v1)
    assert k.shape == (1, 2, 3, 2) and torch.equal(k, k1) and torch.equal(v, v1)
    c.advance(3)
    assert c.get_seq_length() == 3
    k, _ = c.update(1, k1[:, :, :2] + 100, v1[:, :, :2])
    assert k.shape == (1, 2, 5, 2) and torch.equal(k[:, :, :3], k1) and torch.equal(k[:, :, 3:], k1[:, :, :2] + 100)
    c.advance(2)
    with pytest.raises(RuntimeError, match="overflow"):
        c.update(0, k1[:, :, :2], v1[:, :, :2])
    with pytest.raises(ValueError):
        c.crop(6)
    c.crop(4)
    assert c.get_seq_length() == 4
    c.keep_positions(2, [2, 3])
    assert c.get_seq_length() == 4
    c.reset()
    assert c.get_seq_length() == 0
