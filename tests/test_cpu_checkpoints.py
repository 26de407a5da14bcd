"""Bridge checkpoints (subnetwork_draft.py:455-472) and their discovery
(runtime.py:87-98), on the CPU: a checkpoint written by the REFERENCE's
save_bridges (tests/golden/tiny_bridges.pt, made by
tests/golden/make_bridge_ckpt.py) loads into this package's draft model, this
package writes the same format, and build_draft picks online > stage2 > stage1."""

import shutil
from pathlib import Path

import pytest
import torch

from ssd import runtime
from ssd import synthetic as S
from ssd.config import BridgeConfig, SSDConfig, profile_name
from ssd.models import SubnetworkDraftModel

GOLD = Path(__file__).parent / "golden" / "tiny_bridges.pt"
LAYERS = [0, 3, 5]


@pytest.fixture(scope="module")
def base():
    return S.build_base_model("tiny", 0)


def _expected(base):
    d = SubnetworkDraftModel(base, LAYERS, BridgeConfig())
    S.init_bridges_(d.bridges, 0, in_std=0.02, out_std=1e-4)
    return d.bridges.state_dict()


def test_reference_checkpoint_loads(base):
    ckpt = torch.load(GOLD, weights_only=True)
    assert set(ckpt) == {"layer_indices", "bridge_config", "state_dict", "meta"}
    assert ckpt["meta"] == {"stage": 2, "step": 123}
    draft = SubnetworkDraftModel(base, LAYERS, BridgeConfig(**ckpt["bridge_config"]))
    draft.load_bridges(str(GOLD))
    want = _expected(base)
    got = draft.bridges.state_dict()
    assert set(got) == set(want)
    for k in want:
        assert torch.equal(got[k], want[k]), k


def test_checkpoint_round_trip_and_layer_check(base, tmp_path):
    src = SubnetworkDraftModel(base, LAYERS, BridgeConfig())
    S.init_bridges_(src.bridges, 7)
    path = tmp_path / "sub" / "b.pt"
    src.save_bridges(str(path), stage=1, step=5)
    ckpt = torch.load(path, weights_only=True)
    assert ckpt["layer_indices"] == LAYERS and ckpt["meta"] == {"stage": 1, "step": 5}
    assert ckpt["bridge_config"] == vars(BridgeConfig())
    dst = SubnetworkDraftModel(base, LAYERS, BridgeConfig())
    dst.load_bridges(str(path))
    for k, v in src.bridges.state_dict().items():
        assert torch.equal(dst.bridges.state_dict()[k], v)
    other = SubnetworkDraftModel(base, [0, 2, 5], BridgeConfig())
    with pytest.raises(ValueError):
        other.load_bridges(str(path))


def test_checkpoint_discovery_order(base, tmp_path):
    cfg = SSDConfig(draft_layers=LAYERS)
    cfg.training.output_dir = str(tmp_path)
    assert runtime.checkpoint_path(cfg, 2) == tmp_path / profile_name(LAYERS) / "stage2.pt"
    assert runtime.latest_checkpoint(cfg) is None
    prof = tmp_path / profile_name(LAYERS)
    prof.mkdir()
    shutil.copy(GOLD, prof / "stage1.pt")
    assert runtime.latest_checkpoint(cfg) == prof / "stage1.pt"
    shutil.copy(GOLD, prof / "stage2.pt")
    assert runtime.latest_checkpoint(cfg) == prof / "stage2.pt"
    shutil.copy(GOLD, prof / "online.pt")
    assert runtime.latest_checkpoint(cfg) == prof / "online.pt"
    draft = runtime.build_draft(cfg, base, "latest")
    want = _expected(base)
    for k, v in draft.bridges.state_dict().items():
        assert torch.equal(v, want[k]), k


def test_top_vocab_matches_reference_subset():
    """ssd.data.token_freq.top_vocab (token_freq.py:49-55) gives the subset the
    reference chose for the recorded vocab-subset run (tests/golden/tiny.json)."""
    import json

    from ssd.data.token_freq import top_vocab

    gold = json.loads((Path(__file__).parent / "golden" / "tiny.json").read_text())["vocab_subset"]
    sub = top_vocab(torch.arange(128).flip(0), 40, always={127})
    assert sub.tolist() == gold["ids"]
    # ties keep the stable descending-count order; forced ids count toward the size
    counts = torch.tensor([5, 9, 9, 1, 9, 0])
    assert top_vocab(counts, 3).tolist() == [1, 2, 4]
    assert top_vocab(counts, 3, always={5}).tolist() == [1, 2, 5]
