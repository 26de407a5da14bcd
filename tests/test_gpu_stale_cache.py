"""Stale-read check of the round (the race-detection plan for this path: a
kernel that reads a cache slot it has not written this round shows up as a
changed output). Every key and value slot past the prompt is overwritten with
large finite garbage after the prefill; the decode must not change: same
tokens, same committed tokens per round. Masked slots must contribute exact
zeros (garbage, not NaN: a masked probability of 0 times a NaN value is NaN
in any matrix product, so NaN poison would test the arithmetic, not the
masking)."""

import pytest
import torch

from ssd import synthetic as S
from ssd.config import BridgeConfig, DraftingConfig
from ssd.engine.round import GreedyRound, TreePlan, cache_capacity
from ssd.engine.speculative import TargetRunner, _finish
from ssd.models import SubnetworkDraftModel

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TREE = dict(depth=5, branch=[4, 3, 2, 2, 1], width=[4, 6, 6, 4, 4], max_nodes=12)


def _decode(target, draft, cfg, prompt, max_new: int, poison: bool):
    eng = GreedyRound(target, draft, cfg, target.new_cache(cache_capacity(prompt.numel(), max_new, TreePlan(cfg))),
                      max_new)
    eng.prefill(prompt.to(DEV))
    if poison:
        buf = eng.cache.buf  # [layers, k/v, kv heads, slots, head_dim]
        g = torch.Generator(device=DEV).manual_seed(5)
        tail = buf[:, :, :, prompt.numel():]
        tail.copy_(torch.randn(tail.shape, generator=g, device=DEV, dtype=torch.float32) * 50)
    out = eng.tokens()
    while not _finish(out, set(), max_new)[1]:
        eng.run_round(True)
        out = eng.tokens()
    eng.ws.check_status()
    return out[:max_new], list(eng.committed_per_round())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stale_cache_slots_never_reach_the_output(dtype):
    base = S.build_base_model("tiny", 0, torch.float32, "cpu").to(dtype).to(DEV)
    target = TargetRunner(base)
    draft = SubnetworkDraftModel(base, [0, 3, 5], BridgeConfig(init_std=0.02))
    S.init_bridges_(draft.bridges, 0, in_std=0.125, out_std=0.02)
    draft.bridges.to(dtype)
    cfg = DraftingConfig(**TREE)
    for s, n in ((3, 37), (4, 70)):
        prompt = S.make_prompt(s, n, 128)
        clean = _decode(target, draft, cfg, prompt, 40, poison=False)
        dirty = _decode(target, draft, cfg, prompt, 40, poison=True)
        assert dirty == clean
