"""Tensor-parallel parity worker (run under torchrun, one rank per GPU).

Builds the same global synthetic model sharded over the ranks, decodes
greedily target-only and speculatively, and (rank 0) writes the tokens, the
per-step argmax gaps and timings to the JSON file named by argv[1]. The
pytest side (tests/test_gpu_tp.py) compares them with a single-GPU run.
"""

import json
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "subnetwork-speculative-decoding_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

# the parity model: the 70B layer shape, fewer layers and a smaller vocabulary
MODEL = "llama3_70b"
OVERRIDES = dict(num_hidden_layers=4, vocab_size=32000)
DRAFT_LAYERS = [0, 3]
SEED, PROMPT, MAX_NEW = 5, 192, 40
DRAFTING = dict(depth=4, branch=[3, 2, 2, 1], width=8, max_nodes=24)


def build(rank: int, world: int, dev, single: bool):
    from ssd.config import BridgeConfig, DraftingConfig
    from ssd.engine import tp
    from ssd.engine.speculative import TargetRunner
    from ssd.models import SubnetworkDraftModel

    base = tp.build_tp_base(MODEL, SEED, torch.bfloat16, dev, rank, world, plant_layers=DRAFT_LAYERS,
                            plant_scale=0.05, **OVERRIDES)
    group = tp.TPGroup(base.config.hidden_size, PROMPT + 64, dev, group=None if single else "default")
    tp.attach(base, group)
    target = TargetRunner(base)
    draft = SubnetworkDraftModel(base, DRAFT_LAYERS, BridgeConfig(hidden_dim=8192))
    tp.init_bridges_device_(draft.bridges, SEED)
    draft.bridges.to(torch.bfloat16)
    return base, target, draft, DraftingConfig(**DRAFTING)


def ar_steps(target, prompt, max_new):
    """Greedy target-only decode one step at a time: tokens and the argmax gap of every step."""
    from ssd.engine.round import TargetStep, cache_capacity

    eng = TargetStep(target, target.new_cache(cache_capacity(prompt.numel(), max_new)), max_new)
    eng.prefill(prompt.to(target.weights.device))
    gaps = [float(eng.gap[0].item())]
    for _ in range(max_new - 1):
        eng.run(1)
        gaps.append(float(eng.gap[0].item()))
    eng.ws.check_status()
    return eng.tokens()[:max_new], gaps


def run(rank: int, world: int, dev, single: bool) -> dict:
    from ssd import synthetic as S
    from ssd.engine.speculative import SpeculativeGenerator

    base, target, draft, cfg = build(rank, world, dev, single)
    prompt = S.make_prompt(SEED, PROMPT, base.config.vocab_size)
    ar, gaps = ar_steps(target, prompt, MAX_NEW)
    gen = SpeculativeGenerator(base, draft, cfg, target=target)
    res = gen.generate(prompt, MAX_NEW, set())
    return dict(world=world, ar=ar, gaps=gaps, sd=res.tokens, accepted=res.accepted_per_round)


def main() -> None:
    out = sys.argv[1]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    res = run(rank, world, dev, single=world == 1)
    if world > 1:
        got = [None] * world
        dist.all_gather_object(got, res)
        res["replicated"] = all(g["sd"] == res["sd"] and g["ar"] == res["ar"] for g in got)
    if rank == 0:
        with open(out, "w") as f:
            json.dump(res, f)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
