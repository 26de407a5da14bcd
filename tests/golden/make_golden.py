"""Generate golden fixtures by running the REFERENCE implementation.

    python tests/golden/make_golden.py --ref PATH_TO_REFERENCE [--skip-1b]

Needs the reference checkout (importable as `ssd`; `--ref`, or the
SSD_REFERENCE environment variable) and runs on the CPU in fp32. Weights come from this repo's seeded synthetic builder
(subnetwork-speculative-decoding_b200/ssd/synthetic.py, loaded by path so it
does not clash with the reference's `ssd` package); a checksum of every model
is stored so a host whose CPU RNG differs is detected instead of silently
comparing different models.

Outputs (tests/golden/):
  tiny.json  - tiny-Llama cases mirroring the reference's own tests
               (tests/test_engine.py, tests/test_forward_pass.py): forward
               logits, AR tokens, greedy SD over four tree shapes x two
               drafts (+ first-round trees), draft-vocab subset, EOS stop,
               tree-attention-mask logits and keep_positions, sampling runs.
  c1.json    - BASELINE config 1 (Llama-3.2-1B shape, fp32, seed 0): prompt,
               target-only greedy tokens with top-2 gaps, SD chain tokens.
  c2ref.json - config-2 model (seed 1, planted, bf16-rounded weights) run in
               fp32 by the reference: greedy AR tokens + top-2 gaps, and per
               step the top-8 logits (values, ids) and the logits at 64 fixed
               probe ids: the reference for the bf16 tier. Section "bf16":
               the reference's own bf16 run of the same model (its modules
               in torch.bfloat16): its free-running greedy tokens and gaps,
               and its logits at the same ids teacher-forced on the fp32
               tokens, i.e. how far the reference's own bf16 arithmetic lands
               from its fp32 decode.
  sample_next.json - the reference's batched-generation sampler
               (ssd/data/generate_selfdistill.py:51-61: top-64 cut, then
               temperature + top-p) on seeded logit rows: per case the row,
               the settings and the token counts of many seeded draws; greedy
               rows record the argmax.
  warp_probs.json - the reference's warp_probs (ssd/engine/tree_drafter.py:
               34-45) on seeded full-vocabulary rows (regenerated from their
               seeds by the test; a checksum guards the stream): kept-token
               count and the 16 largest probabilities per case.
  verify.json - the reference's verify_inputs and greedy_verify
               (ssd/engine/verify.py:32-57) on seeded random trees with
               integer logits (exact ties exercise the first-maximum rule),
               and DraftTree's children / ancestors / subset
               (ssd/engine/tree_drafter.py:63-95) on the same trees.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
SYN_PATH = REPO / "subnetwork-speculative-decoding_b200" / "ssd" / "synthetic.py"


def load_synthetic():
    spec = importlib.util.spec_from_file_location("ssd_synthetic", SYN_PATH)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ssd_synthetic"] = mod
    spec.loader.exec_module(mod)
    return mod


TREES = {
    "chain": dict(depth=4, branch=1),
    "tree": dict(depth=3, branch=[3, 2, 2]),
    "pruned": dict(depth=5, branch=[4, 3, 2, 2, 1], width=[4, 6, 6, 4, 4], max_nodes=12),
    "deep_chain": dict(depth=8, branch=1),
}


def ref_ar_with_gaps(target, ids, n, eos=frozenset(), probe=None, record=None):
    """The reference's autoregressive_generate loop (ssd/engine/speculative.py:101-122),
    run step by step through the reference TargetRunner to also record each
    step's top-2 logit gap. With `record` (a dict), each step's top-8 logits
    (values and ids) and the logits at the `probe` ids are appended to it."""
    import torch

    cache = target.new_cache(ids.shape[1] + n + 1)

    def note(logits):
        top = logits.float().topk(8)
        gaps.append(float(top.values[0] - top.values[1]))
        if record is not None:
            record.setdefault("top_values", []).append([float(v) for v in top.values])
            record.setdefault("top_ids", []).append([int(i) for i in top.indices])
            record.setdefault("probe_logits", []).append([float(logits[j]) for j in probe])

    with torch.no_grad():
        gaps = []
        logits = target(ids, past_key_values=cache, logits_to_keep=1).logits[0, -1]
        out = [int(logits.argmax())]
        note(logits)
        while len(out) < n:
            logits = target(torch.tensor([[out[-1]]]), past_key_values=cache).logits[0, -1]
            out.append(int(logits.argmax()))
            note(logits)
    return out, gaps


def tree_dict(tree):
    return dict(tokens=list(tree.tokens), parents=list(tree.parents), depths=list(tree.depths),
                ranks=list(tree.ranks), scores=[float(s) for s in tree.scores], draft_pos=list(tree.draft_pos))


def make_tiny(syn, out_path: Path):
    import torch
    from ssd.config import BridgeConfig, DraftingConfig
    from ssd.data.token_freq import top_vocab
    from ssd.engine.speculative import SpeculativeGenerator, TargetRunner, autoregressive_generate
    from ssd.engine.tree_drafter import TreeDrafter
    from ssd.models import SubnetworkDraftModel

    res = {"model": "tiny", "seed": 0, "init_std": 0.02}
    base = syn.build_base_model("tiny", 0, torch.float32, "cpu")
    res["checksum"] = syn.weights_checksum(base)
    target = TargetRunner(base)
    eos = {-1}
    with torch.no_grad():
        ids = syn.make_prompt(100, 13, 128)
        res["forward"] = dict(ids=ids[0].tolist(), logits=target(ids).logits[0].tolist())
    prompts = [syn.make_prompt(s, 5 + 4 * s, 128) for s in range(3)]
    res["prompts"] = [p[0].tolist() for p in prompts]
    res["ar"] = [autoregressive_generate(target, p, 40, eos).tokens for p in prompts]
    drafts = {
        "untrained": ([0, 3, 5], dict(init_std=0.02)),
        "perfect": (list(range(6)), {}),
    }
    res["sd"] = {}
    for dname, (layers, bkw) in drafts.items():
        draft = SubnetworkDraftModel(base, layers, BridgeConfig(**bkw))
        if draft.bridges:
            syn.init_bridges_(draft.bridges, 0, in_std=0.125, out_std=0.02)
        for tname, tcfg in TREES.items():
            cfg = DraftingConfig(**tcfg)
            runs = []
            for p in prompts:
                r = SpeculativeGenerator(base, draft, cfg, target).generate(p, 40, eos)
                runs.append(dict(tokens=r.tokens, accepted_per_round=r.accepted_per_round, tree_sizes=r.tree_sizes))
            # first-round tree of prompt 0, built by the reference drafter
            cache = target.new_cache(64)
            with torch.no_grad():
                logits = target(prompts[0], past_key_values=cache, logits_to_keep=1).logits[0, -1]
                root = int(logits.argmax())
                committed = cache.get_seq_length()
                tree = TreeDrafter(draft, cfg).build(cache, torch.tensor([[root]]), committed)
            runs_tree = dict(root=root, committed=committed, tree=tree_dict(tree))
            res["sd"][f"{dname}/{tname}"] = dict(runs=runs, first_tree=runs_tree)
    # draft vocab subset (tests/test_engine.py:66-81)
    draft = SubnetworkDraftModel(base, list(range(6)))
    sub = top_vocab(torch.arange(128).flip(0), 40, always={127})
    draft.set_vocab_subset(sub)
    p = syn.make_prompt(5, 7, 128)
    r = SpeculativeGenerator(base, draft, DraftingConfig(**TREES["tree"]), target).generate(p, 40, eos)
    res["vocab_subset"] = dict(ids=sub.tolist(), prompt=p[0].tolist(), tokens=r.tokens,
                               accepted_per_round=r.accepted_per_round)
    # EOS stop (tests/test_engine.py:84-92)
    p = syn.make_prompt(6, 6, 128)
    free = autoregressive_generate(target, p, 30, eos).tokens
    e2 = {free[10]}
    ref = autoregressive_generate(target, p, 30, e2).tokens
    sd = SpeculativeGenerator(base, SubnetworkDraftModel(base, list(range(6))), DraftingConfig(**TREES["chain"]),
                              target).generate(p, 30, e2)
    res["eos"] = dict(prompt=p[0].tolist(), eos=sorted(e2), ar=ref, sd=sd.tokens)
    # tree attention mask + keep_positions (tests/test_forward_pass.py:146-180)
    draft = SubnetworkDraftModel(base, [0, 2, 5])
    syn.init_bridges_(draft.bridges, 1, in_std=0.125, out_std=0.02)
    prefix = syn.make_prompt(7, 6, 128)
    a, b, c, d = 10, 20, 30, 40
    parents = [-1, 0, 0, 1]
    depth = [0, 1, 1, 2]
    mask = torch.zeros(4, 4, dtype=torch.bool)
    for i in range(4):
        j = i
        while j != -1:
            mask[i, j] = True
            j = parents[j]
    pos = torch.tensor([[6 + dd for dd in depth]])
    with torch.no_grad():
        cache = draft.new_cache(32)
        draft(prefix, past_key_values=cache)
        tl = draft(torch.tensor([[a, b, c, d]]), position_ids=pos, past_key_values=cache,
                   tree_attention_mask=mask).logits[0]
        cache.keep_positions(6, torch.tensor([6, 7, 9]))
        nxt = draft(torch.tensor([[50]]), past_key_values=cache).logits[0, -1]
    res["tree_mask"] = dict(prefix=prefix[0].tolist(), tokens=[a, b, c, d], parents=parents, depth=depth,
                            logits=tl.tolist(), keep=[6, 7, 9], next_token=50, next_logits=nxt.tolist())
    # sampling runs (tiny_v8, tests/test_engine.py:173-207 setup)
    base8 = syn.build_base_model("tiny_v8", 1, torch.float32, "cpu")
    with torch.no_grad():
        base8.lm_head.weight.mul_(8.0)
    t8 = TargetRunner(base8)
    d8 = SubnetworkDraftModel(base8, [0, 5], BridgeConfig(init_std=0.05))
    syn.init_bridges_(d8.bridges, 2, in_std=0.125, out_std=0.05)
    samp = []
    for cfg in [dict(depth=2, branch=[2, 2], temperature=1.0), dict(depth=2, branch=1, temperature=0.8, top_p=0.9)]:
        sd = SpeculativeGenerator(base8, d8, DraftingConfig(**cfg), t8)
        samp.append(dict(cfg=cfg, tokens=[sd.generate(torch.tensor([[1, 5, 2]]), 3, set(), seed=s).tokens
                                          for s in range(50)]))
    res["sampling"] = dict(checksum=syn.weights_checksum(base8), runs=samp)
    out_path.write_text(json.dumps(res))
    print(f"wrote {out_path}")


def make_c1(syn, out_path: Path):
    import torch
    from ssd.config import BridgeConfig, DraftingConfig
    from ssd.engine.speculative import SpeculativeGenerator, TargetRunner
    from ssd.models import SubnetworkDraftModel

    spec = syn.CONFIGS["c1"]
    t0 = time.time()
    base = syn.build_base_model(spec.model, spec.seed, torch.float32, "cpu")
    print(f"c1 weights {time.time() - t0:.1f}s")
    target = TargetRunner(base)
    ids = syn.make_prompt(spec.seed, spec.prompt_len, base.config.vocab_size)
    t0 = time.time()
    ar, gaps = ref_ar_with_gaps(target, ids, spec.max_new_tokens)
    print(f"c1 AR {time.time() - t0:.1f}s")
    draft = SubnetworkDraftModel(base, spec.draft_layers, BridgeConfig(hidden_dim=spec.bridge_hidden))
    syn.init_bridges_(draft.bridges, spec.seed, spec.bridge_in_std, spec.bridge_out_std)
    t0 = time.time()
    sd = SpeculativeGenerator(base, draft, DraftingConfig(**spec.drafting), target).generate(
        ids, spec.max_new_tokens, set())
    print(f"c1 SD {time.time() - t0:.1f}s  acc {sd.mean_accepted:.2f}")
    res = dict(config="c1", checksum=syn.weights_checksum(base), prompt=ids[0].tolist(), ar=ar, gaps=gaps,
               sd=sd.tokens, accepted_per_round=sd.accepted_per_round, tree_sizes=sd.tree_sizes)
    out_path.write_text(json.dumps(res))
    print(f"wrote {out_path}")


def make_c2ref(syn, out_path: Path, n_new: int = 48):
    import torch
    from ssd.engine.speculative import TargetRunner

    spec = syn.CONFIGS["c2"]
    base = syn.build_base_model(spec.model, spec.seed, torch.float32, "cpu", plant_layers=spec.draft_layers,
                                plant_scale=spec.plant_scale)
    with torch.no_grad():  # the bf16 model's weights, evaluated in fp32
        for p in base.parameters():
            p.copy_(p.bfloat16().float())
    target = TargetRunner(base)
    ids = syn.make_prompt(spec.seed, spec.prompt_len, base.config.vocab_size)
    probe = torch.randperm(base.config.vocab_size, generator=torch.Generator().manual_seed(11))[:64].tolist()
    rec: dict = {}
    ar, gaps = ref_ar_with_gaps(target, ids, n_new, probe=probe, record=rec)
    res = dict(config="c2", checksum=syn.weights_checksum(base), prompt=ids[0].tolist(), ar=ar, gaps=gaps,
               probe_ids=probe, **rec, note="weights rounded to bf16, evaluated by the reference in fp32")
    # the reference's own bf16 arithmetic on the same weights
    base = base.to(torch.bfloat16)
    target = TargetRunner(base)
    ar16, gaps16 = ref_ar_with_gaps(target, ids, n_new)
    cache = target.new_cache(ids.shape[1] + n_new + 1)
    with torch.no_grad():
        rows = [target(ids, past_key_values=cache, logits_to_keep=1).logits[0, -1].float()]
        for t in ar[:-1]:
            rows.append(target(torch.tensor([[t]]), past_key_values=cache).logits[0, -1].float())
    res["bf16"] = dict(ar=ar16, gaps=gaps16,
                       tf_top_values=[[float(r[j]) for j in rec["top_ids"][i]] for i, r in enumerate(rows)],
                       tf_probe_logits=[[float(r[j]) for j in probe] for r in rows],
                       tf_argmax=[int(r.argmax()) for r in rows],
                       note="the reference's modules in torch.bfloat16 (CPU); tf_* teacher-forced on the fp32 tokens")
    out_path.write_text(json.dumps(res))
    print(f"wrote {out_path}")


# (temperature, top_p) per row of sample_next.json: the cut alone, a nucleus
# inside the 64 kept logits, a sharp and a flat temperature
SAMPLE_NEXT_CASES = [(1.0, 1.0), (0.7, 0.9), (1.3, 0.5), (0.5, 0.95), (2.0, 0.8)]


def make_sample_next(out_path: Path, vocab: int = 300, draws: int = 40000):
    """The reference's sample_next on seeded rows of `vocab` logits (more than
    the 64 it keeps): counts of `draws` tokens drawn with a seeded torch
    generator (one batched call per case), and the greedy argmax."""
    import torch
    from ssd.data.generate_selfdistill import sample_next

    g = torch.Generator().manual_seed(11)
    cases = []
    for i, (temp, top_p) in enumerate(SAMPLE_NEXT_CASES):
        row = torch.randn(vocab, generator=g, dtype=torch.float64).float() * (1.0 + i)
        gen = torch.Generator().manual_seed(100 + i)
        tok = sample_next(row.expand(draws, vocab).contiguous(), temp, top_p, gen)[:, 0]
        counts = torch.bincount(tok, minlength=vocab)
        cases.append(dict(logits=[float(x) for x in row], temperature=temp, top_p=top_p, draws=draws,
                          counts=[int(c) for c in counts],
                          greedy=int(sample_next(row[None], 0.0, 1.0)[0, 0])))
    out_path.write_text(json.dumps(dict(vocab=vocab, keep=64, cases=cases)))
    print(f"wrote {out_path}")


# (logit scale, temperature, top_p) per row of warp_probs.json
WARP_CASES = [(1.0, 0.7, 0.9), (3.0, 1.0, 0.5), (8.0, 1.5, 0.99), (2.0, 0.6, 0.95), (0.5, 1.0, 0.8),
              (4.0, 0.9, 0.3), (2.0, 1.0, 1.0)]


def warp_row(seed: int, scale: float, vocab: int = 128256):
    """Seeded fp32 logit row of warp_probs.json (torch CPU generator)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    return (torch.randn(vocab, generator=g, dtype=torch.float64) * scale).float()


def make_warp_probs(out_path: Path):
    from ssd.engine.tree_drafter import warp_probs

    cases = []
    for i, (scale, temp, top_p) in enumerate(WARP_CASES):
        row = warp_row(1000 + i, scale)
        p = warp_probs(row, temp, top_p)
        top = p.topk(16)
        cases.append(dict(seed=1000 + i, scale=scale, temperature=temp, top_p=top_p,
                          row_sum=float(row.double().sum()), row_sq=float(row.double().square().sum()),
                          n_kept=int((p > 0).sum()), top_ids=[int(x) for x in top.indices],
                          top_probs=[float(x) for x in top.values]))
    out_path.write_text(json.dumps(dict(vocab=128256, cases=cases), indent=1))
    print(f"wrote {out_path}")


def random_tree(g, n: int, vocab: int):
    """Seeded tree in the drafter's order (every parent before its children),
    distinct sibling tokens, sibling ranks a random permutation."""
    import torch

    parents, depths, tokens, ranks = [], [], [], []
    kids: dict = {}
    for i in range(n):
        par = -1 if i == 0 or int(torch.randint(0, 4, (1,), generator=g)) == 0 else int(torch.randint(0, i, (1,), generator=g))
        used = {tokens[c] for c in kids.get(par, [])}
        free = [t for t in range(vocab) if t not in used]
        tok = free[int(torch.randint(0, len(free), (1,), generator=g))]
        kids.setdefault(par, []).append(i)
        parents.append(par)
        depths.append(1 if par == -1 else depths[par] + 1)
        tokens.append(tok)
        ranks.append(len(kids[par]) - 1)
    for sib in kids.values():  # proposal order among siblings: a random permutation
        perm = torch.randperm(len(sib), generator=g).tolist()
        for c, r in zip(sib, perm):
            ranks[c] = r
    return tokens, parents, depths, ranks


def make_verify(out_path: Path, vocab: int = 12):
    import torch
    from ssd.engine.tree_drafter import DraftTree
    from ssd.engine.verify import greedy_verify, verify_inputs

    g = torch.Generator().manual_seed(31)
    cases = []
    for n in (0, 1, 3, 7, 12, 20, 31, 40):
        tokens, parents, depths, ranks = random_tree(g, n, vocab)
        tree = DraftTree(tokens=tokens, parents=parents, depths=depths, scores=[0.0] * n, ranks=ranks,
                         draft_pos=[-1] * n)
        root_token, root_pos = int(torch.randint(0, vocab, (1,), generator=g)), int(torch.randint(0, 50, (1,), generator=g))
        past = root_pos
        logits = torch.randint(0, 4, (n + 1, vocab), generator=g).float()  # ties everywhere
        cur = -1  # plant a path: each accepted node's row favours one of its children
        while True:
            kids = [c for c in range(n) if parents[c] == cur]
            if not kids or int(torch.randint(0, 5, (1,), generator=g)) == 0:
                break
            c = kids[int(torch.randint(0, len(kids), (1,), generator=g))]
            logits[cur + 1, tokens[c]] = 4.0
            cur = c
        ids, pos, mask = verify_inputs(tree, root_token, root_pos, past, "cpu")
        acc, bonus = greedy_verify(tree, logits)
        # DraftTree's own methods: children, ancestors, and the subset of an
        # ancestor-closed random node set (its remapped arrays)
        pick = [i for i in range(n) if int(torch.randint(0, 3, (1,), generator=g)) == 0]
        keep = sorted({a for i in pick for a in tree.ancestors(i)})
        sub = tree.subset(keep)
        cases.append(dict(tokens=tokens, parents=parents, depths=depths, ranks=ranks, root_token=root_token,
                          root_pos=root_pos, past=past, logits=logits.int().tolist(), ids=ids[0].tolist(),
                          positions=pos[0].tolist(), mask_rows=[[int(j) for j in torch.nonzero(r)[:, 0]] for r in mask],
                          accepted=acc, bonus=int(bonus),
                          children={str(k): v for k, v in tree.children().items()},
                          ancestors=[tree.ancestors(i) for i in range(n)], keep=keep,
                          subset=dict(tokens=sub.tokens, parents=sub.parents, depths=sub.depths, ranks=sub.ranks)))
    out_path.write_text(json.dumps(dict(vocab=vocab, cases=cases)))
    print(f"wrote {out_path}")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref", default=os.environ.get("SSD_REFERENCE"), required="SSD_REFERENCE" not in os.environ,
                    help="path of the reference checkout (default: $SSD_REFERENCE)")
    ap.add_argument("--skip-1b", action="store_true")
    ap.add_argument("--only", choices=["tiny", "c1", "c2ref", "sample_next", "warp_probs", "verify"])
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    syn = load_synthetic()
    if a.only in (None, "tiny"):
        make_tiny(syn, HERE / "tiny.json")
    if not a.skip_1b and a.only in (None, "c1"):
        make_c1(syn, HERE / "c1.json")
    if not a.skip_1b and a.only in (None, "c2ref"):
        make_c2ref(syn, HERE / "c2ref.json")
    if a.only in (None, "sample_next"):
        make_sample_next(HERE / "sample_next.json")
    if a.only in (None, "warp_probs"):
        make_warp_probs(HERE / "warp_probs.json")
    if a.only in (None, "verify"):
        make_verify(HERE / "verify.json")


if __name__ == "__main__":
    main()
