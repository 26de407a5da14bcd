"""Pin the CPU oracle against golden fixtures produced by the reference itself
(tests/golden/make_golden.py). CPU only."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from oracle.model import bridges_from_module, weights_from_hf
from ssd import synthetic as S
from ssd.config import BridgeConfig

GOLD = Path(__file__).parent / "golden"


@pytest.fixture(scope="module")
def tiny():
    return json.loads((GOLD / "tiny.json").read_text())


@pytest.fixture(scope="module")
def base():
    return S.build_base_model("tiny", 0, torch.float32, "cpu")


def make_bridges(d, layers, n_layers, seed, in_std, out_std, cfg=None):
    from ssd.models.bridges import TransitionBridge
    from ssd.models.subnetwork_draft import plan_bridges

    cfg = cfg or BridgeConfig()
    mods = torch.nn.ModuleDict({s.name: TransitionBridge.from_config(d, cfg) for s in plan_bridges(layers, n_layers)})
    S.init_bridges_(mods, seed, in_std=in_std, out_std=out_std)
    return bridges_from_module(mods, vars(cfg))


def oracle_models(base, layers, bridges=None):
    w, conf = weights_from_hf(base)
    target = O.OracleModel(w, conf, list(range(conf["layers"])))
    draft = O.OracleModel(w, conf, layers, bridges)
    return target, draft


def test_weights_checksum(tiny, base):
    assert S.weights_checksum(base) == tiny["checksum"], "CPU RNG on this host differs from the fixture host"


def test_forward_logits(tiny, base):
    target, _ = oracle_models(base, list(range(6)))
    logits = target.forward(tiny["forward"]["ids"])
    np.testing.assert_allclose(logits, np.array(tiny["forward"]["logits"]), atol=1e-5, rtol=1e-4)


def test_autoregressive_tokens(tiny, base):
    target, _ = oracle_models(base, list(range(6)))
    for p, ref in zip(tiny["prompts"], tiny["ar"]):
        assert O.autoregressive_generate(target, p, 40, {-1})["tokens"] == ref


TREES = {
    "chain": dict(depth=4, branch=1),
    "tree": dict(depth=3, branch=[3, 2, 2]),
    "pruned": dict(depth=5, branch=[4, 3, 2, 2, 1], width=[4, 6, 6, 4, 4], max_nodes=12),
    "deep_chain": dict(depth=8, branch=1),
}


@pytest.mark.parametrize("draft_kind", ["untrained", "perfect"])
@pytest.mark.parametrize("tree_name", list(TREES))
def test_speculative_rounds(tiny, base, draft_kind, tree_name):
    layers = [0, 3, 5] if draft_kind == "untrained" else list(range(6))
    br = make_bridges(64, layers, 6, 0, 0.125, 0.02, BridgeConfig(init_std=0.02)) if draft_kind == "untrained" else {}
    target, draft = oracle_models(base, layers, br)
    gold = tiny["sd"][f"{draft_kind}/{tree_name}"]
    for p, run in zip(tiny["prompts"], gold["runs"]):
        res = O.speculative_generate(target, draft, TREES[tree_name], p, 40, {-1})
        assert res["tokens"] == run["tokens"]
        assert res["accepted_per_round"] == run["accepted_per_round"]
        assert res["tree_sizes"] == run["tree_sizes"]
    # the first round's tree, structure and scores
    ft = gold["first_tree"]
    cache = target.new_cache(64)
    logits = target.forward(tiny["prompts"][0], None, cache, logits_to_keep=1)[-1]
    assert int(np.argmax(logits)) == ft["root"]
    drafter = O.OracleTreeDrafter(draft, **{k: TREES[tree_name].get(k) for k in ("depth", "branch", "width",
                                                                                  "max_nodes")})
    tree = drafter.build(cache, [ft["root"]], ft["committed"])
    ref = ft["tree"]
    for key in ("tokens", "parents", "depths", "ranks", "draft_pos"):
        assert getattr(tree, key) == ref[key], key
    np.testing.assert_allclose(tree.scores, ref["scores"], rtol=1e-5, atol=1e-6)


def test_vocab_subset(tiny, base):
    target, draft = oracle_models(base, list(range(6)))
    vs = tiny["vocab_subset"]
    sub = O.top_vocab(np.arange(128)[::-1].copy(), 40, {127})
    assert sub.tolist() == vs["ids"]
    draft.set_vocab_subset(sub)
    res = O.speculative_generate(target, draft, TREES["tree"], vs["prompt"], 40, {-1})
    assert res["tokens"] == vs["tokens"]
    assert res["accepted_per_round"] == vs["accepted_per_round"]


def test_eos_stop(tiny, base):
    target, draft = oracle_models(base, list(range(6)))
    g = tiny["eos"]
    eos = set(g["eos"])
    assert O.autoregressive_generate(target, g["prompt"], 30, eos)["tokens"] == g["ar"]
    assert O.speculative_generate(target, draft, TREES["chain"], g["prompt"], 30, eos)["tokens"] == g["sd"]


def test_tree_mask_and_keep_positions(tiny, base):
    g = tiny["tree_mask"]
    br = make_bridges(64, [0, 2, 5], 6, 1, 0.125, 0.02)
    _, draft = oracle_models(base, [0, 2, 5], br)
    cache = draft.new_cache(32)
    draft.forward(g["prefix"], None, cache)
    n = len(g["tokens"])
    mask = np.zeros((n, n), dtype=bool)
    for i in range(n):
        j = i
        while j != -1:
            mask[i, j] = True
            j = g["parents"][j]
    pos = [6 + d for d in g["depth"]]
    logits = draft.forward(g["tokens"], pos, cache, tree_mask=mask)
    np.testing.assert_allclose(logits, np.array(g["logits"]), atol=1e-5, rtol=1e-4)
    cache.keep_positions(6, g["keep"])
    nxt = draft.forward([g["next_token"]], None, cache)[-1]
    np.testing.assert_allclose(nxt, np.array(g["next_logits"]), atol=1e-5, rtol=1e-4)


def test_sampling_stream_matches_reference(tiny):
    """Same seeds -> same torch random stream -> the oracle reproduces the
    reference's sampled tokens (allowing a rare flip from float rounding)."""
    g = tiny["sampling"]
    base8 = S.build_base_model("tiny_v8", 1, torch.float32, "cpu")
    with torch.no_grad():
        base8.lm_head.weight.mul_(8.0)
    assert S.weights_checksum(base8) == g["checksum"]
    br = make_bridges(64, [0, 5], 6, 2, 0.125, 0.05, BridgeConfig(init_std=0.05))
    target, draft = oracle_models(base8, [0, 5], br)
    for run in g["runs"]:
        same = 0
        for s, ref in enumerate(run["tokens"]):
            same += O.speculative_generate(target, draft, run["cfg"], [1, 5, 2], 3, set(), seed=s)["tokens"] == ref
        assert same >= 0.95 * len(run["tokens"])


def test_plan_bridges():
    assert O.plan_bridges([0, 2, 5], 6) == [("into_2", 1, 2), ("into_5", 3, 5)]
    assert [s[0] for s in O.plan_bridges([1, 2, 4], 6)] == ["into_1", "into_4", "into_norm"]


def test_c1_fixture_prompt_and_checksum_format():
    p = GOLD / "c1.json"
    if not p.exists():
        pytest.skip("c1 fixture not generated")
    g = json.loads(p.read_text())
    assert len(g["prompt"]) == 128 and len(g["ar"]) == 64
    assert g["prompt"] == S.make_prompt(0, 128, 128256)[0].tolist()
    assert g["sd"] == g["ar"], "the reference's own SD must equal its AR (greedy identity)"


def test_philox_known_answers():
    """The oracle's Philox4x32-10 against the published known-answer vectors
    of the Random123 distribution (philox4x32, 10 rounds)."""
    from oracle.philox import philox4x32_10

    out = philox4x32_10((0, 0, 0, 0), (0, 0))
    assert [int(x) for x in out] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    out = philox4x32_10((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF))
    assert [int(x) for x in out] == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    out = philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0))
    assert [int(x) for x in out] == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_gumbel_max_p_values_uniform_over_seed_blocks():
    """The device samplers' construction (Philox4x32-10 keyed by the seed,
    23-bit open uniform, Gumbel-max) restated by the oracle: over 60 blocks
    of 2000 consecutive seeds, the chi-square p-values of the drawn token
    against an 8-token distribution are uniform (KS p > 0.001), so a fixed
    seed block fails a p > 0.01 test only at the nominal rate."""
    import numpy as np
    from scipy import stats

    from oracle.philox import gumbel

    p = np.array([0.30, 0.22, 0.15, 0.12, 0.09, 0.06, 0.04, 0.02])
    lp = np.log(p)
    pvals = []
    for blk in range(60):
        seeds = range(blk * 2000, (blk + 1) * 2000)
        draws = [int(np.argmax(lp + gumbel(s, 0, 0, np.arange(8), 3))) for s in seeds]
        counts = np.bincount(draws, minlength=8)
        pvals.append(stats.chisquare(counts, p * counts.sum()).pvalue)
    assert stats.kstest(pvals, "uniform").pvalue > 1e-3


def test_top_k_warp_matches_reference_sample_next():
    """The oracle's top_k_warp is the distribution of the reference's batched
    sampler (ssd/data/generate_selfdistill.py:51-61: top-64 cut, temperature,
    top-p): every token the reference drew lies in the oracle's support, and
    the reference's counts fit the oracle's probabilities (pooled Pearson
    chi-square, p > 1e-3 on the fixed fixture); greedy rows give the argmax."""
    from scipy import stats

    from oracle.tree import top_k_warp

    gold = json.loads((GOLD / "sample_next.json").read_text())
    for case in gold["cases"]:
        row = np.asarray(case["logits"], dtype=np.float32)
        counts = np.asarray(case["counts"], dtype=np.float64)
        p = top_k_warp(row, gold["keep"], case["temperature"], case["top_p"])
        assert np.count_nonzero(p) <= gold["keep"]
        assert counts[p <= 0].sum() == 0, "the reference drew a token outside the oracle's support"
        exp = p * counts.sum()
        big = exp >= 5.0
        obs_l, exp_l = list(counts[big]), list(exp[big])
        small = (~big) & (p > 0)
        if small.any():
            obs_l.append(counts[small].sum())
            exp_l.append(exp[small].sum())
        assert stats.chisquare(obs_l, exp_l).pvalue > 1e-3, (case["temperature"], case["top_p"])
        assert int(np.argmax(row)) == case["greedy"]


def test_warp_probs_matches_reference_full_vocabulary():
    """The oracle's warp_probs (fp64) against the reference's (fp32) on
    seeded 128 256-logit rows: the 16 largest probabilities agree (ids exact,
    rtol 2e-4), and the kept-token counts agree except where a token's
    exclusive prefix mass lies within 2e-5 of top_p, where the reference's
    fp32 cumulative sum over the sorted row cannot decide (the oracle keeps
    the exact-arithmetic prefix)."""
    from oracle.tree import warp_probs

    gold = json.loads((GOLD / "warp_probs.json").read_text())
    for case in gold["cases"]:
        g = torch.Generator().manual_seed(case["seed"])
        row = (torch.randn(gold["vocab"], generator=g, dtype=torch.float64) * case["scale"]).float()
        assert abs(float(row.double().sum()) - case["row_sum"]) < 1e-6 * (1 + abs(case["row_sum"]))
        assert abs(float(row.double().square().sum()) - case["row_sq"]) < 1e-9 * case["row_sq"]
        row = row.numpy()
        T, top_p = case["temperature"], case["top_p"]
        p = warp_probs(row, T, top_p)
        m = min(16, case["n_kept"])  # zero-probability ids past the nucleus have no order
        order = np.argsort(-p, kind="stable")[:m]
        assert order.tolist() == case["top_ids"][:m]
        np.testing.assert_allclose(p[order], case["top_probs"][:m], rtol=2e-4)
        n = int(np.count_nonzero(p))
        if n != case["n_kept"]:
            z = row.astype(np.float64) / T
            sp = np.sort(np.exp(z - z.max()))[::-1]
            cum_before = np.cumsum(sp / sp.sum()) - sp / sp.sum()
            lo, hi = sorted((n, case["n_kept"]))
            assert np.all(np.abs(cum_before[lo:hi] - top_p) < 2e-5), (case, n)


def test_verify_inputs_and_greedy_verify_match_reference():
    """verify_inputs and greedy_verify against the reference's own outputs
    (ssd/engine/verify.py:32-57) on seeded random trees of 0-40 nodes with
    integer logits full of exact ties (the first maximum wins): the oracle's
    ids, positions, mask, accepted path and bonus, and the host
    verify_inputs of this package, equal the recorded ones exactly."""
    from oracle.tree import DraftTree as OTree
    from oracle.tree import greedy_verify, verify_inputs
    from ssd.engine import verify as V
    from ssd.engine.tree_drafter import DraftTree

    gold = json.loads((GOLD / "verify.json").read_text())
    for c in gold["cases"]:
        n = len(c["tokens"])
        fields = dict(tokens=c["tokens"], parents=c["parents"], depths=c["depths"], scores=[0.0] * n,
                      ranks=c["ranks"], draft_pos=[-1] * n)
        want_mask = np.zeros((n + 1, c["past"] + n + 1), dtype=bool)
        for i, cols in enumerate(c["mask_rows"]):
            want_mask[i, cols] = True
        ids, pos, mask = verify_inputs(OTree(**fields), c["root_token"], c["root_pos"], c["past"])
        assert (ids, pos) == (c["ids"], c["positions"])
        assert (mask == want_mask).all()
        ids, pos, mask = V.verify_inputs(DraftTree(**fields), c["root_token"], c["root_pos"], c["past"], "cpu")
        assert ids[0].tolist() == c["ids"] and pos[0].tolist() == c["positions"]
        assert (mask.numpy() == want_mask).all()
        acc, bonus = greedy_verify(OTree(**fields), np.asarray(c["logits"], dtype=np.float32))
        assert (acc, bonus) == (c["accepted"], c["bonus"])


def test_draft_tree_methods_match_reference():
    """DraftTree (ssd/engine/tree_drafter.py:48-95, the host type the API
    returns) and the oracle's restatement: children in sibling rank order,
    ancestors root-first, and subset's remapped arrays equal the reference's
    on the seeded random trees of verify.json."""
    from oracle.tree import DraftTree as OTree
    from ssd.engine.tree_drafter import DraftTree

    gold = json.loads((GOLD / "verify.json").read_text())
    for c in gold["cases"]:
        n = len(c["tokens"])
        fields = dict(tokens=c["tokens"], parents=c["parents"], depths=c["depths"], scores=[0.0] * n,
                      ranks=c["ranks"], draft_pos=[-1] * n)
        for tree in (DraftTree(**fields), OTree(**fields)):
            assert {str(k): v for k, v in tree.children().items()} == c["children"]
            assert [tree.ancestors(i) for i in range(n)] == c["ancestors"]
            sub = tree.subset(c["keep"])
            assert dict(tokens=sub.tokens, parents=sub.parents, depths=sub.depths, ranks=sub.ranks) == c["subset"]
