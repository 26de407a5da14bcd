"""End-to-end parity of the B200 round (through the C ABI) against the
reference's recorded outputs and the CPU oracle.

fp32 tier: token ids must equal the reference's exactly (tiny model, and
BASELINE config 1 at full Llama-3.2-1B size). bf16 tier (BASELINE config 2
model at full Llama-3.2-1B size, tests/golden/c2ref.json: the reference's
fp32 greedy decode of the bf16-rounded weights): our bf16 target-only and
speculative decodes are pinned against the reference's fp32 decode and the
reference's own bf16 run (see the note at the bf16 tier below). On the tiny
model the bf16 speculative output also equals our own target-only decode.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from ssd import synthetic as S
from ssd.config import BridgeConfig, DraftingConfig
from ssd.engine.speculative import SpeculativeGenerator, TargetRunner, autoregressive_generate
from ssd.engine.tree_drafter import TreeDrafter
from ssd.models import SubnetworkDraftModel

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"
DEV = torch.device("cuda:0")

TREES = {
    "chain": dict(depth=4, branch=1),
    "tree": dict(depth=3, branch=[3, 2, 2]),
    "pruned": dict(depth=5, branch=[4, 3, 2, 2, 1], width=[4, 6, 6, 4, 4], max_nodes=12),
    "deep_chain": dict(depth=8, branch=1),
}


@pytest.fixture(scope="module")
def tiny():
    return json.loads((GOLD / "tiny.json").read_text())


def tiny_base(dtype=torch.float32):
    base = S.build_base_model("tiny", 0, torch.float32, "cpu")
    return base.to(dtype).to(DEV)


@pytest.fixture(scope="module")
def base32(tiny):
    b = S.build_base_model("tiny", 0, torch.float32, "cpu")
    assert S.weights_checksum(b) == tiny["checksum"]
    return b.to(DEV)


def make_draft(base, layers, seed, in_std, out_std, cfg=None):
    d = SubnetworkDraftModel(base, layers, cfg or BridgeConfig())
    if d.bridges:
        S.init_bridges_(d.bridges, seed, in_std=in_std, out_std=out_std)
        d.bridges.to(base.model.embed_tokens.weight.dtype)
    return d


def test_forward_logits_fp32(tiny, base32):
    target = TargetRunner(base32)
    ids = torch.tensor([tiny["forward"]["ids"]], device=DEV)
    logits = target(ids).logits[0].cpu()
    np.testing.assert_allclose(logits.numpy(), np.array(tiny["forward"]["logits"]), atol=2e-5, rtol=1e-4)


def test_autoregressive_fp32_matches_reference(tiny, base32):
    target = TargetRunner(base32)
    for p, ref in zip(tiny["prompts"], tiny["ar"]):
        res = autoregressive_generate(target, torch.tensor([p]), 40, {-1})
        assert res.tokens == ref


@pytest.mark.parametrize("draft_kind", ["untrained", "perfect"])
@pytest.mark.parametrize("tree_name", list(TREES))
def test_speculative_fp32_matches_reference(tiny, base32, draft_kind, tree_name):
    layers = [0, 3, 5] if draft_kind == "untrained" else list(range(6))
    draft = make_draft(base32, layers, 0, 0.125, 0.02, BridgeConfig(init_std=0.02))
    target = TargetRunner(base32)
    gold = tiny["sd"][f"{draft_kind}/{tree_name}"]
    gen = SpeculativeGenerator(base32, draft, DraftingConfig(**TREES[tree_name]), target)
    for p, run in zip(tiny["prompts"], gold["runs"]):
        res = gen.generate(torch.tensor([p]), 40, {-1})
        assert res.tokens == run["tokens"]
        assert res.accepted_per_round == run["accepted_per_round"]
        assert res.tree_sizes == run["tree_sizes"]


@pytest.mark.parametrize("tree_name", list(TREES))
def test_tree_build_fp32_matches_reference(tiny, base32, tree_name):
    """Device tree (top-k head, level prune, max_nodes prune) == reference tree."""
    draft = make_draft(base32, [0, 3, 5], 0, 0.125, 0.02, BridgeConfig(init_std=0.02))
    target = TargetRunner(base32)
    ft = tiny["sd"][f"untrained/{tree_name}"]["first_tree"]
    cache = target.new_cache(64)
    out = target(torch.tensor([tiny["prompts"][0]], device=DEV), past_key_values=cache, logits_to_keep=1)
    assert int(out.logits[0, -1].argmax()) == ft["root"]
    drafter = TreeDrafter(draft, DraftingConfig(**TREES[tree_name]))
    tree = drafter.build(cache, torch.tensor([[ft["root"]]]), ft["committed"])
    ref = ft["tree"]
    for key in ("tokens", "parents", "depths", "ranks", "draft_pos"):
        assert getattr(tree, key) == ref[key], key
    np.testing.assert_allclose(tree.scores, ref["scores"], rtol=1e-5, atol=1e-5)
    assert cache.get_seq_length() == ft["committed"] + 1 + drafter.max_tree_cache()


def test_tree_mask_and_keep_positions_fp32(tiny, base32):
    g = tiny["tree_mask"]
    draft = make_draft(base32, [0, 2, 5], 1, 0.125, 0.02)
    cache = draft.new_cache(32)
    draft(torch.tensor([g["prefix"]], device=DEV), past_key_values=cache)
    n = len(g["tokens"])
    mask = torch.zeros(n, n, dtype=torch.bool)
    for i in range(n):
        j = i
        while j != -1:
            mask[i, j] = True
            j = g["parents"][j]
    pos = torch.tensor([[6 + d for d in g["depth"]]])
    logits = draft(torch.tensor([g["tokens"]], device=DEV), position_ids=pos, past_key_values=cache,
                   tree_attention_mask=mask).logits[0].cpu()
    np.testing.assert_allclose(logits.numpy(), np.array(g["logits"]), atol=2e-5, rtol=1e-4)
    cache.keep_positions(6, torch.tensor(g["keep"]))
    nxt = draft(torch.tensor([[g["next_token"]]], device=DEV), past_key_values=cache).logits[0, -1].cpu()
    np.testing.assert_allclose(nxt.numpy(), np.array(g["next_logits"]), atol=2e-5, rtol=1e-4)


def test_vocab_subset_and_eos_fp32(tiny, base32):
    from ssd.data.token_freq import top_vocab

    target = TargetRunner(base32)
    vs = tiny["vocab_subset"]
    draft = SubnetworkDraftModel(base32, list(range(6)))
    sub = top_vocab(torch.arange(128).flip(0), 40, always={127})
    assert sub.tolist() == vs["ids"]
    draft.set_vocab_subset(sub)
    res = SpeculativeGenerator(base32, draft, DraftingConfig(**TREES["tree"]), target).generate(
        torch.tensor([vs["prompt"]]), 40, {-1})
    assert res.tokens == vs["tokens"] and res.accepted_per_round == vs["accepted_per_round"]
    out = draft(torch.tensor([vs["prompt"]], device=DEV))
    assert out.logits.shape[-1] == 40 and out.vocab_ids is draft.vocab_ids
    g = tiny["eos"]
    eos = set(g["eos"])
    assert autoregressive_generate(target, torch.tensor([g["prompt"]]), 30, eos).tokens == g["ar"]
    draft = SubnetworkDraftModel(base32, list(range(6)))
    sd = SpeculativeGenerator(base32, draft, DraftingConfig(**TREES["chain"]), target).generate(
        torch.tensor([g["prompt"]]), 30, eos)
    assert sd.tokens == g["sd"] and sd.tokens[-1] in eos


def test_identity_bridges_equal_layer_skipping(base32):
    """Zero-init bridges == the selected layers back to back
    (reference tests/test_forward_pass.py:119-130)."""
    import oracle as O
    from oracle.model import weights_from_hf

    draft = SubnetworkDraftModel(base32, [0, 3, 5], BridgeConfig(init_std=0.0))
    ids = torch.randint(0, 128, (1, 9), generator=torch.Generator().manual_seed(3))
    ours = draft(ids.to(DEV)).logits[0].cpu().numpy()
    w, conf = weights_from_hf(base32)
    skip = O.OracleModel(w, conf, [0, 3, 5], {n: None for n in draft.bridges})
    skip.pre_layer_bridge, skip.pre_norm_bridge = [None] * 3, None  # plain layer skipping
    ref = skip.forward(ids[0].tolist())
    np.testing.assert_allclose(ours, ref, atol=2e-5, rtol=1e-4)


def test_batched_forward_shapes(base32):
    draft = SubnetworkDraftModel(base32, [0, 2, 5])
    S.init_bridges_(draft.bridges, 4, in_std=0.125, out_std=0.02)
    draft.bridges.to(DEV)
    ids = torch.randint(0, 128, (2, 11), generator=torch.Generator().manual_seed(0)).to(DEV)
    out = draft(ids, output_bridge_states=True)
    assert out.logits.shape == (2, 11, 128) and out.hidden_states.shape == (2, 11, 64)
    assert set(out.bridge_states) == {"into_2", "into_5"}
    assert torch.isfinite(out.logits).all()
    assert draft(ids, logits_to_keep=3).logits.shape == (2, 3, 128)
    assert draft(ids, compute_logits=False).logits is None


@pytest.mark.parametrize("tree_name", list(TREES))
def test_bf16_speculative_equals_target_only(tree_name):
    """bf16 tier on the tiny model: greedy SD output == our target-only decode."""
    base = tiny_base(torch.bfloat16)
    target = TargetRunner(base)
    draft = make_draft(base, [0, 3, 5], 0, 0.125, 0.02, BridgeConfig(init_std=0.02))
    for s in range(3):
        p = S.make_prompt(s, 5 + 4 * s, 128)
        ar = autoregressive_generate(target, p, 40, {-1})
        sd = SpeculativeGenerator(base, draft, DraftingConfig(**TREES[tree_name]), target).generate(p, 40, {-1})
        assert sd.tokens == ar.tokens
        assert sum(sd.accepted_per_round) >= 39
        # the reference's per-phase totals (speculative.py:149-171)
        assert set(sd.times) == {"prefill", "draft", "verify", "bookkeeping"}
        assert all(v >= 0 for v in sd.times.values()) and sd.times["verify"] > 0
        assert set(ar.times) == {"prefill", "decode"}


def test_prefill_buffers_reused_across_prompt_lengths():
    """One engine prefills prompts of 300 rows (three GEMM token tiles), 40 rows
    and 300 rows again, reusing its prefill inputs, activations and workspace;
    after each, its state (first token, sequence length) equals a fresh
    engine's for the same prompt (bf16 tiny model)."""
    from ssd.engine.round import TargetStep, cache_capacity

    base = tiny_base(torch.bfloat16)
    target = TargetRunner(base)
    long_p, short_p = S.make_prompt(7, 300, 128), S.make_prompt(8, 40, 128)

    def fresh(p):
        e = TargetStep(target, target.new_cache(cache_capacity(p.numel(), 8)), 8)
        e.prefill(p.to(DEV))
        return e

    ref = {300: fresh(long_p), 40: fresh(short_p)}
    eng = TargetStep(target, target.new_cache(cache_capacity(300, 8)), 8)
    for p in (long_p, short_p, long_p):
        eng.prefill(p.to(DEV))
        torch.cuda.synchronize()
        want = ref[p.numel()]
        assert torch.equal(eng.state, want.state)
        assert torch.equal(eng.out_tokens[:1], want.out_tokens[:1])


@pytest.mark.slow
def test_c1_full_size_fp32_matches_reference():
    """BASELINE config 1 at full size: SD output == the reference's own
    target-only greedy decode (bit-exact ids), fp32."""
    g = json.loads((GOLD / "c1.json").read_text())
    spec = S.CONFIGS["c1"]
    base = S.build_base_model(spec.model, spec.seed, torch.float32, "cpu")
    assert S.weights_checksum(base) == g["checksum"]
    base = base.to(DEV)
    target = TargetRunner(base)
    draft = SubnetworkDraftModel(base, spec.draft_layers, BridgeConfig(hidden_dim=spec.bridge_hidden))
    S.init_bridges_(draft.bridges, spec.seed, spec.bridge_in_std, spec.bridge_out_std)
    draft.bridges.to(DEV)
    ids = torch.tensor([g["prompt"]])
    ar = autoregressive_generate(target, ids, spec.max_new_tokens, set())
    assert ar.tokens == g["ar"]
    sd = SpeculativeGenerator(base, draft, DraftingConfig(**spec.drafting), target).generate(
        ids, spec.max_new_tokens, set())
    assert sd.tokens == g["ar"]
    assert sd.accepted_per_round == g["accepted_per_round"]


def test_generate_batch_greedy_matches_reference(tiny, base32):
    """generate_batch (ssd/data/generate_selfdistill.py:64-108): each row's greedy
    continuation equals the reference's recorded decode of that prompt; rows of
    different lengths; EOS cuts a row after the first EOS."""
    from ssd.data.generate_selfdistill import generate_batch

    target = TargetRunner(base32)
    prompts = [list(p) for p in tiny["prompts"]]
    rows = generate_batch(target, prompts, 40, {-1}, 0.0, 1.0, pad_id=0)
    assert rows == [ref[:40] for ref in tiny["ar"]]
    eos = tiny["ar"][0][5]
    cut = generate_batch(target, prompts[:1], 40, {eos}, 0.0, 1.0, pad_id=0)[0]
    assert cut == tiny["ar"][0][: tiny["ar"][0].index(eos) + 1]
    assert generate_batch(target, [], 8, set(), 0.0, 1.0, pad_id=0) == []


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_batched_decoder_matches_single_sequence_decodes(dtype):
    """One forward per step over several sequences, each in its own cache
    slot range: every row decodes as the sequence alone does, up to a
    near-tie of the single-sequence decode's top-2 gap (fp32: < 1e-4, where
    only the attention's split layout differs; bf16: < 2e-2), with prompts of
    different lengths."""
    from ssd.engine.batch import BatchDecoder
    from ssd.engine.round import TargetStep, cache_capacity

    base = S.build_base_model("llama32_1b", 7, dtype, DEV, gen_device="cuda", num_hidden_layers=2, vocab_size=4096)
    target = TargetRunner(base)
    prompts = [S.make_prompt(30 + b, n, 4096)[0].tolist() for b, n in enumerate([5, 40, 17, 130, 64, 9])]
    n_new = 24
    dec = BatchDecoder(target, len(prompts), 256, sum(map(len, prompts)))
    rows = dec.generate(prompts, n_new, set())
    for p, row in zip(prompts, rows):
        eng = TargetStep(target, target.new_cache(cache_capacity(len(p), n_new)), n_new)
        eng.prefill(torch.tensor([p], device=DEV))
        gaps = [float(eng.gap[0])]
        for _ in range(n_new - 1):
            eng.run(1)
            gaps.append(float(eng.gap[0]))
        single = eng.tokens()
        i = next((j for j, (a, b) in enumerate(zip(row, single)) if a != b), None)
        tie = 1e-4 if dtype == torch.float32 else 2e-2
        assert i is None or gaps[i] < tie, (i, gaps[i] if i is not None else None)


def test_ssd_run_command_line_on_a_synthetic_model(capsys):
    """ssd-run end to end (--synthetic tiny: seeded fp32 random weights, no
    checkpoint or tokenizer): greedy speculative output equals the target-only
    output and the acceptance report is printed."""
    from ssd.cli import run

    run.main(["--synthetic", "tiny", "--prompt", "hello world", "--max-new-tokens", "12", "--no-warmup"])
    out = capsys.readouterr().out
    assert "=== speculative: 12 tokens ===" in out
    assert "greedy output identical to AR: True" in out
    assert "accept rate by depth:" in out
    run.main(["--synthetic", "tiny", "--prompt", "hello world", "--max-new-tokens", "5", "--mode", "target",
              "--no-warmup"])
    assert "=== target: 5 tokens" in capsys.readouterr().out


# ---------------------------------------------------------------- bf16 tier
# The bf16 tier is pinned against the reference itself. tests/golden/c2ref.json
# holds the reference's fp32 decode of the config-2 model with bf16-rounded
# weights (the exact answer for those weights) and the reference's OWN bf16
# run of the same model (its modules in torch.bfloat16). The reference's bf16
# arithmetic lands up to ~0.35 away from its fp32 logits on this model and
# flips the greedy choice at steps whose fp32 top-2 gap is as large as ~0.1,
# so a fixed 1e-2 near-tie threshold cannot be met by any bf16 implementation,
# the reference's included. The B200 bf16 path must be about as close to the
# fp32 answer as the reference's own bf16 path, and may only differ from the
# fp32 greedy choice at steps inside that bf16 noise band.


def _first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None


@pytest.fixture(scope="module")
def c2():
    """The config-2 model (seed 1, planted) with its weights rounded to bf16,
    exactly as the reference decoded it for tests/golden/c2ref.json."""
    g = json.loads((GOLD / "c2ref.json").read_text())
    spec = S.CONFIGS["c2"]
    base = S.build_base_model(spec.model, spec.seed, torch.float32, "cpu", plant_layers=spec.draft_layers,
                              plant_scale=spec.plant_scale)
    with torch.no_grad():
        for p in base.parameters():
            p.copy_(p.bfloat16().float())
    assert S.weights_checksum(base) == g["checksum"], "host RNG differs from the fixture's"
    base = base.to(torch.bfloat16).to(DEV)
    return g, spec, base


def _ref_bf16_errors(g):
    """Per step: max |reference bf16 - reference fp32| over the top-8 and probe ids."""
    b = g["bf16"]
    return [float(np.max(np.abs(np.array(b["tf_top_values"][i] + b["tf_probe_logits"][i]) -
                                np.array(g["top_values"][i] + g["probe_logits"][i]))))
            for i in range(len(g["ar"]))]


def _noise_band(g) -> float:
    """fp32 top-2 gaps below this lie inside bf16 noise: twice the reference's
    own largest bf16 logit error on this run."""
    return 2.0 * max(_ref_bf16_errors(g))


@pytest.mark.slow
def test_c2_bf16_logits_as_close_as_reference_bf16(c2):
    """Teacher-forced on the reference's fp32 tokens (prefill, then one cached
    decode step per token through SubnetworkDraftModel.forward): at every step
    our bf16 logits at the reference's top-8 ids and 64 fixed probe ids are
    compared with the reference's fp32 logits. Our worst and mean errors must
    stay within 10 % of the reference's own bf16 run's (on this model both
    land at ~0.33 worst / ~0.24 mean: the error is that of bf16 arithmetic, not
    of either implementation), our argmax must agree with the fp32 argmax
    about as often as the reference's bf16 argmax does (at most 2 of 48 steps
    fewer), and wherever the fp32 gap is outside the bf16 noise band it must
    agree."""
    g, spec, base = c2
    target = TargetRunner(base)
    n = len(g["ar"])
    cache = target.new_cache(len(g["prompt"]) + n + 1)
    rows = [target(torch.tensor([g["prompt"]], device=DEV), past_key_values=cache, logits_to_keep=1).logits[0, -1]]
    for t in g["ar"][:-1]:
        rows.append(target(torch.tensor([[t]], device=DEV), past_key_values=cache).logits[0, -1])
    ours, agree = [], 0
    band = _noise_band(g)
    for i, row in enumerate(rows):
        row = row.float().cpu().numpy()
        ids = np.array(g["top_ids"][i] + g["probe_ids"])
        ref = np.array(g["top_values"][i] + g["probe_logits"][i])
        ours.append(float(np.max(np.abs(row[ids] - ref))))
        hit = int(np.argmax(row)) == g["top_ids"][i][0]
        agree += hit
        assert hit or g["gaps"][i] < band, f"step {i}: argmax differs at fp32 gap {g['gaps'][i]:.3f}"
    theirs = _ref_bf16_errors(g)
    ref_agree = sum(int(a == t[0]) for a, t in zip(g["bf16"]["tf_argmax"], g["top_ids"]))
    print(f"c2 bf16 |logit error| ours max {max(ours):.3f} mean {np.mean(ours):.3f}; reference bf16 max "
          f"{max(theirs):.3f} mean {np.mean(theirs):.3f}; argmax agreement ours {agree}/{n}, reference bf16 "
          f"{ref_agree}/{n}")
    assert max(ours) <= 1.1 * max(theirs) and np.mean(ours) <= 1.1 * np.mean(theirs)
    assert agree >= ref_agree - 2


@pytest.mark.slow
def test_c2_bf16_decodes_match_reference(c2):
    """Product path in bf16 (folded norms, CUDA-graph engines) at the C2
    shape. Target-only greedy ids follow the reference's fp32 ids until a step
    whose fp32 gap lies inside the bf16 noise band, and at least as long as
    the reference's own bf16 decode does; each step's top logit (the fused
    lm_head + argmax's max) is as close to the reference's fp32 top logit as
    the reference's bf16 error bound, while the decodes agree. Speculative
    decoding (C2 draft: 3 layers + 2 bridges, 32k-vocabulary head) reproduces
    our target-only ids up to a step whose own top-2 gap lies inside the band."""
    from ssd.data.token_freq import top_vocab
    from ssd.engine.round import TargetStep, cache_capacity

    g, spec, base = c2
    band = _noise_band(g)
    target = TargetRunner(base)
    prompt = torch.tensor([g["prompt"]])
    n = len(g["ar"])
    ar = autoregressive_generate(target, prompt, n, set())
    i = _first_divergence(ar.tokens, g["ar"])
    j = _first_divergence(g["bf16"]["ar"], g["ar"])
    assert i is None or (g["gaps"][i] < band and (j is None or i >= j)), (i, j)
    # per-step top logit and gap of the engine's fused head
    eng = TargetStep(target, target.new_cache(cache_capacity(prompt.shape[1], n)), n)
    eng.prefill(prompt.to(DEV))
    tops, gaps = [float(eng.amax[0])], [float(eng.gap[0])]
    for _ in range(n - 1):
        eng.run(1)
        tops.append(float(eng.amax[0]))
        gaps.append(float(eng.gap[0]))
    assert eng.tokens() == ar.tokens
    upto = n if i is None else i
    top_err = np.abs(np.array(tops[:upto]) - np.array([v[0] for v in g["top_values"]][:upto]))
    assert top_err.max() <= max(_ref_bf16_errors(g)[:upto])
    # speculative decoding with the C2 draft
    draft = SubnetworkDraftModel(base, spec.draft_layers, BridgeConfig(hidden_dim=spec.bridge_hidden))
    S.init_bridges_(draft.bridges, spec.seed, spec.bridge_in_std, spec.bridge_out_std)
    draft.bridges.to(torch.bfloat16).to(DEV)
    draft.set_vocab_subset(top_vocab(S.zipf_counts(base.config.vocab_size, spec.seed), spec.draft_vocab))
    sd = SpeculativeGenerator(base, draft, DraftingConfig(**spec.drafting), target).generate(prompt, n, set())
    k = _first_divergence(sd.tokens, ar.tokens)
    assert k is None or gaps[k] < band, (k, gaps[k] if k is not None else None)
    assert sd.mean_accepted > 1.0
