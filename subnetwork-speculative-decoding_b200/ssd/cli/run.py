"""ssd-run: decode one prompt with the draft sub-network and the target
(command line of ssd/cli/run.py in the reference; same flags and report).

    python -m ssd.cli.run --config configs/llama32_1b_subnetwork.yaml --prompt "Explain KV caches."
    python -m ssd.cli.run --config ... --prompt-file test.txt --depth 6 --branch 4,2,2,1,1,1 --max-nodes 32
    python -m ssd.cli.run --config ... --prompt "..." --temperature 0.7 --seed 0
    python -m ssd.cli.run --synthetic c2 --prompt "any text" --max-new-tokens 64

Modes: `sd` (default) decodes speculatively with the draft sub-network and the
tree of `drafting:` (flags override it) and times it against target-only
decoding; `target` decodes with the target only. Bridges load from
{output_dir}/{profile}/ (online, stage2, stage1 in that order) unless --bridges
or --untrained is given.

--synthetic NAME (not in the reference) runs a seeded random-weight model of a
benchmark configuration instead of a checkpoint: there is no tokenizer then,
so the prompt's UTF-8 bytes (modulo the vocabulary) are the token ids and the
output is printed as ids.
"""

from __future__ import annotations

import argparse
import logging
from dataclasses import replace
from typing import Optional

import torch

from ssd.config import BridgeConfig, DraftingConfig, SSDConfig, profile_name
from ssd.engine.speculative import SpeculativeGenerator, TargetRunner, autoregressive_generate

log = logging.getLogger("ssd")


def encode_prompt(tokenizer, prompt: str, raw: bool) -> torch.Tensor:
    """[1, n] ids: the chat template around a user turn unless `raw` or the
    tokenizer has none."""
    if not raw and getattr(tokenizer, "chat_template", None):
        enc = tokenizer.apply_chat_template([{"role": "user", "content": prompt}], add_generation_prompt=True,
                                            return_tensors="pt", return_dict=True)
        return enc["input_ids"]
    return tokenizer(prompt, return_tensors="pt")["input_ids"]


def byte_ids(prompt: str, vocab: int) -> torch.Tensor:
    """Token ids of a prompt for a model without a tokenizer: its UTF-8 bytes."""
    data = prompt.encode("utf-8") or b" "
    return torch.tensor([[b % vocab for b in data]], dtype=torch.long)


def int_or_list(s: str):
    vals = [int(x) for x in s.split(",")]
    return vals[0] if len(vals) == 1 else vals


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="ssd-run", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", help="SSD YAML config (required unless --synthetic)")
    p.add_argument("--synthetic", help="seeded random-weight model of a benchmark configuration (c1, c2, c3, ...)")
    src = p.add_mutually_exclusive_group(required=True)
    src.add_argument("--prompt")
    src.add_argument("--prompt-file")
    p.add_argument("--mode", choices=["sd", "target"], default="sd")
    p.add_argument("--max-new-tokens", type=int, default=256)
    p.add_argument("--raw", action="store_true", help="don't wrap the prompt in the chat template")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-warmup", action="store_true")
    t = p.add_argument_group("tree overrides (default: the config's `drafting:`)")
    t.add_argument("--depth", type=int)
    t.add_argument("--branch", type=int_or_list, help="int or comma list per depth, e.g. 3,2,2,1")
    t.add_argument("--width", type=int_or_list)
    t.add_argument("--max-nodes", type=int)
    t.add_argument("--temperature", type=float)
    t.add_argument("--top-p", type=float)
    t.add_argument("--draft-vocab", type=int, help="draft scores the N most frequent tokens; 0 = full vocabulary")
    b = p.add_mutually_exclusive_group()
    b.add_argument("--bridges", help="explicit bridge checkpoint path")
    b.add_argument("--untrained", action="store_true", help="use freshly initialised bridges")
    return p


def tree_overrides(args) -> dict:
    keys = ("depth", "branch", "width", "max_nodes", "temperature", "top_p", "draft_vocab")
    out = {k: getattr(args, k) for k in keys if getattr(args, k) is not None}
    if out.get("draft_vocab") == 0:
        out["draft_vocab"] = None
    return out


def _load(args, prompt: str):
    """(base, draft or None, drafting config, ids [1, n], eos ids, decode(tokens) -> str, draft layers)."""
    from ssd import runtime

    if args.synthetic:
        from ssd import synthetic as S
        from ssd.data.token_freq import top_vocab
        from ssd.models import SubnetworkDraftModel

        if args.synthetic not in S.CONFIGS:
            raise SystemExit(f"ssd-run: unknown synthetic configuration {args.synthetic!r} "
                             f"(one of {', '.join(sorted(S.CONFIGS))})")
        base, spec = runtime.synthetic_base_model(args.synthetic)
        dcfg = replace(DraftingConfig(**spec.drafting, draft_vocab=spec.draft_vocab), **tree_overrides(args))
        draft = None
        if args.mode == "sd":
            draft = SubnetworkDraftModel(base, spec.draft_layers, BridgeConfig(hidden_dim=spec.bridge_hidden))
            if draft.bridges and not args.untrained:
                S.init_bridges_(draft.bridges, spec.seed, spec.bridge_in_std, spec.bridge_out_std)
            if args.bridges:
                draft.load_bridges(args.bridges)
            draft.bridges.to(base.model.embed_tokens.weight.dtype)
            if dcfg.draft_vocab:
                draft.set_vocab_subset(top_vocab(S.zipf_counts(base.config.vocab_size, spec.seed), dcfg.draft_vocab))
        ids = byte_ids(prompt, base.config.vocab_size)
        return base, draft, dcfg, ids, set(), lambda toks: " ".join(map(str, toks)), spec.draft_layers

    if not args.config:
        raise SystemExit("ssd-run: --config is required (or --synthetic NAME)")
    cfg = SSDConfig.from_yaml(args.config)
    cfg.drafting = replace(cfg.drafting, **tree_overrides(args))
    base = runtime.load_base_model(cfg)
    tokenizer = runtime.load_tokenizer(cfg)
    draft = None
    if args.mode == "sd":
        draft = runtime.build_draft(cfg, base, None if args.untrained else (args.bridges or "latest"),
                                    inference=True)
    ids = encode_prompt(tokenizer, prompt, args.raw)
    eos = getattr(base.generation_config, "eos_token_id", None)
    eos_ids = set(eos if isinstance(eos, list) else ([] if eos is None else [eos]))
    return (base, draft, cfg.drafting, ids, eos_ids, lambda toks: tokenizer.decode(toks, skip_special_tokens=True),
            cfg.draft_layers)


def acceptance_by_depth(accepted_per_round: list[int], depth: int) -> list[tuple[int, float]]:
    """Of the rounds that accepted every drafted token up to depth d - 1, the
    fraction that also accepted depth d (bonus token excluded)."""
    drafted = [n - 1 for n in accepted_per_round]
    out = []
    for d in range(1, depth + 1):
        reached = sum(a >= d - 1 for a in drafted)
        if reached:
            out.append((d, sum(a >= d for a in drafted) / reached))
    return out


def main(argv: Optional[list[str]] = None) -> None:
    args = parser().parse_args(argv)
    if not args.synthetic and not args.config:
        raise SystemExit("ssd-run: --config is required (or --synthetic NAME)")
    from ssd import runtime

    runtime.setup_env()
    prompt = args.prompt if args.prompt is not None else open(args.prompt_file).read()
    base, draft, dcfg, ids, eos_ids, decode, layers = _load(args, prompt)
    dcfg.validate()
    dev = runtime.input_device(base)
    ids = ids.to(dev)
    n_layers = base.config.num_hidden_layers
    target = TargetRunner(base)
    print(f"\nprompt: {ids.shape[1]} tokens | device: {dev} | draft layers {profile_name(layers)} "
          f"({len(layers)}/{n_layers})")
    print(f"tree: depth={dcfg.depth} branch={dcfg.branch} width={dcfg.width} max_nodes={dcfg.max_nodes} "
          f"temperature={dcfg.temperature} top_p={dcfg.top_p} draft_vocab={dcfg.draft_vocab or 'full'}")

    def run_ar(n: int):
        return autoregressive_generate(target, ids, n, eos_ids, dcfg.temperature, dcfg.top_p, args.seed)

    if not args.no_warmup:  # first calls capture the CUDA graphs
        run_ar(8)
        if args.mode == "sd":
            SpeculativeGenerator(base, draft, dcfg, target).generate(ids, 8, eos_ids, seed=args.seed)
    ar = run_ar(args.max_new_tokens)
    ar_tps = len(ar.tokens) / max(ar.decode_time, 1e-9)
    if args.mode == "target":
        print(f"\n=== target: {len(ar.tokens)} tokens, {ar_tps:.1f} tok/s ===")
        print(decode(ar.tokens))
        return

    sd = SpeculativeGenerator(base, draft, dcfg, target).generate(ids, args.max_new_tokens, eos_ids, seed=args.seed)
    sd_tps = len(sd.tokens) / max(sd.decode_time, 1e-9)
    rounds = len(sd.accepted_per_round)
    print(f"\n=== speculative: {len(sd.tokens)} tokens ===")
    print(decode(sd.tokens))
    print("\n--- stats (decode phase; prefill excluded) ---")
    print(f"rounds:                {rounds}")
    print(f"accepted tokens/round: {sd.mean_accepted:.2f}   (incl. bonus; max {dcfg.depth + 1})")
    print(f"mean tree size:        {sum(sd.tree_sizes) / max(1, rounds):.1f} nodes")
    by_depth = "  ".join(f"d{d}={r:.0%}" for d, r in acceptance_by_depth(sd.accepted_per_round, dcfg.depth))
    print(f"accept rate by depth:  {by_depth}   (given all shallower depths accepted)")
    per = {k: 1000 * v / max(1, rounds) for k, v in sd.times.items() if k != "prefill"}
    print("per round:             " + "  ".join(f"{k}={v:.1f}ms" for k, v in per.items()))
    print(f"target step (AR):      {1000 * ar.decode_time / max(1, len(ar.tokens) - 1):.1f}ms/token")
    print(f"throughput:            AR {ar_tps:.1f} tok/s  |  SD {sd_tps:.1f} tok/s  |  speedup {sd_tps / ar_tps:.2f}x")
    if dcfg.temperature == 0:
        n = min(len(ar.tokens), len(sd.tokens))
        same = ar.tokens[:n] == sd.tokens[:n]
        print(f"greedy output identical to AR: {same}" +
              ("" if same else "  (bf16 rounding of batched rows can flip near-ties)"))


if __name__ == "__main__":
    main()
