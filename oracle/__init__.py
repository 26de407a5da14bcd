"""CPU oracle for the SSD speculative-decoding round -- TEST INFRASTRUCTURE.

This package restates, in numpy (model math) and plain Python (tree logic),
the reference's hot path: the sub-network draft / target forward over one
shared KV cache, the level-by-level tree drafter, greedy and sampling
verification, and KV compaction. Each function cites the reference file:line
it follows (paths inside yotamabramson/subnetwork-speculative-decoding).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this package, and only as the checker (or the timed CPU baseline) --
never as the thing measured or shipped. The product path (the `ssd` package)
never imports it.

Pinning: tests/golden/ holds fixtures produced by running the reference
itself (tests/golden/make_golden.py); tests/test_oracle_golden.py checks this
oracle against them.
"""

from oracle.model import OracleKVCache, OracleModel, weights_from_hf  # noqa: F401
from oracle.tree import (  # noqa: F401
    ROOT,
    DraftTree,
    OracleTreeDrafter,
    greedy_verify,
    plan_bridges,
    sample_verify,
    top_vocab,
    verify_inputs,
    warp_probs,
)
from oracle.engine import autoregressive_generate, speculative_generate  # noqa: F401
