"""Write a bridge checkpoint with the REFERENCE's SubnetworkDraftModel.save_bridges
(ssd/models/subnetwork_draft.py:455-466), for the format test in
tests/test_cpu_checkpoints.py.

    python tests/golden/make_bridge_ckpt.py --ref PATH_TO_REFERENCE   (or set SSD_REFERENCE)

Base: this repo's seeded tiny Llama (synthetic.py, loaded by path so it does not
clash with the reference's `ssd` package). Draft layers [0, 3, 5] give the
bridges into_3 and into_5; they are filled by synthetic.init_bridges_ (seed 0,
in 0.02, out 1e-4), which the test repeats on this package's draft model.
Output: tests/golden/tiny_bridges.pt (CPU tensors, fp32).
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SYN_PATH = HERE.parent.parent / "subnetwork-speculative-decoding_b200" / "ssd" / "synthetic.py"
LAYERS = [0, 3, 5]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SSD_REFERENCE"), required="SSD_REFERENCE" not in os.environ,
                    help="path of the reference checkout (default: $SSD_REFERENCE)")
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location("ssd_synthetic", SYN_PATH)
    syn = importlib.util.module_from_spec(spec)
    sys.modules["ssd_synthetic"] = syn
    spec.loader.exec_module(syn)
    sys.path.insert(0, args.ref)
    from ssd.config import BridgeConfig
    from ssd.models.subnetwork_draft import SubnetworkDraftModel

    base = syn.build_base_model("tiny", 0)
    draft = SubnetworkDraftModel(base, LAYERS, BridgeConfig())
    syn.init_bridges_(draft.bridges, 0, in_std=0.02, out_std=1e-4)
    out = HERE / "tiny_bridges.pt"
    draft.save_bridges(str(out), stage=2, step=123)
    print(f"wrote {out} with bridges {sorted(draft.bridges.keys())}")


if __name__ == "__main__":
    main()
