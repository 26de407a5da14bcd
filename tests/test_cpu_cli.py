"""The ssd-run command line (ssd/cli/run.py in the reference): its flags, the
tree overrides and the per-depth acceptance report, without a GPU."""

import pytest

from ssd.cli import run


def test_reference_flags_parse():
    a = run.parser().parse_args(["--config", "c.yaml", "--prompt", "hi", "--mode", "target", "--max-new-tokens", "7",
                                 "--raw", "--seed", "3", "--no-warmup", "--depth", "4", "--branch", "3,2,2,1",
                                 "--width", "8", "--max-nodes", "24", "--temperature", "0.7", "--top-p", "0.9",
                                 "--draft-vocab", "0", "--untrained"])
    assert (a.config, a.prompt, a.mode, a.max_new_tokens, a.raw, a.seed, a.no_warmup) == \
        ("c.yaml", "hi", "target", 7, True, 3, True)
    assert a.branch == [3, 2, 2, 1] and a.width == 8 and a.untrained
    ov = run.tree_overrides(a)
    assert ov == dict(depth=4, branch=[3, 2, 2, 1], width=8, max_nodes=24, temperature=0.7, top_p=0.9,
                      draft_vocab=None)


@pytest.mark.parametrize("argv", [["--config", "c.yaml"],  # no prompt
                                  ["--config", "c.yaml", "--prompt", "a", "--prompt-file", "f"],
                                  ["--config", "c.yaml", "--prompt", "a", "--bridges", "b.pt", "--untrained"],
                                  ["--config", "c.yaml", "--prompt", "a", "--mode", "other"]])
def test_bad_command_lines_exit(argv):
    with pytest.raises(SystemExit):
        run.parser().parse_args(argv)


def test_config_or_synthetic_required():
    with pytest.raises(SystemExit):
        run.main(["--prompt", "hello"])


def test_acceptance_by_depth_and_byte_ids():
    # rounds committing 1 (nothing accepted), 3 (two accepted), 4 (three accepted)
    rep = dict(run.acceptance_by_depth([1, 3, 4], 3))
    assert rep == {1: 2 / 3, 2: 1.0, 3: 0.5}
    ids = run.byte_ids("hé", 128)
    assert ids.shape == (1, 3) and int(ids.max()) < 128
