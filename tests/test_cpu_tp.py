"""Host-side tensor-parallel layout: the ranks' shards tile every global
matrix exactly once, shard configs keep the model width and vocabulary, and
random-stream ids are stable."""

import pytest

from ssd.engine import tp
from ssd import synthetic as S


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_tile_every_global_matrix(world):
    cfg = S.llama_config("llama3_70b", num_hidden_layers=2)
    shapes = tp.global_shapes(cfg)
    for name, shape in shapes.items():
        if len(shape) == 1:
            continue
        R, C = shape
        cover = {}
        for r in range(world):
            b = tp.shard_block(name, shape, r, world)
            assert (b.global_rows, b.global_cols) == (R, C)
            assert 0 <= b.row0 and b.row0 + b.rows <= R and 0 <= b.col0 and b.col0 + b.cols <= C
            cover[(b.row0, b.col0)] = (b.rows, b.cols)
        split = name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight", "gate_proj.weight",
                               "up_proj.weight", "lm_head.weight", "o_proj.weight", "down_proj.weight"))
        if split:  # disjoint blocks covering the matrix once
            assert len(cover) == world
            assert sum(r * c for r, c in cover.values()) == R * C
        else:  # replicated: every rank holds the whole matrix
            assert cover == {(0, 0): (R, C)}


def test_shard_config_of_70b():
    cfg = S.llama_config("llama3_70b")
    for world in (2, 4, 8):
        sc = tp.shard_config(cfg, world)
        assert sc.hidden_size == 8192 and sc.vocab_size == cfg.vocab_size and sc.head_dim == 128
        assert sc.num_attention_heads * world == 64 and sc.num_key_value_heads * world == 8
        assert sc.intermediate_size * world == 28672
    with pytest.raises(ValueError):
        tp.shard_config(cfg, 3)


def test_column_and_row_parallel_blocks():
    q = tp.shard_block("model.layers.0.self_attn.q_proj.weight", (8192, 8192), 3, 8)
    assert (q.row0, q.rows, q.col0, q.cols) == (3072, 1024, 0, 8192)
    o = tp.shard_block("model.layers.0.self_attn.o_proj.weight", (8192, 8192), 3, 8)
    assert (o.row0, o.rows, o.col0, o.cols) == (0, 8192, 3072, 1024)
    e = tp.shard_block("model.embed_tokens.weight", (128256, 8192), 5, 8)
    assert (e.row0, e.rows, e.col0, e.cols) == (0, 128256, 0, 8192)
    h = tp.shard_block("lm_head.weight", (128256, 8192), 7, 8)
    assert (h.row0, h.rows) == (7 * 16032, 16032)


def test_stream_ids_are_stable_and_distinct():
    a = tp.stream_id("model.layers.0.mlp.up_proj.weight")
    assert a == tp.stream_id("model.layers.0.mlp.up_proj.weight")
    assert a != tp.stream_id("model.layers.0.mlp.gate_proj.weight")
    assert 0 <= a < 2 ** 64


def test_allreduce_parity_alternates_and_checks_even_forwards():
    """Consecutive all-reduce calls alternate the two partial buffers; every
    forward restarts at parity 0 and must issue an even number of calls, so
    forwards (and CUDA graphs of forwards) concatenate without two
    consecutive calls on one buffer."""
    g = tp.TPGroup.__new__(tp.TPGroup)  # host bookkeeping only, no device region
    seq = []
    for n_layers in (3, 1, 2):
        g.begin()
        for _ in range(2 * n_layers):
            seq.append(g.next_parity())
        g.end()
    assert all(a != b for a, b in zip(seq, seq[1:]))
    g.begin()
    g.next_parity()
    with pytest.raises(RuntimeError):
        g.end()
