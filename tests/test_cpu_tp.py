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


# ------------------------------------------------------------ two gloo ranks
def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rms(x, w, eps):
    import torch

    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w


def _sharded_logits(base, rank: int, world: int, ids):
    """Forward of this rank's shard in plain torch: column-parallel q/k/v and
    gate/up, row-parallel o_proj and down (partials summed over the ranks
    before each residual add), vocabulary-parallel lm_head. Returns the
    rank's logit columns [T, V / world]."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    cfg = base.config
    shapes = tp.global_shapes(cfg)
    params = dict(base.named_parameters())
    sc = tp.shard_config(cfg, world)
    H, Hkv, hd, eps = sc.num_attention_heads, sc.num_key_value_heads, sc.head_dim, cfg.rms_norm_eps

    def part(name):
        w = params[name].detach()
        b = tp.shard_block(name, shapes[name], rank, world)
        return w if w.dim() == 1 else w[b.row0:b.row0 + b.rows, b.col0:b.col0 + b.cols]

    def rope(t, cos, sin):
        half = t.shape[-1] // 2
        rot = torch.cat([-t[..., half:], t[..., :half]], -1)
        return t * cos[:, None] + rot * sin[:, None]

    T = ids.numel()
    x = params["model.embed_tokens.weight"].detach()[ids]
    cos, sin = (c[0] for c in base.model.rotary_emb(x[None], torch.arange(T)[None]))
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        xn = _rms(x, part(p + "input_layernorm.weight"), eps)
        q = rope((xn @ part(p + "self_attn.q_proj.weight").T).view(T, H, hd), cos, sin)
        k = rope((xn @ part(p + "self_attn.k_proj.weight").T).view(T, Hkv, hd), cos, sin)
        v = (xn @ part(p + "self_attn.v_proj.weight").T).view(T, Hkv, hd)
        k, v = (t.repeat_interleave(H // Hkv, dim=1) for t in (k, v))
        a = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), is_causal=True)
        o = a.transpose(0, 1).reshape(T, H * hd) @ part(p + "self_attn.o_proj.weight").T
        dist.all_reduce(o)
        x = x + o
        xn = _rms(x, part(p + "post_attention_layernorm.weight"), eps)
        m = (F.silu(xn @ part(p + "mlp.gate_proj.weight").T) * (xn @ part(p + "mlp.up_proj.weight").T))
        m = m @ part(p + "mlp.down_proj.weight").T
        dist.all_reduce(m)
        x = x + m
    return _rms(x, part("model.norm.weight"), eps) @ part("lm_head.weight").T


def _tp_worker(rank: int, world: int, port: int, q) -> None:
    import os

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        base = S.build_base_model("tiny", 0, torch.float32, "cpu")
        ids = S.make_prompt(21, 12, base.config.vocab_size)[0]
        with torch.no_grad():
            local = _sharded_logits(base, rank, world, ids)
        q.put((rank, local.numpy()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_sharded_forward_equals_full_model():
    """The tensor-parallel layout on two gloo ranks: each rank holds the blocks
    shard_block gives it and the head counts of shard_config; summing the
    row-parallel partials and concatenating the vocabulary shards (rank r owns
    ids [r V/2, (r+1) V/2)) gives the unsharded model's logits, so the merged
    argmax is the full model's."""
    import numpy as np
    import torch
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    base = S.build_base_model("tiny", 0, torch.float32, "cpu")
    ids = S.make_prompt(21, 12, base.config.vocab_size)
    with torch.no_grad():
        full = base(ids).logits[0].numpy()
    merged = np.concatenate([got[r] for r in range(world)], axis=-1)
    np.testing.assert_allclose(merged, full, rtol=1e-4, atol=1e-5)
    assert (merged.argmax(-1) == full.argmax(-1)).all()
