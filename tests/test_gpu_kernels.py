"""Kernel-level parity: each sm_100a kernel (through the C ABI) against a plain
PyTorch fp32 reference of the same op, on seeded inputs.

Tolerances: bf16 tensor-core GEMMs accumulate in fp32 over bf16 operands, so
they are compared with the fp32 product of the same bf16 values (rtol 1e-2 on
bf16-rounded outputs, 1e-4 relative on fp32 outputs); the fp32 CUDA-core tier
is compared at 1e-5 relative.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from ssd import ops as O

    return O


@pytest.fixture(scope="module")
def ws(ops):
    return ops.Workspace(torch.device(DEV), max_rows=512, vocab=128256)


def _rand(*shape, dtype=torch.bfloat16, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(dtype)


def _close(a, b, rtol, atol_frac):
    a, b = a.float(), b.float()
    atol = atol_frac * b.abs().max().item() + 1e-12
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol)


GEMM_SHAPES = [(1, 128, 64), (5, 256, 192), (33, 4096, 4096), (16, 1000, 512), (300, 384, 256), (64, 2048, 8192),
               (1, 14336, 4096)]


@pytest.mark.parametrize("T,N,K", GEMM_SHAPES)
def test_linear_store_bf16(ops, ws, T, N, K):
    x = _rand(T, K, seed=1)
    w = _rand(N, K, scale=0.02, seed=2)
    out = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    ops.linear(x, [w], ws, out=out)
    ref = x.float() @ w.float().T
    torch.cuda.synchronize()
    ws.check_status()
    _close(out, ref, rtol=1e-2, atol_frac=1e-2)


@pytest.mark.parametrize("T,N,K", [(1, 128, 64), (7, 512, 320), (33, 2048, 2048), (40, 300, 96)])
def test_linear_store_f32(ops, ws, T, N, K):
    x = _rand(T, K, dtype=torch.float32, seed=3)
    w = _rand(N, K, dtype=torch.float32, scale=0.02, seed=4)
    out = torch.empty(T, N, dtype=torch.float32, device=DEV)
    ops.linear(x, [w], ws, out=out)
    ref = (x.double() @ w.double().T).float()
    torch.cuda.synchronize()
    _close(out, ref, rtol=1e-5, atol_frac=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("act", ["none", "silu", "gelu", "relu"])
def test_linear_bias_act(ops, ws, dtype, act):
    T, N, K = 9, 512, 256
    x = _rand(T, K, dtype=dtype, seed=5)
    w = _rand(N, K, dtype=dtype, scale=0.05, seed=6)
    b = _rand(N, dtype=dtype, scale=0.1, seed=7)
    out = torch.empty(T, N, dtype=dtype, device=DEV)
    ops.linear(x, [w], ws, biases=[b], act=act, out=out)
    ref = x.float() @ w.float().T + b.float()
    ref = {"none": ref, "silu": torch.nn.functional.silu(ref), "gelu": torch.nn.functional.gelu(ref),
           "relu": torch.relu(ref)}[act]
    torch.cuda.synchronize()
    _close(out, ref, rtol=1e-2 if dtype == torch.bfloat16 else 1e-5, atol_frac=1e-2 if dtype == torch.bfloat16 else 1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T,N,K", [(1, 4096, 4096), (33, 2048, 8192), (6, 64, 128), (300, 512, 256)])
def test_linear_residual(ops, ws, dtype, T, N, K):
    x = _rand(T, K, dtype=dtype, seed=8)
    w = _rand(N, K, dtype=dtype, scale=0.02, seed=9)
    resid = _rand(T, N, dtype=torch.float32, seed=10)
    ref = resid + x.float() @ w.float().T
    ops.linear(x, [w], ws, epilogue=1, resid=resid)
    torch.cuda.synchronize()
    _close(resid, ref, rtol=1e-4, atol_frac=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T,F,K", [(1, 14336, 4096), (17, 128, 64), (33, 8192, 2048), (300, 256, 128)])
def test_swiglu(ops, ws, dtype, T, F, K):
    x = _rand(T, K, dtype=dtype, seed=11)
    wg = _rand(F, K, dtype=dtype, scale=0.02, seed=12)
    wu = _rand(F, K, dtype=dtype, scale=0.02, seed=13)
    out = torch.empty(T, F, dtype=dtype, device=DEV)
    ops.linear(x, [wg, wu], ws, epilogue=2, layout=1, out=out)
    ref = torch.nn.functional.silu(x.float() @ wg.float().T) * (x.float() @ wu.float().T)
    torch.cuda.synchronize()
    _close(out, ref, rtol=1e-2 if dtype == torch.bfloat16 else 1e-5, atol_frac=1e-2 if dtype == torch.bfloat16 else 1e-5)


def rope_tables(head_dim, max_pos, theta=500000.0):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    f = torch.arange(max_pos).float()[:, None] * inv[None, :]
    return f.cos().to(DEV), f.sin().to(DEV)


def rope_ref(x, pos, cos, sin):
    # x [T, H, hd]
    c = cos[pos.long()][:, None, :].repeat(1, 1, 2)
    s = sin[pos.long()][:, None, :].repeat(1, 1, 2)
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], -1)
    return x * c + rot * s


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,Hkv,hd,d,T", [(32, 8, 128, 4096, 33), (32, 8, 64, 2048, 1), (4, 2, 16, 64, 7)])
def test_qkv_rope(ops, ws, dtype, H, Hkv, hd, d, T):
    x = _rand(T, d, dtype=dtype, seed=14)
    wq = _rand(H * hd, d, dtype=dtype, scale=0.02, seed=15)
    wk = _rand(Hkv * hd, d, dtype=dtype, scale=0.02, seed=16)
    wv = _rand(Hkv * hd, d, dtype=dtype, scale=0.02, seed=17)
    cos, sin = rope_tables(hd, 4096)
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32)
    slots = torch.randperm(T + 10, device=DEV)[:T].to(torch.int32)
    max_slots = T + 16
    kc = torch.zeros(Hkv, max_slots, hd, dtype=dtype, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.empty(T, H * hd, dtype=dtype, device=DEV)
    ops.qkv_rope(x, wq, wk, wv, H, Hkv, hd, cos, sin, pos, slots, kc, vc, q, ws)
    torch.cuda.synchronize()
    ws.check_status()
    xf = x.float()
    qr = rope_ref((xf @ wq.float().T).view(T, H, hd), pos, cos, sin).reshape(T, -1)
    kr = rope_ref((xf @ wk.float().T).view(T, Hkv, hd), pos, cos, sin)
    vr = (xf @ wv.float().T).view(T, Hkv, hd)
    tol = dict(rtol=1e-2, atol_frac=1e-2) if dtype == torch.bfloat16 else dict(rtol=1e-4, atol_frac=1e-5)
    _close(q, qr, **tol)
    _close(kc[:, slots.long()].permute(1, 0, 2), kr, **tol)
    _close(vc[:, slots.long()].permute(1, 0, 2), vr, **tol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T,V,K", [(1, 128256, 4096), (25, 128256, 2048), (3, 1000, 64)])
def test_head_argmax(ops, ws, dtype, T, V, K):
    x = _rand(T, K, dtype=dtype, seed=18)
    w = _rand(V, K, dtype=dtype, scale=0.02, seed=19)
    idx = torch.empty(T, dtype=torch.int32, device=DEV)
    mx = torch.empty(T, dtype=torch.float32, device=DEV)
    gap = torch.empty(T, dtype=torch.float32, device=DEV)
    ops.head_argmax(x, w, idx, ws, out_max=mx, out_gap=gap)
    logits = x.double() @ w.double().T
    top2 = logits.topk(2, dim=-1).values
    torch.cuda.synchronize()
    ref = logits.argmax(-1)
    near_tie = (top2[:, 0] - top2[:, 1]) < 1e-4
    assert ((idx.long() == ref) | near_tie).all()
    torch.testing.assert_close(mx.double(), top2[:, 0], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(gap.double(), top2[:, 0] - top2[:, 1], rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T,V,K,k,subset", [(1, 128256, 4096, 4, False), (16, 32768, 2048, 2, True),
                                             (8, 128, 64, 3, False), (4, 5000, 256, 16, True)])
def test_head_topk(ops, ws, dtype, T, V, K, k, subset):
    x = _rand(T, K, dtype=dtype, seed=20)
    w = _rand(V, K, dtype=dtype, scale=0.05, seed=21)
    vocab_ids = None
    if subset:
        vocab_ids = torch.randperm(V * 3, device=DEV)[:V].sort().values.to(torch.int64)
    tok = torch.empty(T, k, dtype=torch.int32, device=DEV)
    lp = torch.empty(T, k, dtype=torch.float32, device=DEV)
    ops.head_topk(x, w, k, tok, lp, ws, vocab_ids=vocab_ids)
    logits = x.double() @ w.double().T
    ref_lp, ref_i = torch.log_softmax(logits, -1).topk(k, dim=-1)
    torch.cuda.synchronize()
    ref_tok = vocab_ids[ref_i] if subset else ref_i
    srt = torch.log_softmax(logits, -1).topk(k + 1, dim=-1).values
    gaps = (srt[:, :-1] - srt[:, 1:]).abs()
    ok = (tok.long() == ref_tok) | (gaps < 1e-4)
    assert ok.all()
    torch.testing.assert_close(lp.double(), ref_lp, rtol=1e-4, atol=2e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gemm_batch_invariance(ops, ws, dtype):
    """A token's output bits do not depend on how many rows share the GEMM."""
    K, N, T = 4096, 6144, 33
    x = _rand(T, K, dtype=dtype, seed=22)
    w = _rand(N, K, dtype=dtype, scale=0.02, seed=23)
    full = torch.empty(T, N, dtype=torch.float32, device=DEV)
    ops.linear(x, [w], ws, epilogue=3, out=full)
    for t in (0, 7, 32):
        one = torch.empty(1, N, dtype=torch.float32, device=DEV)
        ops.linear(x[t:t + 1].contiguous(), [w], ws, epilogue=3, out=one)
        torch.cuda.synchronize()
        assert torch.equal(one[0], full[t]), f"row {t} differs between T=1 and T={T}"


def attention_ref(q, kc, vc, prefix, spec_base, mask, H, Hkv, hd, start=None):
    """Explicit per-row masked softmax attention in fp64 (row t sees slots
    [start[t], prefix[t]) plus its mask bits)."""
    T = q.shape[0]
    G = H // Hkv
    out = torch.zeros(T, H * hd, dtype=torch.float64, device=DEV)
    S = kc.shape[1]
    for t in range(T):
        valid = torch.zeros(S, dtype=torch.bool, device=DEV)
        valid[int(start[t]) if start is not None else 0: int(prefix[t])] = True
        if mask is not None:
            for b in range(mask.shape[1] * 64):
                if (int(mask[t, b // 64].item()) >> (b % 64)) & 1:
                    valid[int(spec_base) + b] = True
        idx = valid.nonzero().flatten()
        for h in range(H):
            g = h // G
            qv = q[t, h * hd:(h + 1) * hd].double()
            k = kc[g, idx].double()
            v = vc[g, idx].double()
            p = torch.softmax(k @ qv / math.sqrt(hd), 0)
            out[t, h * hd:(h + 1) * hd] = p @ v
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,Hkv,hd,ctx,T,tree", [(32, 8, 128, 2048, 33, True), (4, 2, 16, 40, 5, True),
                                                  (32, 8, 64, 300, 1, False), (8, 8, 128, 5000, 9, True),
                                                  (64, 8, 128, 700, 33, True), (16, 2, 128, 16384, 17, True),
                                                  (32, 8, 128, 130, 40, False), (8, 4, 64, 1000, 16, True),
                                                  (32, 8, 128, 32768, 9, True), (32, 8, 128, 20000, 60, True),
                                                  (16, 4, 64, 12000, 25, True)])
def test_tree_attention(ops, ws, dtype, H, Hkv, hd, ctx, T, tree):
    torch.manual_seed(0)
    S = ctx + 80
    kc = _rand(Hkv, S, hd, dtype=dtype, seed=24)
    vc = _rand(Hkv, S, hd, dtype=dtype, seed=25)
    q = _rand(T, H * hd, dtype=dtype, seed=26)
    if tree:
        # row 0 = root (prefix only); nodes see random ancestors among spec slots
        prefix = torch.full((T,), ctx, dtype=torch.int32, device=DEV)
        m = torch.zeros(T, 1, dtype=torch.int64)
        for t in range(1, T):
            bits = (1 << (t - 1))
            for j in range(t - 1):
                if torch.rand(()) < 0.3:
                    bits |= 1 << j
            m[t, 0] = bits
        mask = m.to(DEV)  # int64 storage carries the uint64 bit pattern
        spec_base = torch.tensor([ctx], dtype=torch.int32, device=DEV)
    else:
        prefix = torch.tensor([ctx - T + 1 + t for t in range(T)], dtype=torch.int32, device=DEV)
        mask, spec_base = None, None
    out = torch.empty(T, H * hd, dtype=dtype, device=DEV)
    ops.tree_attention(q, kc, vc, H, Hkv, hd, prefix, out, ws, spec_base=spec_base, spec_mask=mask, kv_bound=S)
    torch.cuda.synchronize()
    ws.check_status()
    ref = attention_ref(q, kc, vc, prefix.cpu(), ctx, mask.cpu() if mask is not None else None,
                        H, Hkv, hd)
    tol = dict(rtol=2e-2, atol_frac=1e-2) if dtype == torch.bfloat16 else dict(rtol=1e-4, atol_frac=1e-5)
    _close(out, ref, **tol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,Hkv,hd,B,region,T_per", [(32, 8, 128, 4, 700, 1), (32, 8, 128, 8, 2304, 1),
                                                     (32, 8, 64, 3, 300, 2), (32, 8, 128, 6, 1000, 4)])
def test_tree_attention_per_row_slot_ranges(ops, ws, dtype, H, Hkv, hd, B, region, T_per):
    """Batched decoding: B sequences share one cache, sequence b in slots
    [b * region, (b + 1) * region); each row sees only its own sequence's
    slots [prefix_start, prefix_len). Covers the mma.sync kernel (<= 16 rows per
    KV head), the tcgen05 kernel (more) and the fp32 kernel."""
    T = B * T_per
    S = B * region
    kc = _rand(Hkv, S, hd, dtype=dtype, seed=31)
    vc = _rand(Hkv, S, hd, dtype=dtype, seed=32)
    q = _rand(T, H * hd, dtype=dtype, seed=33)
    g = torch.Generator().manual_seed(5)
    lens = torch.randint(region // 4, region - T_per, (B,), generator=g)
    start = torch.tensor([b * region for b in range(B) for _ in range(T_per)], dtype=torch.int32)
    prefix = torch.tensor([b * region + int(lens[b]) + j + 1 for b in range(B) for j in range(T_per)],
                          dtype=torch.int32)
    out = torch.empty(T, H * hd, dtype=dtype, device=DEV)
    ops.tree_attention(q, kc, vc, H, Hkv, hd, prefix.to(DEV), out, ws, kv_bound=S, prefix_start=start.to(DEV))
    torch.cuda.synchronize()
    ws.check_status()
    ref = attention_ref(q, kc, vc, prefix, None, None, H, Hkv, hd, start=start)
    tol = dict(rtol=2e-2, atol_frac=1e-2) if dtype == torch.bfloat16 else dict(rtol=1e-4, atol_frac=1e-5)
    _close(out, ref, **tol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("keep", [[6, 7, 9], [10, 12, 13, 15], [3, 4, 5], [20]])
def test_kv_compact(ops, dtype, keep):
    Lyr, Hkv, S, hd = 3, 2, 32, 64
    cache = _rand(Lyr, 2, Hkv, S, hd, dtype=dtype, seed=27)
    ref = cache.clone()
    start = keep[0]
    idx = torch.tensor(keep, device=DEV)
    ref[:, :, :, start:start + len(keep)] = ref.index_select(3, idx)
    ks = torch.tensor(keep, dtype=torch.int32, device=DEV)
    st = torch.tensor([start], dtype=torch.int32, device=DEV)
    nk = torch.tensor([len(keep)], dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.kv_compact(cache, st, ks, nk, max_keep=8, status=status)
    torch.cuda.synchronize()
    assert torch.equal(cache, ref)
    assert int(status.item()) == 0


def test_kv_compact_rejects_a_keep_list_that_does_not_fit(ops):
    """A keep list naming a slot past the cache, or longer than max_keep,
    copies nothing and sets the status word's bad-index bit."""
    cache = _rand(2, 2, 2, 16, 64, dtype=torch.bfloat16, seed=28)
    ref = cache.clone()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    i32 = dict(dtype=torch.int32, device=DEV)
    ops.kv_compact(cache, torch.tensor([4], **i32), torch.tensor([5, 16], **i32), torch.tensor([2], **i32),
                   max_keep=4, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 2 and torch.equal(cache, ref)
    status.zero_()
    ops.kv_compact(cache, torch.tensor([4], **i32), torch.tensor([5, 6, 7], **i32), torch.tensor([3], **i32),
                   max_keep=2, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 2 and torch.equal(cache, ref)


@pytest.mark.parametrize("name,over", [("tiny", {}), ("llama32_1b", dict(num_hidden_layers=2, vocab_size=4096))])
def test_folded_rmsnorm_matches_standalone(name, over):
    """bf16 forward with the RMSNorms folded into the GEMM epilogues vs the
    standalone RMSNorm kernel: same logits up to bf16 rounding."""
    from ssd import synthetic as S
    from ssd.engine.speculative import TargetRunner
    from ssd.models import runner as R

    base = S.build_base_model(name, 3, torch.bfloat16, DEV, gen_device="cuda", **over)
    target = TargetRunner(base)
    w = target.weights
    T = 9
    ids = torch.randint(0, w.V, (T,), generator=torch.Generator().manual_seed(1))
    outs = []
    for folded in (False, True):
        cache = target.new_cache(32)
        cache.allocate(w.Hkv, w.hd, w.dtype, w.device)
        fwd = R.ForwardInputs(T, DEV, mask_words=1)
        fwd.fill(ids, torch.arange(T), 0, None)
        scratch = R.Scratch(w, T)
        from ssd import ops as O
        wsp = O.Workspace(DEV, max_rows=64, vocab=w.V, max_head_rows=T)
        layers = list(range(w.L))
        logits = torch.empty(T, w.V, dtype=torch.float32, device=DEV)
        if folded:
            R.run_stack_folded(w, layers, [None] * w.L, None, fwd, T, cache, scratch, wsp, cache.max_length)
            x, rn = R.final_norm_folded(w, scratch, 0, T)
            O.linear(x, [w.lm_head], wsp, epilogue=3, out=logits, in_norm=rn)
        else:
            R.run_stack(w, layers, [None] * w.L, None, fwd, T, cache, scratch, wsp, cache.max_length)
            x = R.final_norm(w, scratch, 0, T)
            O.linear(x, [w.lm_head], wsp, epilogue=3, out=logits)
        torch.cuda.synchronize()
        wsp.check_status()
        outs.append(logits)
    ref, got = outs
    scale = ref.abs().max()
    assert (got - ref).abs().max() <= 2e-2 * scale, ((got - ref).abs().max(), scale)
    assert (got.argmax(-1) == ref.argmax(-1)).float().mean() >= 0.8


@pytest.mark.parametrize("seed,n", [(0, 1), (1, 6), (2, 24), (3, 32)])
def test_greedy_verify_matches_oracle(seed, n):
    """greedy_verify (verify.py:45-57) on the device tree walk: accepted path
    and bonus equal the oracle's on random trees whose target rows often pick
    a child's token (deep walks), including duplicate sibling tokens, where
    the first child in rank order must win."""
    import random

    import numpy as np

    from oracle import tree as OT
    from ssd.engine.verify import greedy_verify
    from test_cpu_host import _random_tree

    V = 50
    t = _random_tree(seed, n, vocab=8)  # few distinct tokens: sibling duplicates
    rng = random.Random(seed + 100)
    logits = np.random.default_rng(seed).standard_normal((n + 1, V)).astype(np.float32)
    kids = t.children()
    for row in range(n + 1):
        ch = kids.get(row - 1, [])
        if ch and rng.random() < 0.8:
            logits[row, t.tokens[rng.choice(ch)]] = 10.0
    ot = OT.DraftTree(tokens=list(t.tokens), parents=list(t.parents), depths=list(t.depths), scores=list(t.scores),
                      ranks=list(t.ranks), draft_pos=list(t.draft_pos))
    want = OT.greedy_verify(ot, logits)
    got = greedy_verify(t, torch.tensor(logits, device=DEV))
    assert got == (want[0], want[1])


# ------------------------------------------------------------ GEMM chain
def _chain_layer(ops, ws, T, d, F, H, Hkv, hd, chained, seed=40, bridge=None, draw_rows=None):
    """One decoder layer's GEMMs after attention: o_proj (+ residual, next
    norm input), gate/up SwiGLU (folded norm), down (+ residual, next norm
    input), optionally a SwiGLU bridge (gate/up, out_proj + residual), then
    the next layer's q/k/v with RoPE and cache write; either as one
    ssd_linear_chain launch or as separate launches. Row inputs are drawn
    for `draw_rows` rows and the first T used, so row t sees the same data
    whatever T is."""
    import ssd._lib as L

    R = draw_rows or T
    g = torch.Generator(device=DEV).manual_seed(seed)
    rn = lambda *s, scale=1.0: (torch.randn(*s, generator=g, device=DEV) * scale)
    wo = rn(d, H * hd, scale=0.02).bfloat16()
    wg, wu = rn(F, d, scale=0.02).bfloat16(), rn(F, d, scale=0.02).bfloat16()
    wd = rn(d, F, scale=0.02).bfloat16()
    wq, wk, wv = rn(H * hd, d, scale=0.02).bfloat16(), rn(Hkv * hd, d, scale=0.02).bfloat16(), \
        rn(Hkv * hd, d, scale=0.02).bfloat16()
    ln2, ln_mid, ln_next = [(1 + 0.1 * rn(d)).bfloat16() for _ in range(3)]
    bw = [rn(bridge, d, scale=0.02).bfloat16(), rn(bridge, d, scale=0.02).bfloat16(),
          rn(d, bridge, scale=0.02).bfloat16()] if bridge else None
    attn = rn(R, H * hd).bfloat16()[:T].contiguous()
    resid = rn(R, d)[:T].contiguous()
    parts = d // 128
    xg = torch.zeros(T, d, dtype=torch.bfloat16, device=DEV)
    ssq = torch.zeros(T, parts, device=DEV)
    hid = torch.zeros(T, F, dtype=torch.bfloat16, device=DEV)
    cos, sin = rope_tables(hd, 4096)
    pos = ((torch.arange(T, device=DEV, dtype=torch.int32) * 37 + 5) % 4000).to(torch.int32)
    slots = torch.arange(T, device=DEV, dtype=torch.int32)
    kc = torch.zeros(Hkv, T + 8, hd, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.zeros(T, H * hd, dtype=torch.bfloat16, device=DEV)
    c = ops.GemmChain(ws, T, chained)
    c.linear(attn, [wo], epilogue=L.EPI_RESIDUAL, resid=resid, norm_out=ops.NormOut(ln2, xg, ssq))
    c.linear(xg, [wg, wu], epilogue=L.EPI_SWIGLU, layout=L.SEG_PAIRS, out=hid,
             in_norm=ops.RowNorm(ssq, parts, d, 1e-5))
    c.linear(hid, [wd], epilogue=L.EPI_RESIDUAL, resid=resid,
             norm_out=ops.NormOut(ln_mid if bridge else ln_next, xg, ssq))
    out = {}
    if bridge:
        bh = torch.zeros(T, bridge, dtype=torch.bfloat16, device=DEV)
        c.linear(xg, bw[:2], epilogue=L.EPI_SWIGLU, layout=L.SEG_PAIRS, out=bh,
                 in_norm=ops.RowNorm(ssq, parts, d, 1e-5))
        c.linear(bh, [bw[2]], epilogue=L.EPI_RESIDUAL, resid=resid, norm_out=ops.NormOut(ln_next, xg, ssq))
        out["bh"] = bh
    c.qkv(xg, wq, wk, wv, H, Hkv, hd, cos, sin, pos, slots, kc, vc, q, in_norm=ops.RowNorm(ssq, parts, d, 1e-6))
    c.flush()
    torch.cuda.synchronize()
    ws.check_status()
    out.update(resid=resid, xg=xg, ssq=ssq, hid=hid, q=q, k=kc[:, :T].transpose(0, 1), v=vc[:, :T].transpose(0, 1))
    return out


CHAIN_SHAPES = [(33, 4096, 14336, 32, 8, 128), (1, 4096, 14336, 32, 8, 128), (7, 256, 512, 4, 2, 64),
                (64, 1024, 2816, 8, 2, 128)]


@pytest.mark.parametrize("T,d,F,H,Hkv,hd", CHAIN_SHAPES)
@pytest.mark.parametrize("bridge", [None, 1024])
def test_linear_chain_matches_separate_launches(ops, ws, T, d, F, H, Hkv, hd, bridge):
    """ssd_linear_chain vs the same GEMMs launched one by one. The K splits
    differ, so a link's fp32 sums differ in the last bits; where a link's
    output is rounded to bf16 (norm inputs, SwiGLU) such a difference can
    move a value by one bf16 step, and the next link carries that on: the
    fp32 residual agrees to 3e-3 of its scale, bf16 outputs to 3e-2."""
    a = _chain_layer(ops, ws, T, d, F, H, Hkv, hd, True, bridge=bridge)
    b = _chain_layer(ops, ws, T, d, F, H, Hkv, hd, False, bridge=bridge)
    _close(a["resid"], b["resid"], rtol=1e-2, atol_frac=3e-3)
    _close(a["ssq"], b["ssq"], rtol=1e-2, atol_frac=3e-3)
    for key in ("xg", "hid", "q", "k", "v") + (("bh",) if bridge else ()):
        _close(a[key], b[key], rtol=3e-2, atol_frac=3e-2)


@pytest.mark.parametrize("T,K,N", [(33, 4096, 4096), (1, 14336, 4096), (7, 256, 384), (64, 4096, 6144)])
def test_linear_chain_single_link_matches_linear(ops, ws, T, K, N):
    """One residual link with a folded norm output: the chain and ssd_linear
    see identical inputs, so the fp32 residual agrees to fp32 summation
    order (1e-5 of its scale) and the bf16 norm input to one bf16 step."""
    import ssd._lib as L

    x = _rand(T, K, seed=50)
    w = _rand(N, K, scale=0.02, seed=51)
    wn = (1 + 0.1 * _rand(N, dtype=torch.float32, seed=52)).bfloat16()
    r0 = _rand(T, N, dtype=torch.float32, seed=53)
    outs = []
    for chained in (True, False):
        resid = r0.clone()
        xg = torch.zeros(T, N, dtype=torch.bfloat16, device=DEV)
        ssq = torch.zeros(T, (N + 127) // 128, device=DEV)
        c = ops.GemmChain(ws, T, chained)
        c.linear(x, [w], epilogue=L.EPI_RESIDUAL, resid=resid, norm_out=ops.NormOut(wn, xg, ssq))
        c.flush()
        torch.cuda.synchronize()
        ws.check_status()
        outs.append((resid, xg, ssq))
    ref = r0 + x.float() @ w.float().T
    _close(outs[0][0], ref, rtol=1e-4, atol_frac=1e-5)
    _close(outs[0][0], outs[1][0], rtol=1e-5, atol_frac=1e-5)
    _close(outs[0][1], outs[1][1], rtol=1e-2, atol_frac=1e-2)
    _close(outs[0][2], outs[1][2], rtol=1e-4, atol_frac=1e-5)


@pytest.mark.parametrize("d,F,H,Hkv,hd", [(4096, 14336, 32, 8, 128), (256, 512, 4, 2, 64)])
def test_linear_chain_batch_invariant(ops, ws, d, F, H, Hkv, hd):
    """A row's chained results do not depend on how many rows run with it:
    every link's K split depends only on the weight shapes and the grid."""
    full = _chain_layer(ops, ws, 64, d, F, H, Hkv, hd, True, seed=41, bridge=512, draw_rows=64)
    for T in (1, 17, 33):
        part = _chain_layer(ops, ws, T, d, F, H, Hkv, hd, True, seed=41, bridge=512, draw_rows=64)
        for key, v in part.items():
            assert torch.equal(v, full[key][:T]), (T, key)


def test_linear_chain_rejects_bad_arguments(ops, ws):
    import ssd._lib as L

    x = torch.zeros(4, 128, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(128, 128, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros(4, 128, dtype=torch.bfloat16, device=DEV)
    a = ops.linear_args(x, [w], out=out)
    with pytest.raises(ValueError):
        ops.linear_chain([a] * 7, 4, ws)  # more than 6 links
    big = torch.zeros(65, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(L.SSDError):
        ops.linear_chain([ops.linear_args(big, [w], out=torch.zeros_like(big))], 65, ws)  # T > 64
    bad = ops.linear_args(x, [w], out=out)
    bad.epilogue = 99
    with pytest.raises(ValueError):
        ops.linear_chain([bad], 4, ws)
