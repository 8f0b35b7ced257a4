"""Layer kernels and the speculative engine on the B200 against the CPU oracle (oracle/model.py), and the
engine's own invariants: a verify row equals a one-row decode bit for bit, so speculative decoding returns
exactly the tokens of plain greedy decoding (the reference's "speculation changes no answer",
tests/engine/test_speculation.py:79-125), and a draft model identical to the target has every draft accepted."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ironmule_b200 import engine, kernels
from oracle import bf16
from oracle import model as om

from .gpu_util import bf16_bits_to_torch, torch_to_bf16_bits

pytestmark = pytest.mark.gpu


def rand_bits(rng, shape, sigma=1.0):
    return bf16.from_f32(rng.normal(0, sigma, shape).astype(np.float32))


def test_rmsnorm_matches_oracle(cuda):
    rng = np.random.default_rng(0)
    for gemma in (False, True):
        x = rand_bits(rng, (7, 2560))
        w = rand_bits(rng, (2560,), 0.3)
        got = torch_to_bf16_bits(kernels.rmsnorm(bf16_bits_to_torch(x, cuda), bf16_bits_to_torch(w, cuda), 1e-6,
                                                 gemma=gemma))
        want = om.rmsnorm(x, w, 1e-6, gemma)
        assert np.mean(got == want) > 0.99
        assert np.max(np.abs(bf16.to_f32(got) - bf16.to_f32(want))) <= 2 ** -6 * np.max(np.abs(bf16.to_f32(want)))


def test_strided_rmsnorm_rows(cuda):
    rng = np.random.default_rng(1)
    x = rand_bits(rng, (6, 256))
    w = rand_bits(rng, (256,))
    xt, wt = bf16_bits_to_torch(x, cuda), bf16_bits_to_torch(w, cuda)
    every_other = kernels.rmsnorm(xt[1:], wt, 1e-6, rows=3, ldx=512)
    assert torch.equal(every_other, kernels.rmsnorm(xt, wt, 1e-6)[1::2])


def test_qk_norm_rope_kv_matches_oracle(cuda):
    rng = np.random.default_rng(2)
    m, hq, hkv, d = 5, 8, 2, 128
    qkv = rand_bits(rng, (m, (hq + 2 * hkv) * d))
    qn, kn = rand_bits(rng, (d,), 0.5), rand_bits(rng, (d,), 0.5)
    pos = np.array([3, 17, 18, 400, 900], dtype=np.int32)
    inv_freq = (1e6 ** (-2.0 * np.arange(d // 2) / d)).astype(np.float32)
    pages, max_pages = 64, 64
    kc = torch.zeros((pages, hkv, 16, d), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    table = torch.arange(pages, dtype=torch.int32, device=cuda).flip(0).view(1, max_pages).contiguous()
    p = torch.from_numpy(pos).to(cuda)
    q = kernels.qk_norm_rope_kv(bf16_bits_to_torch(qkv, cuda), bf16_bits_to_torch(qn, cuda),
                                bf16_bits_to_torch(kn, cuda), torch.from_numpy(inv_freq).to(cuda), p, p,
                                torch.zeros(m, dtype=torch.int32, device=cuda), table, hq, hkv, d, 1e-6, kc, vc)
    x = qkv.reshape(m, hq + 2 * hkv, d)
    want_q = om.rope(bf16.to_f32(om.rmsnorm(x[:, :hq], qn, 1e-6)), pos, inv_freq)
    want_k = om.rope(bf16.to_f32(om.rmsnorm(x[:, hq:hq + hkv], kn, 1e-6)), pos, inv_freq)
    got_q = torch_to_bf16_bits(q)
    assert np.mean(got_q == want_q) > 0.97
    assert np.max(np.abs(bf16.to_f32(got_q) - bf16.to_f32(want_q))) < 0.05
    tbl = table.cpu().numpy()[0]
    for r, s in enumerate(pos):
        page = tbl[s // 16]
        got_k = torch_to_bf16_bits(kc[page, :, s % 16])
        assert np.mean(got_k == want_k[r]) > 0.97
        assert np.array_equal(torch_to_bf16_bits(vc[page, :, s % 16]), x[r, hq + hkv:])


def _paged(kv_bits, table_row, pages, cuda):
    """[S, Hkv, D] slot-major bits -> a [pages, Hkv, 16, D] cache laid out by the page table row."""
    s, hkv, d = kv_bits.shape
    cache = np.zeros((pages, hkv, 16, d), dtype=np.uint16)
    for slot in range(s):
        cache[table_row[slot // 16], :, slot % 16] = kv_bits[slot]
    return bf16_bits_to_torch(cache, cuda)


@pytest.mark.parametrize("d,hq,hkv,rows,window,kpc", [(128, 32, 8, 5, 0, 64), (128, 16, 8, 2, 0, 128),
                                                       (256, 16, 8, 5, 100, 64), (128, 4, 1, 32, 0, 256)])
def test_attention_matches_oracle(cuda, d, hq, hkv, rows, window, kpc):
    rng = np.random.default_rng(d + hq + rows)
    b = 3
    lens = [700, 130, 17 + rows]
    max_pages = 48
    table = rng.permutation(b * max_pages).reshape(b, max_pages).astype(np.int32)  # disjoint pages per sequence
    kcache = np.zeros((b * max_pages, hkv, 16, d), dtype=np.uint16)
    vcache = np.zeros_like(kcache)
    qs, slots, seq_rows, per_seq = [], [], [0], []
    for s in range(b):
        k = rand_bits(rng, (lens[s], hkv, d))
        v = rand_bits(rng, (lens[s], hkv, d))
        for slot in range(lens[s]):
            kcache[table[s, slot // 16], :, slot % 16] = k[slot]
            vcache[table[s, slot // 16], :, slot % 16] = v[slot]
        rs = np.arange(lens[s] - rows, lens[s])
        q = rand_bits(rng, (rows, hq, d))
        qs.append(q)
        slots.append(rs)
        seq_rows.append(seq_rows[-1] + rows)
        per_seq.append((k, v, rs, q))
    q_all = np.concatenate(qs)
    out = kernels.attention(bf16_bits_to_torch(q_all, cuda), bf16_bits_to_torch(kcache, cuda),
                            bf16_bits_to_torch(vcache, cuda), torch.from_numpy(table).to(cuda),
                            torch.tensor(seq_rows, dtype=torch.int32, device=cuda),
                            torch.from_numpy(np.concatenate(slots).astype(np.int32)).to(cuda),
                            max_rows_per_seq=rows, max_kv_len=max_pages * 16, scale=d ** -0.5,
                            keys_per_split=kpc, window=window)
    got = torch_to_bf16_bits(out)
    for s, (k, v, rs, q) in enumerate(per_seq):
        want = om.attention(q, k, v, rs, d ** -0.5, window)
        part = got[seq_rows[s]:seq_rows[s + 1]]
        err = np.abs(bf16.to_f32(part) - bf16.to_f32(want))
        assert err.max() <= 1e-2 * np.abs(bf16.to_f32(want)).max() + 1e-3
        assert np.mean(part == want) > 0.9


def test_attention_tree_mask(cuda):
    rng = np.random.default_rng(9)
    d, hq, hkv = 128, 4, 2
    prefix, nodes = 40, 6
    parents = [-1, 0, 0, 1, 2, 2]  # node 0 is the root of the draft tree
    masks = []
    for i in range(nodes):
        m, j = 0, i
        while j >= 0:
            m |= 1 << j
            j = parents[j]
        masks.append(m)
    total = prefix + nodes
    k, v = rand_bits(rng, (total, hkv, d)), rand_bits(rng, (total, hkv, d))
    table = np.arange(8, dtype=np.int32)[None]
    slots = np.arange(prefix, total)
    q = rand_bits(rng, (nodes, hq, d))
    out = kernels.attention(bf16_bits_to_torch(q, cuda), _paged(k, table[0], 8, cuda), _paged(v, table[0], 8, cuda),
                            torch.from_numpy(table).to(cuda), torch.tensor([0, nodes], dtype=torch.int32, device=cuda),
                            torch.from_numpy(slots.astype(np.int32)).to(cuda), max_rows_per_seq=nodes,
                            max_kv_len=128, scale=d ** -0.5,
                            tree_mask=torch.tensor(masks, dtype=torch.int64, device=cuda),
                            tree_base=torch.tensor([prefix], dtype=torch.int32, device=cuda))
    want = om.attention(q, k, v, slots, d ** -0.5, tree_mask=masks, tree_base=prefix)
    err = np.abs(bf16.to_f32(torch_to_bf16_bits(out)) - bf16.to_f32(want))
    assert err.max() <= 1e-2 * np.abs(bf16.to_f32(want)).max() + 1e-3


@pytest.mark.parametrize("d,hq,hkv,rows,window,kpc,tree,gemma", [
    (128, 32, 8, 5, 0, 64, False, False), (128, 16, 8, 2, 0, 64, False, False), (128, 4, 1, 32, 0, 128, False, False),
    (256, 16, 8, 5, 100, 64, False, True), (128, 8, 2, 6, 0, 64, True, False)])
def test_fused_attention_equals_rope_then_attention(cuda, d, hq, hkv, rows, window, kpc, tree, gemma):
    """im_attention_qkv_paged == im_qk_norm_rope_kv + im_attention_paged, bit for bit: outputs and the K/V it
    writes. The fused path must not read the new rows' slots from the cache, so they start as garbage there."""
    rng = np.random.default_rng(d + hq + rows + 7 * tree)
    b, max_pages = 3, 48
    lens = [700, 130, 17 + rows]
    table = rng.permutation(b * max_pages).reshape(b, max_pages).astype(np.int32)
    shape = (b * max_pages, hkv, 16, d)
    kc0, vc0 = rand_bits(rng, shape), rand_bits(rng, shape)
    m = b * rows
    qkv = rand_bits(rng, (m, (hq + 2 * hkv) * d))
    qn, kn = rand_bits(rng, (d,), 0.5), rand_bits(rng, (d,), 0.5)
    inv_freq = torch.from_numpy((1e6 ** (-2.0 * np.arange(d // 2) / d)).astype(np.float32)).to(cuda)
    slots = np.concatenate([np.arange(n - rows, n) for n in lens]).astype(np.int32)
    pos = slots.copy()
    masks = tb = None
    if tree:  # rows are draft-tree nodes: a chain per sequence off node 0, RoPE positions by depth
        parents = [-1] + list(range(rows - 1))
        mk = []
        for i in range(rows):
            mm, j = 0, i
            while j >= 0:
                mm |= 1 << j
                j = parents[j]
            mk.append(mm)
        masks = torch.tensor(mk * b, dtype=torch.int64, device=cuda)
        tb = torch.tensor([n - rows for n in lens], dtype=torch.int32, device=cuda)
        pos = np.concatenate([np.arange(n - rows, n) - 3 for n in lens]).astype(np.int32)
    seq_rows = torch.arange(0, m + 1, rows, dtype=torch.int32, device=cuda)
    row_seq = torch.arange(b, dtype=torch.int32, device=cuda).repeat_interleave(rows)
    tbl, sl, ps = torch.from_numpy(table).to(cuda), torch.from_numpy(slots).to(cuda), torch.from_numpy(pos).to(cuda)
    qkv_t, qn_t, kn_t = bf16_bits_to_torch(qkv, cuda), bf16_bits_to_torch(qn, cuda), bf16_bits_to_torch(kn, cuda)
    kw = dict(max_rows_per_seq=rows, max_kv_len=max_pages * 16, scale=d ** -0.5, keys_per_split=kpc, window=window,
              tree_mask=masks, tree_base=tb)
    kc_a, vc_a = bf16_bits_to_torch(kc0, cuda), bf16_bits_to_torch(vc0, cuda)
    q = kernels.qk_norm_rope_kv(qkv_t, qn_t, kn_t, inv_freq, ps, sl, row_seq, tbl, hq, hkv, d, 1e-6, kc_a, vc_a,
                                gemma=gemma)
    want = kernels.attention(q, kc_a, vc_a, tbl, seq_rows, sl, **kw)
    kc_b, vc_b = bf16_bits_to_torch(kc0, cuda), bf16_bits_to_torch(vc0, cuda)
    got = kernels.attention_qkv(qkv_t, qn_t, kn_t, inv_freq, ps, kc_b, vc_b, tbl, seq_rows, sl, hq=hq, hkv=hkv, d=d,
                                eps=1e-6, gemma=gemma, **kw)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert torch.equal(kc_a.view(torch.int16), kc_b.view(torch.int16))
    assert torch.equal(vc_a.view(torch.int16), vc_b.view(torch.int16))


@pytest.mark.parametrize("d,hq,hkv,rows,tree", [(128, 32, 8, 5, False), (256, 16, 8, 7, True),
                                                 (128, 16, 8, 1, False)])
def test_attention_ctas_per_group_change_no_bits(cuda, d, hq, hkv, rows, tree):
    """32 sequences: with few waves a CTA walks several splits; with many, each split has its own CTA. Outputs
    and the K/V written are the same bits either way, fused and unfused."""
    rng = np.random.default_rng(d + rows)
    b, max_pages = 32, 40
    lens = rng.integers(rows + 1, max_pages * 16 - 8, b).tolist()
    table = rng.permutation(b * max_pages).reshape(b, max_pages).astype(np.int32)
    shape = (b * max_pages, hkv, 16, d)
    kc0, vc0 = rand_bits(rng, shape), rand_bits(rng, shape)
    m = b * rows
    qkv = rand_bits(rng, (m, (hq + 2 * hkv) * d))
    qn, kn = rand_bits(rng, (d,), 0.5), rand_bits(rng, (d,), 0.5)
    inv_freq = torch.from_numpy((1e6 ** (-2.0 * np.arange(d // 2) / d)).astype(np.float32)).to(cuda)
    slots = np.concatenate([np.arange(n - rows, n) for n in lens]).astype(np.int32)
    masks = tb = None
    if tree:
        masks = torch.tensor([(1 << (i + 1)) - 1 for i in range(rows)] * b, dtype=torch.int64, device=cuda)
        tb = torch.tensor([n - rows for n in lens], dtype=torch.int32, device=cuda)
    seq_rows = torch.arange(0, m + 1, rows, dtype=torch.int32, device=cuda)
    tbl, sl = torch.from_numpy(table).to(cuda), torch.from_numpy(slots).to(cuda)
    qkv_t, qn_t, kn_t = bf16_bits_to_torch(qkv, cuda), bf16_bits_to_torch(qn, cuda), bf16_bits_to_torch(kn, cuda)
    kw = dict(max_rows_per_seq=rows, max_kv_len=max_pages * 16, scale=d ** -0.5, tree_mask=masks, tree_base=tb)
    q = bf16_bits_to_torch(rand_bits(rng, (m, hq, d)), cuda)
    outs = []
    try:
        for waves in (1, 64):
            kernels.attention_tune(waves)
            kc, vc = bf16_bits_to_torch(kc0, cuda), bf16_bits_to_torch(vc0, cuda)
            got = kernels.attention_qkv(qkv_t, qn_t, kn_t, inv_freq, sl, kc, vc, tbl, seq_rows, sl, hq=hq, hkv=hkv,
                                        d=d, eps=1e-6, **kw)
            plain = kernels.attention(q, kc, vc, tbl, seq_rows, sl, **kw)
            torch.cuda.synchronize()
            outs.append([t.view(torch.int16).clone() for t in (got, plain, kc, vc)])
    finally:
        kernels.attention_tune(2)
    for x, y in zip(*outs):
        assert torch.equal(x, y)


@pytest.mark.parametrize("d,hq,hkv,rows,lens,kpc,hidden", [
    (128, 16, 8, 1, [600], 128, 1024),        # a config-2 draft pass
    (128, 16, 8, 2, [601], 128, 1024),        # its two-row catch-up pass
    (128, 16, 8, 1, [700, 130], 128, 1024),   # two sequences
    (128, 16, 8, 1, [1500], 64, 1024),        # 24 splits: the two-pass merge
    (256, 8, 4, 1, [333], 64, 1536)])
def test_o_projection_merges_the_attention_splits(cuda, d, hq, hkv, rows, lens, kpc, hidden):
    """attention_qkv(defer) + qgemm_packed_attn == attention_qkv + qgemm_packed(residual), bit for bit: the
    o-projection's prologue merges the split partials exactly as the attention's own merge does."""
    rng = np.random.default_rng(d + rows + len(lens) + kpc)
    b, max_pages = len(lens), 96
    table = rng.permutation(b * max_pages).reshape(b, max_pages).astype(np.int32)
    shape = (b * max_pages, hkv, 16, d)
    kc0, vc0 = rand_bits(rng, shape), rand_bits(rng, shape)
    m = b * rows
    qkv = rand_bits(rng, (m, (hq + 2 * hkv) * d))
    qn, kn = rand_bits(rng, (d,), 0.5), rand_bits(rng, (d,), 0.5)
    inv_freq = torch.from_numpy((1e6 ** (-2.0 * np.arange(d // 2) / d)).astype(np.float32)).to(cuda)
    slots = np.concatenate([np.arange(n - rows, n) for n in lens]).astype(np.int32)
    seq_rows = torch.arange(0, m + 1, rows, dtype=torch.int32, device=cuda)
    tbl, sl = torch.from_numpy(table).to(cuda), torch.from_numpy(slots).to(cuda)
    qkv_t, qn_t, kn_t = bf16_bits_to_torch(qkv, cuda), bf16_bits_to_torch(qn, cuda), bf16_bits_to_torch(kn, cuda)
    k = hq * d
    assert kernels.qgemm_packed_attn_rows(hidden, k) >= m
    w = torch.randint(-2 ** 31, 2 ** 31 - 1, (hidden, k // 8), dtype=torch.int32, device=cuda)
    sc = bf16_bits_to_torch(rand_bits(rng, (hidden, k // 64), 0.02), cuda)
    bi = bf16_bits_to_torch(rand_bits(rng, (hidden, k // 64), 0.02), cuda)
    p = kernels.Packed(w, sc, bi)
    h0 = bf16_bits_to_torch(rand_bits(rng, (m, hidden)), cuda)
    kw = dict(max_rows_per_seq=rows, max_kv_len=max_pages * 16, scale=d ** -0.5, keys_per_split=kpc)
    need = kernels.attention_workspace_bytes(b, rows, hq, hkv, d, max_pages * 16, kpc)
    outs = []
    for fused in (False, True):
        kc, vc = bf16_bits_to_torch(kc0, cuda), bf16_bits_to_torch(vc0, cuda)
        ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
        h, sq = h0.clone(), torch.zeros((hidden // 32, 32), dtype=torch.float32, device=cuda)
        attn = kernels.attention_qkv(qkv_t, qn_t, kn_t, inv_freq, sl, kc, vc, tbl, seq_rows, sl, hq=hq, hkv=hkv, d=d,
                                     eps=1e-6, ws=ws, defer=fused, **kw)
        if fused:
            assert attn is None
            kernels.qgemm_packed_attn(ws, p, seq_rows, sl, residual=h, out=h, rows=m, max_rows_per_seq=rows, hq=hq,
                                      hkv=hkv, d=d, max_kv_len=max_pages * 16, keys_per_split=kpc, out_sq=sq, sq_ld=32)
        else:
            kernels.qgemm_packed(attn.view(m, k), p, epilogue="residual", residual=h, out=h, rows=m, out_sq=sq,
                                 sq_ld=32)
        torch.cuda.synchronize()
        outs.append((h.view(torch.int16).clone(), sq.clone(), kc.view(torch.int16).clone()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1].view(torch.int32), outs[1][1].view(torch.int32))
    assert torch.equal(outs[0][2], outs[1][2])


def tiny(name="tiny-target", seed=0, **kw):
    return engine.QuantModel(engine.PRESETS[name], "cuda", seed=seed, max_ctx=256, **kw)


def test_tiny_forward_matches_oracle(cuda):
    model = tiny(sigma=0.08)
    oracle = om.OracleModel.from_device(model)
    oracle.reset(model.max_ctx)
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, model.cfg.vocab, 24).astype(np.int32)
    got = torch_to_bf16_bits(model.logits_for(torch.from_numpy(prompt).to(cuda), 0))
    want = oracle.forward(prompt.tolist(), list(range(24)))
    a, b = bf16.to_f32(got), bf16.to_f32(want)
    assert np.max(np.abs(a - b)) <= 2e-2 * np.max(np.abs(b))
    # greedy picks agree except where the oracle's top-2 margin is inside the tolerance
    top2 = np.sort(b, axis=1)[:, -2:]
    margin = top2[:, 1] - top2[:, 0]
    agree = a.argmax(1) == b.argmax(1)
    assert np.all(agree | (margin < 2e-2 * np.abs(b).max()))
    assert agree.mean() > 0.8


def test_rmsnorm_residual_matches_oracle(cuda):
    rng = np.random.default_rng(11)
    y, h = rand_bits(rng, (5, 640)), rand_bits(rng, (5, 640))
    w = rand_bits(rng, (640,), 0.3)
    ht = bf16_bits_to_torch(h, cuda)
    sq = torch.zeros(32, dtype=torch.float32, device=cuda)
    kernels.rmsnorm_residual(bf16_bits_to_torch(y, cuda), bf16_bits_to_torch(w, cuda), ht, 1e-6, gemma=True,
                             out_sq=sq)
    want = om.residual(h, om.rmsnorm(y, w, 1e-6, True))
    got = torch_to_bf16_bits(ht)
    assert np.mean(got == want) > 0.99
    assert np.max(np.abs(bf16.to_f32(got) - bf16.to_f32(want))) <= 2 ** -6 * np.max(np.abs(bf16.to_f32(want)))
    ref = (bf16.to_f32(got).astype(np.float64) ** 2).sum(axis=1)
    assert np.allclose(sq[:5].cpu().numpy(), ref, rtol=1e-5)


def test_tiny_gemma_forward_matches_oracle(cuda):
    """Gemma-3 shapes: (1 + w) norms, post-attention / post-feedforward norms, sqrt(H) embedding scale, GeGLU,
    sliding-window layers with the local RoPE base and a global layer."""
    model = engine.QuantModel(engine.PRESETS["tiny-gemma"], "cuda", seed=4, sigma=0.08, max_ctx=256)
    assert model.layers[0].post_attn_norm is not None
    oracle = om.OracleModel.from_device(model)
    oracle.reset(model.max_ctx)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, model.cfg.vocab, 28).astype(np.int32)
    got = torch_to_bf16_bits(model.logits_for(torch.from_numpy(prompt).to(cuda), 0))
    want = oracle.forward(prompt.tolist(), list(range(28)))
    a, b = bf16.to_f32(got), bf16.to_f32(want)
    assert np.max(np.abs(a - b)) <= 2e-2 * np.max(np.abs(b))
    top2 = np.sort(b, axis=1)[:, -2:]
    agree = a.argmax(1) == b.argmax(1)
    assert np.all(agree | (top2[:, 1] - top2[:, 0] < 2e-2 * np.abs(b).max()))


def test_gemma_speculation_changes_no_answer(cuda):
    target = engine.QuantModel(engine.PRESETS["tiny-gemma"], "cuda", seed=4, sigma=0.08, max_ctx=256)
    draft = engine.QuantModel(engine.PRESETS["tiny-gemma"], "cuda", seed=6, sigma=0.08, max_ctx=256)
    prompt = torch.randint(0, 1000, (20,), generator=torch.Generator().manual_seed(8)).to(torch.int32).to(cuda)
    solo = engine.QuantModel(engine.PRESETS["tiny-gemma"], "cuda", seed=4, sigma=0.08, max_ctx=256)
    plain = engine.greedy_decode(solo, prompt, 30)
    dec = engine.SpecDecoder(target, draft, k=4)
    dec.start([prompt], max_new=30)
    dec.round()
    dec.capture()
    while not dec.done():
        dec.run_rounds(3)
    assert dec.generated(0, prompt.numel()) == plain


def test_verify_rows_equal_one_row_decodes(cuda):
    model = tiny(sigma=0.08)
    rng = np.random.default_rng(4)
    toks = torch.from_numpy(rng.integers(0, 1000, 30).astype(np.int32)).to(cuda)
    model.prefill(toks[:20])
    many = model.logits_for(toks[20:25], 20).clone()
    one = [model.logits_for(toks[20 + i:21 + i], 20 + i).clone() for i in range(5)]
    for i in range(5):
        assert torch.equal(many[i].view(torch.int16), one[i][0].view(torch.int16)), i


def test_launch_overlap_changes_no_bits(cuda):
    """Programmatic dependent launch only moves when CTAs start: logits are identical with it off."""
    model = tiny(sigma=0.08)
    toks = torch.from_numpy(np.random.default_rng(7).integers(0, 1000, 25).astype(np.int32)).to(cuda)
    model.prefill(toks[:20])
    on = model.logits_for(toks[20:25], 20).clone()
    prev = kernels.set_launch_overlap(False)
    try:
        model.prefill(toks[:20])
        off = model.logits_for(toks[20:25], 20).clone()
    finally:
        kernels.set_launch_overlap(prev)
    assert prev is True
    assert torch.equal(on.view(torch.int16), off.view(torch.int16))


@pytest.mark.parametrize("graph", [False, True])
def test_speculation_changes_no_answer(cuda, graph):
    target = tiny("tiny-target", seed=1, sigma=0.08)
    draft = tiny("tiny-draft", seed=2, sigma=0.08, max_rows=8, max_logit_rows=8)
    prompt = torch.randint(0, 1000, (24,), generator=torch.Generator().manual_seed(5)).to(torch.int32).to(cuda)
    plain = engine.greedy_decode(target, prompt, 40)
    dec = engine.SpecDecoder(target, draft, k=4)
    dec.start([prompt], max_new=40)
    if graph:
        dec.round()
        dec.capture()
    while not dec.done():
        dec.run_rounds(4)
    assert dec.generated(0, prompt.numel()) == plain


def test_identical_draft_has_every_draft_accepted(cuda):
    target = tiny("tiny-target", seed=1, sigma=0.08)
    draft = tiny("tiny-target", seed=1, sigma=0.08)
    prompt = torch.arange(2, 30, dtype=torch.int32, device=cuda)
    dec = engine.SpecDecoder(target, draft, k=4)
    dec.start([prompt], max_new=25)
    dec.run_rounds(5)
    st = dec.read_stats()
    assert st.rounds == 5 and st.tokens == 25 and st.accepted == 20
    assert dec.generated(0, prompt.numel()) == engine.greedy_decode(target, prompt, 25)


def test_batched_speculation_beyond_32_verify_rows(cuda):
    """7 sequences x (k + 1) = 35 verify rows: the qGEMMs take two 32-row chunks; every sequence still gets
    exactly its own greedy tokens."""
    b = 7
    target = tiny("tiny-target", seed=1, sigma=0.08, max_seqs=b, max_rows=40, max_logit_rows=40)
    draft = tiny("tiny-draft", seed=2, sigma=0.08, max_seqs=b, max_rows=16, max_logit_rows=16)
    gen = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, 1000, (n,), generator=gen).to(torch.int32).to(cuda) for n in (5, 9, 30, 17, 3, 22, 11)]
    dec = engine.SpecDecoder(target, draft, k=4, batch=b)
    dec.start(prompts, max_new=16)
    dec.round()
    dec.capture()
    while not dec.done():
        dec.run_rounds(3)
    solo = tiny("tiny-target", seed=1, sigma=0.08)
    for i, p in enumerate(prompts):
        solo_dec = engine.greedy_decode(solo, p, 16)
        assert dec.generated(i, p.numel()) == solo_dec, i


def test_batched_speculation(cuda):
    target = tiny("tiny-target", seed=1, sigma=0.08, max_seqs=3)
    draft = tiny("tiny-draft", seed=2, sigma=0.08, max_seqs=3)
    gen = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, 1000, (n,), generator=gen).to(torch.int32).to(cuda) for n in (10, 31, 5)]
    dec = engine.SpecDecoder(target, draft, k=3, batch=3)
    dec.start(prompts, max_new=20)
    while not dec.done():
        dec.run_rounds(3)
    for b, p in enumerate(prompts):
        solo = tiny("tiny-target", seed=1, sigma=0.08)
        assert dec.generated(b, p.numel()) == engine.greedy_decode(solo, p, 20), b


def test_batched_prefill_writes_the_same_kv(cuda):
    """prefill_many packs several sequences' 32-token chunks into one forward (here 96 rows per forward): the
    caches hold the same bits as prefilling the sequences one at a time."""
    lens = (70, 33, 5, 100)
    gen = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, 1000, (n,), generator=gen).to(torch.int32).to(cuda) for n in lens]
    one = tiny("tiny-target", seed=4, sigma=0.08, max_seqs=4, max_rows=96, max_logit_rows=8)
    many = tiny("tiny-target", seed=4, sigma=0.08, max_seqs=4, max_rows=96, max_logit_rows=8)
    for b, p in enumerate(prompts):
        one.prefill(p, seq=b)
    many.prefill_many(list(enumerate(prompts)))
    torch.cuda.synchronize()
    for b, n in enumerate(lens):
        pages = one.page_table[b]
        for cache in ("k_cache", "v_cache"):
            def slots(model):  # [layers, pages, Hkv, 16, D] -> [layers, slot, Hkv, D]
                t = getattr(model, cache)[:, pages].permute(0, 1, 3, 2, 4)
                return t.reshape(model.cfg.layers, -1, model.cfg.kv_heads, model.cfg.head_dim)[:, :n]
            assert torch.equal(slots(one).view(torch.int16), slots(many).view(torch.int16)), (b, cache)


def test_wide_prefill_chunks_write_the_same_kv(cuda):
    """Prefill in chunks wider than the fused attention's 32 rows per sequence (the q/k norm + RoPE + KV write
    kernel, then the paged attention): the caches and the next token's logits are the same bits as with 32-row
    chunks through the fused attention."""
    gen = torch.Generator().manual_seed(21)
    prompt = torch.randint(0, 1000, (200,), generator=gen).to(torch.int32).to(cuda)
    narrow = tiny("tiny-target", seed=5, sigma=0.08, max_rows=32, max_logit_rows=8)
    wide = tiny("tiny-target", seed=5, sigma=0.08, max_rows=256, max_logit_rows=8)
    for model in (narrow, wide):
        model.prefill(prompt[:-1])
    torch.cuda.synchronize()
    pages = narrow.page_table[0]
    for cache in ("k_cache", "v_cache"):
        def slots(model):  # [layers, pages, Hkv, 16, D] -> [layers, slot, Hkv, D]
            t = getattr(model, cache)[:, pages].permute(0, 1, 3, 2, 4)
            return t.reshape(model.cfg.layers, -1, model.cfg.kv_heads, model.cfg.head_dim)[:, :prompt.numel() - 1]
        assert torch.equal(slots(narrow).view(torch.int16), slots(wide).view(torch.int16)), cache
    last = prompt[-1:].contiguous()
    a = narrow.logits_for(last, prompt.numel() - 1).clone()
    b = wide.logits_for(last, prompt.numel() - 1).clone()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("rows,hq", [(1, 16), (2, 16), (5, 32)])
def test_attention_row_alone_equals_row_in_a_batch(cuda, rows, hq):
    """20 sequences in one launch (160 kv-head groups: the large-batch warp layout and several splits per CTA)
    against each sequence alone (8 groups: the one-sequence layout, one split per CTA): the same bits."""
    rng = np.random.default_rng(rows * hq)
    b, hkv, d, max_pages = 20, 8, 128, 40
    lens = rng.integers(rows + 1, max_pages * 16 - 8, b).tolist()
    table = rng.permutation(b * max_pages).reshape(b, max_pages).astype(np.int32)
    shape = (b * max_pages, hkv, 16, d)
    kc, vc = bf16_bits_to_torch(rand_bits(rng, shape), cuda), bf16_bits_to_torch(rand_bits(rng, shape), cuda)
    q = bf16_bits_to_torch(rand_bits(rng, (b * rows, hq, d)), cuda)
    slots = torch.tensor(np.concatenate([np.arange(n - rows, n) for n in lens]).astype(np.int32), device=cuda)
    tbl = torch.from_numpy(table).to(cuda)
    kw = dict(max_rows_per_seq=rows, max_kv_len=max_pages * 16, scale=d ** -0.5, keys_per_split=128)
    seq_rows = torch.arange(0, b * rows + 1, rows, dtype=torch.int32, device=cuda)
    together = kernels.attention(q, kc, vc, tbl, seq_rows, slots, **kw).clone()
    one_rows = torch.tensor([0, rows], dtype=torch.int32, device=cuda)
    for s in range(b):
        alone = kernels.attention(q[s * rows:(s + 1) * rows].contiguous(), kc, vc, tbl[s:s + 1].contiguous(), one_rows,
                                  slots[s * rows:(s + 1) * rows].contiguous(), **kw)
        assert torch.equal(alone.view(torch.int16), together[s * rows:(s + 1) * rows].view(torch.int16)), s
