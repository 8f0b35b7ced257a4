"""The B200 qGEMM against the oracle (the reference's qmv arithmetic, pinned bit-for-bit to the reference's
own kernel source). Tolerance: max |y - y_ref| / max |y_ref| <= 1e-2 and mean |y - y_ref| / mean |y_ref| <= 1e-3,
both outputs bf16."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from ironmule_b200 import _lib, kernels
from oracle import bf16, qmv, quant

from .gpu_util import MAX_REL, MEAN_REL, bf16_bits_to_torch, case, rel_errors, to_device, torch_to_bf16_bits

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def run(dev, wq, s, b, x, **kw):
    w_t, s_t, b_t, x_t = to_device(wq, s, b, x, dev)
    y = kernels.qgemm(x_t, w_t, s_t, b_t, **kw)
    torch.cuda.synchronize()
    return torch_to_bf16_bits(y)


@pytest.mark.parametrize("m", [1, 5])
@pytest.mark.parametrize("variant,split", [("mma", True), ("mma", False), ("fma", False)])
def test_config1_full_size(cuda, m, variant, split):
    """K=3840, N=15360, W ~ N(0, 0.02), seed 0; M=1 decode and M=5 verify."""
    wq, s, b, x = case(15360, 3840, m, seed=0)
    want = qmv.qmv(wq, s, b, x, vpt=8)
    got = run(cuda, wq, s, b, x, variant=variant, split_k=split)
    mx, mean = rel_errors(got, want)
    assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("qmv_*.npz")), ids=lambda p: p.stem)
def test_reference_golden_vectors(cuda, path):
    d = np.load(path)
    got = run(cuda, d["wq"], d["scales"], d["biases"], d["x"])
    mx, mean = rel_errors(got, d["y_bf0"])
    assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)


@pytest.mark.parametrize("n,k", [(15360, 3840), (2560, 9728), (1024, 1024), (96, 320)])
def test_row_invariance(cuda, n, k):
    """A row's bits do not depend on how many rows share the call (verify == decode)."""
    wq, s, b, x = case(n, k, 32, seed=5)
    full = {m: run(cuda, wq, s, b, x[:m]) for m in (1, 5, 8, 13, 32)}
    for m, y in full.items():
        assert np.array_equal(y, full[32][:m]), m


def test_split_k_is_deterministic_and_within_tolerance(cuda):
    wq, s, b, x = case(2560, 9728, 5, seed=2)
    want = qmv.qmv(wq, s, b, x, vpt=8)
    a = run(cuda, wq, s, b, x, split_k=True)
    c = run(cuda, wq, s, b, x, split_k=True)
    assert np.array_equal(a, c)
    for got in (a, run(cuda, wq, s, b, x, split_k=False)):
        mx, mean = rel_errors(got, want)
        assert mx <= MAX_REL and mean <= MEAN_REL


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 40])
def test_forced_splits(cuda, splits):
    wq, s, b, x = case(640, 5120, 3, seed=9)
    want = qmv.qmv(wq, s, b, x, vpt=8)
    _lib.call("im_qgemm_set_splits", splits)
    try:
        got = run(cuda, wq, s, b, x, split_k=True)
    finally:
        _lib.call("im_qgemm_set_splits", 0)
    mx, mean = rel_errors(got, want)
    assert mx <= MAX_REL and mean <= MEAN_REL


@pytest.mark.parametrize("n,k,m", [(1, 64, 1), (33, 64, 2), (17, 128, 7), (40, 1088, 9), (64, 4096, 32), (8, 15360, 2)])
def test_edge_shapes(cuda, n, k, m):
    wq, s, b, x = case(n, k, m, seed=n + k + m)
    want = qmv.qmv(wq, s, b, x, vpt=8)
    got = run(cuda, wq, s, b, x)
    mx, mean = rel_errors(got, want)
    assert mx <= MAX_REL and mean <= 2 * MEAN_REL  # tiny outputs: a few values dominate the mean


def test_fma_variant_edge_shapes(cuda):
    for n, k, m in [(1, 64, 1), (37, 320, 8), (1000, 2048, 3)]:
        wq, s, b, x = case(n, k, m, seed=n)
        got = run(cuda, wq, s, b, x, variant="fma")
        mx, _ = rel_errors(got, qmv.qmv(wq, s, b, x, vpt=8))
        assert mx <= MAX_REL


def test_residual_epilogue_is_the_rounded_sum(cuda):
    wq, s, b, x = case(1536, 1024, 5, seed=4)
    w_t, s_t, b_t, x_t = to_device(wq, s, b, x, cuda)
    res = torch.randn(5, 1536, device=cuda).to(torch.bfloat16)
    y0 = kernels.qgemm(x_t, w_t, s_t, b_t)
    y1 = kernels.qgemm(x_t, w_t, s_t, b_t, epilogue="residual", residual=res)
    inplace = res.clone()
    kernels.qgemm(x_t, w_t, s_t, b_t, epilogue="residual", residual=inplace, out=inplace)
    want = (res.float() + y0.float()).to(torch.bfloat16)
    assert torch.equal(y1.view(torch.int16), want.view(torch.int16))
    assert torch.equal(inplace.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("epi", ["swiglu", "geglu"])
def test_gated_epilogues(cuda, epi):
    inter, k, m = 96, 512, 5
    rng = np.random.default_rng(11)
    wg = bf16.round_f32(rng.normal(0, 0.05, (inter, k)).astype(np.float32))
    wu = bf16.round_f32(rng.normal(0, 0.05, (inter, k)).astype(np.float32))
    x = bf16.from_f32(rng.normal(0, 1, (m, k)).astype(np.float32))
    inter_w = np.concatenate([np.concatenate([wg[i:i + 16], wu[i:i + 16]]) for i in range(0, inter, 16)])
    wq, s, b = quant.quantize(inter_w)
    got = run(cuda, wq, s, b, x, epilogue=epi)
    plain = bf16.to_f32(run(cuda, wq, s, b, x)).reshape(m, inter // 16, 2, 16)
    g = plain[:, :, 0, :].reshape(m, inter)
    u = plain[:, :, 1, :].reshape(m, inter)
    if epi == "swiglu":
        sig = bf16.round_f32((1.0 / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32))
        act = bf16.round_f32(g * sig)
    else:
        inner = np.float32(0.7978845608028654) * (g + np.float32(0.044715) * g * g * g)
        act = bf16.round_f32((0.5 * g * (1.0 + np.tanh(inner.astype(np.float64)))).astype(np.float32))
    want = bf16.from_f32(act * u)
    diff = np.abs(bf16.to_f32(got) - bf16.to_f32(want))
    ulp = np.abs(bf16.to_f32(want)) * 2.0 ** -7 + 1e-30
    assert np.all(diff <= 2 * ulp)  # transcendental ulps may move one bf16 rounding
    assert np.mean(got == want) > 0.97


def test_gpu_quantiser_matches_the_oracle_bit_for_bit(cuda):
    rng = np.random.default_rng(21)
    w = bf16.round_f32(rng.normal(0, 0.02, (300, 1024)).astype(np.float32))
    w[3, :64] = 0.125  # a constant group
    wq, s, b = quant.quantize(w)
    gq, gs, gb = kernels.quantize(bf16_bits_to_torch(bf16.from_f32(w), cuda))
    assert np.array_equal(gq.cpu().numpy().view(np.uint32), wq)
    assert np.array_equal(torch_to_bf16_bits(gs), s)
    assert np.array_equal(torch_to_bf16_bits(gb), b)


def test_qmv_surface_modules(cuda):
    from ironmule_b200 import qmv_fast_shared, qmv_k3840, qmv_shared

    wq, s, b, x = case(256, 3840, 2, seed=13)
    w_t, s_t, b_t, x_t = to_device(wq, s, b, x, cuda)
    want = qmv.qmv(wq, s, b, x, vpt=8)
    y = qmv_k3840.run(qmv_k3840.K3840, w_t, s_t, b_t, x_t[0:1], 256, 3840)
    assert y.shape == (1, 256)
    a, c = qmv_shared.run_shared(w_t, s_t, b_t, [x_t[0:1], x_t[1:2]], 256)
    assert torch.equal(a.view(torch.int16), y.view(torch.int16))  # shared == alone, bit for bit
    mx, mean = rel_errors(torch_to_bf16_bits(torch.cat([a, c])), want)
    assert mx <= MAX_REL and mean <= MEAN_REL
    wq2, s2, b2, x2 = case(64, 4096, 2, seed=14)
    w2, s2t, b2t, x2t = to_device(wq2, s2, b2, x2, cuda)
    outs = qmv_fast_shared.run_fast(w2, s2t, b2t, [x2t[0:1], x2t[1:2]], 64, 4096)
    mx, _ = rel_errors(torch_to_bf16_bits(torch.cat(outs)), qmv.qmv(wq2, s2, b2, x2, vpt=16))
    assert mx <= MAX_REL


def test_k3840_enable_and_variant_install(cuda):
    from ironmule_b200 import qmv_k3840, qmv_variant
    from ironmule_b200.layers import QuantizedLinear

    wq, s, b, x = case(64, 3840, 1, seed=15)
    w_t, s_t, b_t, x_t = to_device(wq, s, b, x, cuda)
    model = torch.nn.Sequential(QuantizedLinear(w_t, s_t, b_t), torch.nn.Identity())
    with pytest.raises(qmv_k3840.K3840Unsupported):
        qmv_k3840.enable(model, None)
    assert isinstance(model[0], QuantizedLinear)  # refused: untouched
    before = model(x_t.view(1, 1, -1))
    info = qmv_k3840.enable(model, identity="random-init")
    assert info["admitted"] == 1 and isinstance(model[0], qmv_k3840.K3840QuantizedLinear)
    assert torch.equal(model(x_t.view(1, 1, -1)).view(torch.int16), before.view(torch.int16))
    assert qmv_k3840.disable(model) == 1
    gate, report = qmv_variant.install(model, "random-init")
    assert report["admitted"] == 1 and not gate.active
    gate.open("test")
    assert torch.equal(model(x_t.view(1, 1, -1)).view(torch.int16), before.view(torch.int16))
    assert qmv_variant.uninstall(model) == 1


# ---- v4: packed weights --------------------------------------------------------------------------------------
def packed_case(cuda, n, k, m, seed):
    wq, s, b, x = case(n, k, m, seed=seed)
    w_t, s_t, b_t, x_t = to_device(wq, s, b, x, cuda)
    return wq, s, b, x, kernels.Packed(w_t, s_t, b_t), x_t


@pytest.mark.parametrize("n,k,m", [(15360, 3840, 1), (15360, 3840, 5), (6144, 2560, 5), (2560, 9728, 5),
                                   (151936, 2560, 5), (1024, 1024, 2), (96, 256, 13), (50, 768, 32), (4104, 2048, 8)])
def test_packed_kernel_matches_oracle(cuda, n, k, m):
    wq, s, b, x, p, x_t = packed_case(cuda, n, k, m, n + 5 * k + m)
    got = torch_to_bf16_bits(kernels.qgemm_packed(x_t, p))
    mx, mean = rel_errors(got, qmv.qmv(wq, s, b, x, vpt=8))
    assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)


def test_packed_row_invariance(cuda):
    wq, s, b, x, p, x_t = packed_case(cuda, 6144, 2560, 32, 77)
    full = {mm: torch_to_bf16_bits(kernels.qgemm_packed(x_t[:mm].contiguous(), p)) for mm in (1, 5, 8, 13, 32)}
    for mm, y in full.items():
        assert np.array_equal(y, full[32][:mm]), mm


def test_packed_fused_rmsnorm_and_sums_of_squares(cuda):
    """residual epilogue with out_sq, then a GEMM whose prologue normalises from those sums == explicit RMSNorm."""
    from oracle import model as om

    rng = np.random.default_rng(5)
    m, h = 5, 2560
    wq, s, b, x, p_o, x_t = packed_case(cuda, h, 1024, m, 91)       # an "o_proj": K=1024 -> N=h
    res = torch.randn(m, h, device=cuda).to(torch.bfloat16)
    sq = torch.zeros((p_o.tiles, 32), dtype=torch.float32, device=cuda)
    h_new = kernels.qgemm_packed(x_t, p_o, epilogue="residual", residual=res, out_sq=sq)
    hb = torch_to_bf16_bits(h_new)
    want_sq = (bf16.to_f32(hb).astype(np.float64) ** 2).sum(axis=1)
    assert np.allclose(sq.sum(0).cpu().numpy()[:m], want_sq, rtol=1e-5)
    wq2, s2, b2, _, p_qkv, _ = packed_case(cuda, 3072, h, m, 92)
    nw = bf16.from_f32(rng.normal(1, 0.1, h).astype(np.float32))
    nw_t = torch.from_numpy(nw.view(np.int16)).view(torch.bfloat16).to(cuda)
    fused = torch_to_bf16_bits(kernels.qgemm_packed(h_new, p_qkv, norm_sq=sq, norm_parts=p_o.tiles, norm_weight=nw_t))
    normed = om.rmsnorm(hb, nw, 1e-6)
    mx, mean = rel_errors(fused, qmv.qmv(wq2, s2, b2, normed, vpt=8))
    assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)


@pytest.mark.parametrize("m", [33, 70, 160])
def test_packed_many_rows_match_oracle(cuda, m):
    """More than 32 rows go in chunks of 32, each exactly as a call of those rows alone."""
    wq, s, b, x, p, x_t = packed_case(cuda, 2048, 1536, m, 40 + m)
    got = torch_to_bf16_bits(kernels.qgemm_packed(x_t, p))
    mx, mean = rel_errors(got, qmv.qmv(wq, s, b, x, vpt=8))
    assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)
    for r0 in range(0, m, 32):
        alone = torch_to_bf16_bits(kernels.qgemm_packed(x_t[r0:r0 + 32].contiguous(), p))
        assert np.array_equal(alone, got[r0:r0 + 32]), r0
    one = torch_to_bf16_bits(kernels.qgemm_packed(x_t[m - 1:].contiguous(), p))
    assert np.array_equal(one[0], got[m - 1])


def test_packed_many_rows_fused_norm_and_sums_of_squares(cuda):
    """A 70-row residual GEMM's sums of squares (row stride 96) feed a 70-row normalised GEMM: equal to the
    same two calls made 32 rows at a time."""
    rng = np.random.default_rng(8)
    m, h, ld = 70, 1024, 96
    wq, s, b, x, p_o, x_t = packed_case(cuda, h, 512, m, 94)
    res = torch.randn(m, h, device=cuda).to(torch.bfloat16)
    sq = torch.zeros((p_o.tiles, ld), dtype=torch.float32, device=cuda)
    h_new = kernels.qgemm_packed(x_t, p_o, epilogue="residual", residual=res, out_sq=sq, sq_ld=ld)
    want_sq = (bf16.to_f32(torch_to_bf16_bits(h_new)).astype(np.float64) ** 2).sum(axis=1)
    assert np.allclose(sq.sum(0).cpu().numpy()[:m], want_sq, rtol=1e-5)
    _, _, _, _, p2, _ = packed_case(cuda, 768, h, m, 95)
    nw = torch.from_numpy(bf16.from_f32(rng.normal(1, 0.1, h).astype(np.float32)).view(np.int16)).view(torch.bfloat16)
    nw = nw.to(cuda)
    big = kernels.qgemm_packed(h_new, p2, norm_sq=sq, norm_parts=p_o.tiles, norm_weight=nw, sq_ld=ld)
    for r0 in range(0, m, 32):
        n = min(32, m - r0)
        sq_c = sq[:, r0:r0 + n].contiguous()
        part = kernels.qgemm_packed(h_new[r0:r0 + n].contiguous(), p2, norm_sq=sq_c, norm_parts=p_o.tiles,
                                    norm_weight=nw, sq_ld=n)
        assert torch.equal(part.view(torch.int16), big[r0:r0 + n].view(torch.int16)), r0


@pytest.mark.parametrize("epi", ["swiglu", "geglu"])
def test_packed_gated_epilogues(cuda, epi):
    from oracle import model as om

    wq, s, b, x, p, x_t = packed_case(cuda, 2048, 1024, 5, 93)
    plain = torch_to_bf16_bits(kernels.qgemm_packed(x_t, p))
    got = torch_to_bf16_bits(kernels.qgemm_packed(x_t, p, epilogue=epi))
    g = plain.reshape(5, -1, 2, 16)
    want = (om.silu_mul if epi == "swiglu" else om.gelu_mul)(g[:, :, 0, :].reshape(5, -1), g[:, :, 1, :].reshape(5, -1))
    diff = np.abs(bf16.to_f32(got) - bf16.to_f32(want))
    assert np.all(diff <= 2 * (np.abs(bf16.to_f32(want)) * 2.0 ** -7 + 1e-30))


@pytest.mark.parametrize("n,k,m", [(2048, 1536, 64), (2048, 1536, 65), (40, 512, 100), (6144, 2560, 160),
                                   (2560, 9728, 320), (19456, 2560, 128), (1000, 4096, 33)])
def test_tensor_core_rows_equal_32_row_calls(cuda, n, k, m):
    """More than 32 rows on the tcgen05 kernel: every row gets the bits a call of at most 32 rows gives it
    (dead tiles, partial tiles and a ragged last chunk included), and every bounded wait completes."""
    wq, s, b, x, p, x_t = packed_case(cuda, n, k, m, 7 * m + n)
    kernels.qgemm_packed_path(2)
    try:
        ws = kernels.workspace(kernels.qgemm_packed_workspace_bytes(m, n, k), cuda)
        got = torch_to_bf16_bits(kernels.qgemm_packed(x_t, p, ws=ws))
        assert kernels.qgemm_packed_status(ws) == 0
    finally:
        kernels.qgemm_packed_path(0)
    for r0 in range(0, m, 32):
        alone = torch_to_bf16_bits(kernels.qgemm_packed(x_t[r0:r0 + 32].contiguous(), p))
        assert np.array_equal(alone, got[r0:r0 + 32]), r0
    if n * k * m <= 2048 * 1536 * 100:
        mx, mean = rel_errors(got, qmv.qmv(wq, s, b, x, vpt=8))
        assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)


@pytest.mark.parametrize("splits", [1, 3, 16])
def test_tensor_core_forced_splits(cuda, splits):
    """Any K split: the tcgen05 kernel's split-K partials and merge equal the warp-MMA kernel's."""
    wq, s, b, x, p, x_t = packed_case(cuda, 1536, 3072, 96, 50 + splits)
    kernels.qgemm_packed_tune(split_override=splits)
    kernels.qgemm_packed_path(2)
    try:
        got = torch_to_bf16_bits(kernels.qgemm_packed(x_t, p))
        for r0 in range(0, 96, 32):
            alone = torch_to_bf16_bits(kernels.qgemm_packed(x_t[r0:r0 + 32].contiguous(), p))
            assert np.array_equal(alone, got[r0:r0 + 32]), r0
    finally:
        kernels.qgemm_packed_tune()
        kernels.qgemm_packed_path(0)


@pytest.mark.parametrize("epi", ["residual", "swiglu", "geglu"])
def test_tensor_core_epilogues_equal_32_row_calls(cuda, epi):
    """Residual (with sums of squares), SwiGLU and GeGLU epilogues over 150 rows, with the fused RMSNorm
    prologue: the same bits as 32-row calls."""
    rng = np.random.default_rng(17)
    m, n, k, ld = 150, 2048, 1024, 160
    wq, s, b, x, p, x_t = packed_case(cuda, n, k, m, 61)
    tiles_in = 8
    sq_in = torch.from_numpy(rng.uniform(50, 200, (tiles_in, ld)).astype(np.float32)).to(cuda)
    nw = torch.from_numpy(bf16.from_f32(rng.normal(1, 0.1, k).astype(np.float32)).view(np.int16)).view(torch.bfloat16)
    nw = nw.to(cuda)
    kw = dict(norm_sq=sq_in, norm_parts=tiles_in, norm_weight=nw, sq_ld=ld)
    res = torch.randn(m, n, device=cuda).to(torch.bfloat16) if epi == "residual" else None
    sq = torch.zeros((p.tiles, ld), dtype=torch.float32, device=cuda) if epi == "residual" else None
    kernels.qgemm_packed_path(2)
    try:
        big = kernels.qgemm_packed(x_t, p, epilogue=epi, residual=res, out_sq=sq, **kw)
    finally:
        kernels.qgemm_packed_path(0)
    for r0 in range(0, m, 32):
        nr = min(32, m - r0)
        sq_c = torch.zeros((p.tiles, nr), dtype=torch.float32, device=cuda) if sq is not None else None
        part = kernels.qgemm_packed(x_t[r0:r0 + nr].contiguous(), p, epilogue=epi,
                                    residual=None if res is None else res[r0:r0 + nr].contiguous(), out_sq=sq_c,
                                    norm_sq=sq_in[:, r0:r0 + nr].contiguous(), norm_parts=tiles_in, norm_weight=nw,
                                    sq_ld=nr)
        assert torch.equal(part.view(torch.int16), big[r0:r0 + nr].view(torch.int16)), r0
        if sq is not None:
            assert torch.equal(sq_c.view(torch.int32), sq[:, r0:r0 + nr].view(torch.int32)), r0


@pytest.mark.parametrize("m", [1, 2, 5, 13, 32])
def test_tensor_core_path_for_few_rows_gives_the_same_bits(cuda, m):
    """With the tensor-core kernel chosen for every M, calls of up to 32 rows (store, residual + sums of
    squares with the fused RMSNorm, SwiGLU) return exactly the warp-MMA kernel's bits."""
    rng = np.random.default_rng(m)
    n, k, ld = 2048, 2560, 32
    wq, s, b, x, p, x_t = packed_case(cuda, n, k, m, 300 + m)
    sq_in = torch.from_numpy(rng.uniform(50, 200, (4, ld)).astype(np.float32)).to(cuda)
    nw = torch.from_numpy(bf16.from_f32(rng.normal(1, 0.1, k).astype(np.float32)).view(np.int16)).view(torch.bfloat16)
    nw = nw.to(cuda)
    res = torch.randn(m, n, device=cuda).to(torch.bfloat16)
    outs = []
    for path in (0, 2):
        kernels.qgemm_packed_path(path)
        try:
            ws = kernels.workspace(kernels.qgemm_packed_workspace_bytes(m, n, k), cuda)
            sq = torch.zeros((p.tiles, ld), dtype=torch.float32, device=cuda)
            plain = kernels.qgemm_packed(x_t, p, ws=ws)
            resid = kernels.qgemm_packed(x_t, p, epilogue="residual", residual=res, out_sq=sq, sq_ld=ld,
                                         norm_sq=sq_in, norm_parts=4, norm_weight=nw, ws=ws)
            glu = kernels.qgemm_packed(x_t, p, epilogue="swiglu", ws=ws)
            torch.cuda.synchronize()
            if path == 2:
                assert kernels.qgemm_packed_status(ws) == 0
            outs.append([plain.view(torch.int16).clone(), resid.view(torch.int16).clone(),
                         glu.view(torch.int16).clone(), sq[:, :m].view(torch.int32).clone()])
        finally:
            kernels.qgemm_packed_path(0)
    for a, c in zip(*outs):
        assert torch.equal(a, c)


@pytest.mark.parametrize("n,k", [(6144, 2560), (2560, 4096), (2560, 9728), (1024, 3072), (4096, 1024),
                                 (3840, 15360), (5376, 21504), (200, 640)])
@pytest.mark.parametrize("m", [1, 5, 17, 40])
def test_cluster_split_k_equals_the_counter_reduction(cuda, n, k, m):
    """The K splits of a CTA column summed inside a thread-block cluster (through distributed shared memory) give
    the bits of the workspace-and-counter reduction, for every epilogue, with the fused RMSNorm and the sums of
    squares, at one to several 32-row chunks."""
    rng = np.random.default_rng(n + k + m)
    _, _, _, _, p, x_t = packed_case(cuda, n, k, m, n + 3 * k + m)
    res = torch.from_numpy(bf16.from_f32(rng.normal(0, 1, (m, n)).astype(np.float32)).view(np.int16)).view(
        torch.bfloat16).to(cuda)
    parts = 7
    sq_in = torch.from_numpy((rng.random((parts, 64)) * 50 + 1).astype(np.float32)).to(cuda)
    nw = torch.from_numpy(bf16.from_f32(rng.normal(1, 0.1, k).astype(np.float32)).view(np.int16)).view(
        torch.bfloat16).to(cuda)
    outs = {}
    for on in (True, False):
        kernels.qgemm_packed_cluster(on)
        try:
            sq = torch.full((p.tiles, 64), -1.0, dtype=torch.float32, device=cuda)
            store = kernels.qgemm_packed(x_t, p, norm_sq=sq_in, norm_parts=parts, norm_weight=nw, sq_ld=64)
            resid = kernels.qgemm_packed(x_t, p, epilogue="residual", residual=res.clone(), out_sq=sq, sq_ld=64)
            glu = kernels.qgemm_packed(x_t, p, epilogue="swiglu") if n % 32 == 0 else store
            torch.cuda.synchronize()
            outs[on] = [t.view(torch.int16).cpu() for t in (store, resid, glu)] + [sq.cpu()]
        finally:
            kernels.qgemm_packed_cluster(True)
    for a, b in zip(outs[True], outs[False]):
        assert torch.equal(a, b)
