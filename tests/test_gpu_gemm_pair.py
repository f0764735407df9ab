"""CTA-pair (cta_group::2) 256x256-tile GEMM: numerics against the fp32 oracle and against the 128-row kernel.

Covers dense bf16 output (ragged M and N, short and long K, several tiles per persistent CTA pair so both
accumulator stages and their shared TMEM columns are exercised), expert-grouped SwiGLU + down projection on a
256-row-aligned layout, the o_proj scatter epilogue, and the DSA indexer epilogue.
"""
import pytest
import torch

from carbon_b200.ref import ops as R

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ext():
    from carbon_b200.ops._ext import ext

    return ext()


def rel_err(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _weight(N, K, seed, scale=0.02):
    from carbon_b200.ops.quant import Fp8Weight

    g = torch.Generator().manual_seed(seed)
    W = Fp8Weight.from_float(torch.randn(N, K, generator=g) * scale)
    return W, Fp8Weight(W.q.to(DEV), W.sf.to(DEV), W.scale.to(DEV))


@pytest.mark.parametrize("M,N,K", [(512, 256, 512), (1000, 1536, 2048), (777, 576, 7168), (4096, 4096, 1024),
                                   (1024, 512, 128), (2048, 7168, 1536)])
def test_pair_gemm_dense_matches_oracle_and_single_cta(M, N, K):
    from carbon_b200.ops.gemm import fp8_gemm
    from carbon_b200.ops.quant import quant_act

    torch.manual_seed(11)
    x = torch.randn(M, K).to(torch.bfloat16)
    W, Wd = _weight(N, K, 12)
    q, sf = quant_act(x.to(DEV))
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out_pair = fp8_gemm(q, sf, Wd, pair=1, status=status)
    out_single = fp8_gemm(q, sf, Wd, pair=0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    ref = R.fp8_gemm(q_ref, s_ref, W.q, W.scale)
    assert rel_err(out_pair, ref) < 5e-3, rel_err(out_pair, ref)
    # same products in the same K order: the two kernels agree to bf16 rounding
    assert rel_err(out_pair, out_single) < 1e-3


def test_pair_gemm_repeated_launches_are_deterministic():
    from carbon_b200.ops.gemm import fp8_gemm
    from carbon_b200.ops.quant import quant_act

    x = torch.randn(3000, 2048, device=DEV).to(torch.bfloat16)
    _, Wd = _weight(3072, 2048, 13)
    q, sf = quant_act(x)
    a = fp8_gemm(q, sf, Wd, pair=1)
    for _ in range(3):
        b = fp8_gemm(q, sf, Wd, pair=1)
        assert torch.equal(a, b)


def _grouped(T, E, k, seed, align):
    from carbon_b200.ops.core import MoeLayout

    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    return ids, MoeLayout(ids.to(DEV), E, align=align)


def test_layout_align_256_blocks():
    T, E, k = 700, 6, 2
    ids, lay = _grouped(T, E, k, 21, 256)
    torch.cuda.synchronize()
    counts = torch.bincount(ids.view(-1).long(), minlength=E)
    nb = int(lay.num_blocks.cpu())
    assert nb == int(((counts + 255) // 256).sum()) * 2
    mbe = lay.m_block_expert.cpu()
    assert all(int(mbe[2 * i]) == int(mbe[2 * i + 1]) for i in range(nb // 2))
    slot = lay.slot_pos.cpu()
    for t in range(T):
        for j in range(k):
            assert int(mbe[int(slot[t, j]) // 128]) == int(ids[t, j])


@pytest.mark.parametrize("T,align,mode", [(900, 256, 1), (40, 128, 2), (3, 128, 2)])
def test_pair_grouped_swiglu_and_down_projection(T, align, mode):
    """mode 1: CTA-pair tiles on 256-row segments; mode 2: decode weight streaming (fp32 up-projection + row-wise
    SwiGLU/requant, padding rows never written)."""
    from carbon_b200.ops.gemm import fp8_gemm, fp8_gemm_swiglu, interleave_gate_up
    from carbon_b200.ops.quant import Fp8Weight, pack_sf, quant_act, unpack_sf

    E, k, K, I, D = 4, 2, 512, 256, 512
    ids, lay = _grouped(T, E, k, 22, align)
    assert lay.pair == mode
    g = torch.Generator().manual_seed(23)
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    w1 = torch.randn(E, I, K, generator=g) * 0.05
    w3 = torch.randn(E, I, K, generator=g) * 0.05
    w2 = torch.randn(E, D, I, generator=g) * 0.05
    W13 = [Fp8Weight.from_float(interleave_gate_up(w1[e], w3[e])) for e in range(E)]
    W2 = [Fp8Weight.from_float(w2[e]) for e in range(E)]

    def stack(Ws, rows):
        return Fp8Weight(torch.cat([W.q for W in Ws]).to(DEV),
                         pack_sf(torch.cat([W.scale.repeat_interleave(128, 0)[:rows] for W in Ws])).to(DEV), None)

    q, sf = quant_act(x.to(DEV), src_rows=lay.row_src)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    act, act_sf = fp8_gemm_swiglu(q, sf, stack(W13, 2 * I), 0.0, lay.m_block_expert, lay.num_blocks, 2 * I,
                                  status=status, pair=mode, row_valid=lay.row_src)
    y = fp8_gemm(act, act_sf, stack(W2, D), m_block_expert=lay.m_block_expert, num_m_blocks=lay.num_blocks,
                 n_per_group=D, status=status, pair=mode, row_valid=lay.row_src)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    rows = lay.rows
    act_d = act.cpu().float() * unpack_sf(act_sf.cpu(), rows, I).repeat_interleave(128, 1)
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    xd = R.dequant_fp8_rows(q_ref, s_ref)
    slot = lay.slot_pos.cpu()
    y = y.cpu()
    for t in range(0, T, 7 if T > 50 else 1):
        for j in range(k):
            e = int(ids[t, j])
            gu = (xd[t] @ W13[e].dequant().t()).view(-1, 2, 128)
            ref_act = R.swiglu(gu[:, 0].reshape(-1), gu[:, 1].reshape(-1))
            p = int(slot[t, j])
            assert rel_err(act_d[p], ref_act) < 0.05      # fp8 e4m3 requantisation of the activations
            ref_y = act_d[p] @ W2[e].dequant().t()
            assert rel_err(y[p], ref_y) < 1e-2


def test_pair_scatter_epilogue_single_rank():
    """o_proj GEMM -> row scatter with one rank: the rows land in slot 0 of this rank's own buffer."""
    from carbon_b200.ops.quant import quant_act

    M, N, K = 1100, 1024, 2048
    x = torch.randn(M, K, device=DEV).to(torch.bfloat16)
    W, Wd = _weight(N, K, 31)
    q, sf = quant_act(x)
    buf = torch.zeros(M, N, dtype=torch.bfloat16, device=DEV)
    ptrs = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=DEV)
    bounds = torch.tensor([0, M], dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    _ext().gemm_fp8_scatter(q, sf, Wd.q, Wd.sf, ptrs, bounds, 0, M, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    from carbon_b200.ops.gemm import fp8_gemm

    ref = fp8_gemm(q, sf, Wd, pair=0)
    assert rel_err(buf, ref) < 1e-3


@pytest.mark.parametrize("n,H", [(300, 64), (1100, 64), (700, 32), (530, 16), (260, 128)])
def test_pair_indexer_logits(n, H):
    torch.manual_seed(6)
    q = torch.randn(n, H, 128).to(torch.bfloat16)
    k = torch.randn(n, 128).to(torch.bfloat16)
    w = torch.randn(n, H)
    ldo = (n + 3) // 4 * 4
    out = torch.full((n, ldo), float("nan"), device=DEV)
    _ext().indexer_logits(k.to(DEV), q.to(DEV), w.to(DEV), out, True)
    ref = R.indexer_logits(q.float(), k.float(), w)
    causal = torch.ones(n, n, dtype=torch.bool).tril_()
    got = out[:, :n].cpu()
    assert rel_err(got[causal], ref[causal]) < 1e-5


@pytest.mark.parametrize("M,N,K", [(32, 7168, 16384), (1, 256, 7168), (100, 1536, 7168), (7, 576, 7168),
                                   (64, 128, 7168)])
def test_small_m_split_k(M, N, K):
    """Decode-sized GEMMs split K over CTAs (fp32 partial slabs, ordered reduction)."""
    from carbon_b200.ops.gemm import fp8_gemm
    from carbon_b200.ops.quant import quant_act

    torch.manual_seed(41)
    x = torch.randn(M, K).to(torch.bfloat16)
    W, Wd = _weight(N, K, 42)
    q, sf = quant_act(x.to(DEV))
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    ref = R.fp8_gemm(q_ref, s_ref, W.q, W.scale)
    out32 = fp8_gemm(q, sf, Wd, out_dtype=torch.float32)
    out16 = fp8_gemm(q, sf, Wd)
    again = fp8_gemm(q, sf, Wd)
    torch.cuda.synchronize()
    assert rel_err(out32, ref) < 1e-5, rel_err(out32, ref)
    assert rel_err(out16, ref) < 5e-3
    assert torch.equal(out16, again)          # the split reduction is ordered: bitwise repeatable


@pytest.mark.parametrize("M", [1, 32, 130])
def test_small_m_split_k_swiglu(M):
    from carbon_b200.ops.gemm import fp8_gemm_swiglu, interleave_gate_up
    from carbon_b200.ops.quant import Fp8Weight, quant_act, unpack_sf

    K, I = 7168, 512
    g = torch.Generator().manual_seed(43)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w1 = torch.randn(I, K, generator=g) * 0.02
    w3 = torch.randn(I, K, generator=g) * 0.02
    W = Fp8Weight.from_float(interleave_gate_up(w1, w3))
    Wd = Fp8Weight(W.q.to(DEV), W.sf.to(DEV), W.scale.to(DEV))
    q, sf = quant_act(x.to(DEV))
    act, act_sf = fp8_gemm_swiglu(q, sf, Wd, 0.0)
    torch.cuda.synchronize()
    act_d = act.cpu().float() * unpack_sf(act_sf.cpu(), M, I).repeat_interleave(128, 1)
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    gu = (R.dequant_fp8_rows(q_ref, s_ref) @ W.dequant().t()).view(M, -1, 2, 128)
    ref = R.swiglu(gu[:, :, 0].reshape(M, -1), gu[:, :, 1].reshape(M, -1))
    assert rel_err(act_d, ref) < 0.04, rel_err(act_d, ref)


def test_gather_fp8_rows_matches_gather_quantise():
    """Quantise-once + row gather (MoE dispatch) == gather + quantise, bitwise on every row with a source (-1 rows
    are expert-segment padding, which the gather leaves unwritten)."""
    from carbon_b200.ops.quant import gather_rows_fp8, quant_act, unpack_sf

    x = torch.randn(300, 7168, device=DEV).to(torch.bfloat16)
    src = torch.randint(-1, 300, (1024,), dtype=torch.int32, device=DEV)
    q1, sf1 = quant_act(x, src_rows=src)
    tq, tsf = quant_act(x)
    q2, sf2 = gather_rows_fp8(tq, tsf, src)
    torch.cuda.synchronize()
    ok = (src >= 0).cpu()
    assert torch.equal(q1.view(torch.uint8).cpu()[ok], q2.view(torch.uint8).cpu()[ok])
    assert torch.equal(unpack_sf(sf1.cpu(), 1024, 7168)[ok], unpack_sf(sf2.cpu(), 1024, 7168)[ok])


@pytest.mark.parametrize("H", [64, 32])
def test_indexer_logits_fp8(H):
    """Block-scaled fp8 indexer logits (keys / queries in e4m3 with 1x128 UE8M0 scales) against the fp32 oracle of
    the same fp8-rounded inputs, on the causal entries."""
    from carbon_b200.ops.quant import quant_act
    from carbon_b200.ref import ops as R

    torch.manual_seed(0)
    L, Tq, Di = 700, 700, 128
    k = torch.randn(L, Di).to(torch.bfloat16)
    q = torch.randn(Tq, H, Di).to(torch.bfloat16)
    w = torch.randn(Tq, H) * (H ** -0.5) * (Di ** -0.5)
    kq, ksf = quant_act(k.cuda())
    qq, qsf = quant_act(q.reshape(Tq * H, Di).cuda())
    out = torch.empty(Tq, (L + 3) // 4 * 4, device="cuda")
    _ext().indexer_logits_fp8(kq, ksf, qq, qsf, H, w.cuda(), out, True)
    kf, qf = R.fake_quant_fp8_rows(k.float()), R.fake_quant_fp8_rows(q.float())
    ref = R.indexer_logits(qf, kf, w)
    causal = torch.arange(L)[None, :] <= torch.arange(Tq)[:, None]
    got = out[:, :L].cpu()          # tiles wholly above the diagonal are skipped (the top-k reads causal keys only)
    assert ((got[causal] - ref[causal]).norm() / ref[causal].norm()).item() < 1e-3
