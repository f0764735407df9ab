"""GPU numerics of every CUDA kernel against the plain-PyTorch fp32 oracle of the same op."""
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


# ----------------------------------------------------------------------------------------------------------------------
# quantisation
# ----------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("M,K", [(1, 128), (37, 512), (200, 1536), (128, 7168), (5, 576 - 64)])
def test_act_quant_matches_oracle(M, K):
    from carbon_b200.ops.quant import quant_act, unpack_sf

    torch.manual_seed(0)
    x = (torch.randn(M, K) * 3).to(torch.bfloat16)
    q, sf = quant_act(x.to(DEV))
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    s = unpack_sf(sf.cpu(), M, K)
    assert torch.equal(s, s_ref)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))


def test_act_quant_gather_rows():
    from carbon_b200.ops.quant import quant_act, unpack_sf

    x = torch.randn(10, 256).to(torch.bfloat16)
    src = torch.tensor([3, -1, 0, 9, 9, -1, 2], dtype=torch.int32)
    q, sf = quant_act(x.to(DEV), src_rows=src.to(DEV))
    xs = torch.where((src >= 0)[:, None], x.float()[src.clamp(min=0).long()], torch.zeros(()))
    q_ref, s_ref = R.quant_fp8_rows(xs)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))
    assert torch.equal(unpack_sf(sf.cpu(), 7, 256), s_ref)


# ----------------------------------------------------------------------------------------------------------------------
# GEMMs
# ----------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 384, 512), (1, 256, 1024), (300, 576, 7168),
                                   (1000, 1536, 2048), (77, 4096, 640)])
def test_fp8_gemm_dense(M, N, K):
    from carbon_b200.ops.gemm import fp8_gemm
    from carbon_b200.ops.quant import Fp8Weight, quant_act

    torch.manual_seed(1)
    x = torch.randn(M, K).to(torch.bfloat16)
    w = torch.randn(N, K) * 0.02
    W = Fp8Weight.from_float(w)
    Wd = Fp8Weight(W.q.to(DEV), W.sf.to(DEV), W.scale.to(DEV))
    q, sf = quant_act(x.to(DEV))
    out = fp8_gemm(q, sf, Wd, out_dtype=torch.float32)
    torch.cuda.synchronize()
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    ref = R.fp8_gemm(q_ref, s_ref, W.q, W.scale)
    assert rel_err(out, ref) < 1e-5, rel_err(out, ref)
    out_bf = fp8_gemm(q, sf, Wd)
    assert rel_err(out_bf, ref) < 5e-3


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (200, 256, 512), (1, 128, 192), (513, 640, 1024)])
def test_bf16_gemm(M, N, K):
    from carbon_b200.ops.gemm import bf16_gemm

    torch.manual_seed(2)
    a = torch.randn(M, K).to(torch.bfloat16)
    b = torch.randn(N, K).to(torch.bfloat16)
    out = bf16_gemm(a.to(DEV), b.to(DEV), out_dtype=torch.float32)
    ref = a.float() @ b.float().t()
    assert rel_err(out, ref) < 1e-5


def test_bf16_gemm_strided_a():
    from carbon_b200.ops.gemm import bf16_gemm

    a_full = torch.randn(64, 384).to(torch.bfloat16).to(DEV)
    a = a_full[:, 128:320]                       # row stride 384 elements, 192 wide
    b = torch.randn(256, 192).to(torch.bfloat16).to(DEV)
    out = bf16_gemm(a, b, out_dtype=torch.float32)
    assert rel_err(out, a.float() @ b.float().t()) < 1e-5


def _grouped_case(T=300, E=8, k=2, D=512, N=256, seed=3):
    from carbon_b200.ops.core import MoeLayout

    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    lay = MoeLayout(ids.to(DEV), E)
    return ids, lay


def test_moe_layout_and_grouped_fp8_gemm():
    from carbon_b200.ops.gemm import fp8_gemm
    from carbon_b200.ops.quant import Fp8Weight, quant_act

    T, E, k, K, N = 300, 8, 2, 512, 256
    ids, lay = _grouped_case(T, E, k, K, N)
    torch.cuda.synchronize()
    slot_pos = lay.slot_pos.cpu()
    row_src = lay.row_src.cpu()
    mbe = lay.m_block_expert.cpu()
    nb = int(lay.num_blocks.cpu())
    counts = torch.bincount(ids.view(-1).long(), minlength=E)
    assert nb == int(((counts + 127) // 128).sum())
    for t in range(T):
        for j in range(k):
            p = int(slot_pos[t, j])
            assert row_src[p] == t and mbe[p // 128] == ids[t, j]
    x = torch.randn(T, K).to(torch.bfloat16)
    w = torch.randn(E, N, K) * 0.02
    Ws = [Fp8Weight.from_float(w[e]) for e in range(E)]
    Wq = torch.cat([W.q for W in Ws]).to(DEV)
    from carbon_b200.ops.quant import pack_sf
    Wsf = pack_sf(torch.cat([W.scale.repeat_interleave(128, 0)[:N] for W in Ws])).to(DEV)
    Wall = Fp8Weight(Wq, Wsf, None)
    q, sf = quant_act(x.to(DEV), src_rows=lay.row_src)
    out = fp8_gemm(q, sf, Wall, out_dtype=torch.float32, m_block_expert=lay.m_block_expert,
                   num_m_blocks=lay.num_blocks, n_per_group=N)
    torch.cuda.synchronize()
    out = out.cpu()
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    xd = R.dequant_fp8_rows(q_ref, s_ref)
    for t in range(0, T, 7):
        for j in range(k):
            e = int(ids[t, j])
            ref = xd[t] @ Ws[e].dequant().t()
            got = out[int(slot_pos[t, j])]
            assert rel_err(got, ref) < 1e-5


def test_grouped_swiglu_fp8_epilogue():
    from carbon_b200.ops.gemm import fp8_gemm_swiglu, interleave_gate_up
    from carbon_b200.ops.quant import Fp8Weight, pack_sf, quant_act, unpack_sf

    T, E, k, K, I = 200, 4, 2, 256, 256
    ids, lay = _grouped_case(T, E, k, K, 2 * I, seed=4)
    x = torch.randn(T, K).to(torch.bfloat16)
    w1 = torch.randn(E, I, K) * 0.05
    w3 = torch.randn(E, I, K) * 0.05
    Ws = [Fp8Weight.from_float(interleave_gate_up(w1[e], w3[e])) for e in range(E)]
    Wall = Fp8Weight(torch.cat([W.q for W in Ws]).to(DEV),
                     pack_sf(torch.cat([W.scale.repeat_interleave(128, 0)[:2 * I] for W in Ws])).to(DEV), None)
    q, sf = quant_act(x.to(DEV), src_rows=lay.row_src)
    act, act_sf = fp8_gemm_swiglu(q, sf, Wall, 0.0, lay.m_block_expert, lay.num_blocks, 2 * I)
    torch.cuda.synchronize()
    rows = lay.rows
    a_s = unpack_sf(act_sf.cpu(), rows, I)
    act_d = act.cpu().float() * a_s.repeat_interleave(128, 1)
    q_ref, s_ref = R.quant_fp8_rows(x.float())
    xd = R.dequant_fp8_rows(q_ref, s_ref)
    slot_pos = lay.slot_pos.cpu()
    for t in range(0, T, 5):
        for j in range(k):
            e = int(ids[t, j])
            wd = Ws[e].dequant()
            gu = xd[t] @ wd.t()
            gu = gu.view(-1, 2, 128)
            ref = R.swiglu(gu[:, 0].reshape(-1), gu[:, 1].reshape(-1))
            got = act_d[int(slot_pos[t, j])]
            assert rel_err(got, ref) < 0.04, rel_err(got, ref)


# ----------------------------------------------------------------------------------------------------------------------
# small ops
# ----------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("M,D", [(3, 256), (65, 1536), (17, 7168)])
def test_rms_norm(M, D):
    from carbon_b200.ops.core import rms_norm
    from carbon_b200.ops.quant import unpack_sf

    x = torch.randn(M, D).to(torch.bfloat16)
    w = torch.rand(D) + 0.5
    y, (q, sf) = rms_norm(x.to(DEV), w.to(DEV), 1e-6, want_bf16=True, want_fp8=True)
    ref = R.rms_norm(x.float(), w, 1e-6)
    assert rel_err(y, ref) < 4e-3
    deq = q.cpu().float() * unpack_sf(sf.cpu(), M, D).repeat_interleave(128, 1)
    assert rel_err(deq, ref) < 0.04


def test_rope_matches_oracle():
    from carbon_b200.ops.core import rope_, rope_table

    T, H, d, off = 9, 3, 64, 128
    x = torch.randn(T, H, off + d).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32)
    tab = rope_table(4096, d, 10000.0, DEV)
    y = x.to(DEV)
    rope_(y, off, d, tab, pos.to(DEV))
    ref = R.apply_rope(x[..., off:].float(), pos, 10000.0)
    assert rel_err(y[..., off:], ref) < 4e-3
    assert torch.equal(y[..., :off].cpu(), x[..., :off])
    rope_(y, off, d, tab, pos.to(DEV), inverse=True)
    assert rel_err(y[..., off:], x[..., off:].float()) < 8e-3


@pytest.mark.parametrize("score", ["sigmoid", "sqrtsoftplus", "softmax"])
@pytest.mark.parametrize("E,k", [(8, 2), (256, 8), (384, 6)])
def test_router_topk(score, E, k):
    from carbon_b200.ops.core import router_topk

    T = 97
    logits = torch.randn(T, E)
    bias = torch.randn(E) * 0.5
    w, ids = router_topk(logits.to(DEV), bias.to(DEV), k, score, 2.5, True)
    w_ref, ids_ref = R.router_topk(logits, bias, k, score, 2.5, True)
    assert torch.equal(ids.cpu(), ids_ref)
    assert rel_err(w, w_ref) < 1e-5


@pytest.mark.parametrize("E,k,ng,tg", [(256, 8, 8, 4), (64, 6, 4, 2), (160, 6, 5, 3)])
def test_router_group_limited(E, k, ng, tg):
    """Group-limited routing (DeepSeek-V3: 8 groups, the 4 best by their top-2 sum) in the router kernel."""
    from carbon_b200.ops.core import router_topk

    torch.manual_seed(4)
    T = 211
    logits = torch.randn(T, E)
    bias = torch.randn(E) * 0.5
    w, ids = router_topk(logits.to(DEV), bias.to(DEV), k, "sigmoid", 2.5, True, n_groups=ng, topk_groups=tg)
    w_ref, ids_ref = R.router_topk(logits, bias, k, "sigmoid", 2.5, True, ng, tg)
    assert torch.equal(ids.cpu(), ids_ref)
    assert rel_err(w, w_ref) < 1e-5


def test_router_ties_prefer_lower_id():
    from carbon_b200.ops.core import router_topk

    logits = torch.zeros(4, 64)
    w, ids = router_topk(logits.to(DEV), None, 6, "sigmoid", 1.0, True)
    assert torch.equal(ids.cpu(), torch.arange(6, dtype=torch.int32).expand(4, 6))


def test_moe_combine():
    from carbon_b200.ops.core import moe_combine

    T, k, D = 33, 3, 256
    Y = torch.randn(200, D).to(torch.bfloat16)
    pos = torch.randint(-1, 200, (T, k), dtype=torch.int32)
    w = torch.rand(T, k)
    add = torch.randn(T, D).to(torch.bfloat16)
    out = moe_combine(Y.to(DEV), w.to(DEV), pos.to(DEV), add.to(DEV), T)
    ref = moe_combine(Y, w, pos, add, T)
    assert rel_err(out, ref) < 4e-3


def test_mhc_kernels():
    from carbon_b200.ops.core import split_hi_lo
    from carbon_b200.ops.gemm import bf16_gemm

    T, D, hc = 50, 256, 4
    X = torch.randn(T, hc, D).to(torch.bfloat16)
    fn = torch.randn(24, hc * D) * 0.02
    base = torch.randn(24) * 0.1
    scale = torch.tensor([1.0, 0.9, 1.1])
    pre_r, post_r, comb_r = R.mhc_coeffs(X.float(), fn, base, scale, hc, 20, 1e-6, 1e-6)
    Xd = X.to(DEV)
    fhl = split_hi_lo(fn)
    fpad = torch.zeros(64, hc * D, dtype=torch.bfloat16)
    fpad[:48] = fhl
    mix = bf16_gemm(Xd.view(T, -1), fpad.to(DEV), out_dtype=torch.float32)
    ss = torch.empty(T, device=DEV)
    _ext().row_sumsq(Xd.view(T, -1), ss)
    pre = torch.empty(T, 4, device=DEV); post = torch.empty(T, 4, device=DEV); comb = torch.empty(T, 16, device=DEV)
    _ext().mhc_coeffs(mix, ss, base.to(DEV), scale.to(DEV), hc * D, 20, 1e-6, 1e-6, pre, post, comb)
    assert rel_err(pre, pre_r) < 1e-4 and rel_err(post, post_r) < 1e-4
    assert rel_err(comb.view(T, 4, 4), comb_r) < 1e-4
    w = torch.rand(D) + 0.5
    y = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    _ext().mhc_pre_norm(Xd, pre_r.to(DEV), w.to(DEV), 1e-6, y, None, None, None)
    y_ref = R.rms_norm(R.mhc_pre_mix(X.float(), pre_r), w, 1e-6)
    assert rel_err(y, y_ref) < 5e-3
    out = torch.randn(T, D).to(torch.bfloat16)
    Xn = torch.empty_like(Xd)
    ss2 = torch.empty(T, device=DEV)
    _ext().mhc_post_mix(Xd, out.to(DEV), post_r.to(DEV), comb_r.reshape(T, 16).to(DEV), Xn, ss2)
    Xn_ref = R.mhc_post_mix(X.float(), out.float(), post_r, comb_r)
    assert rel_err(Xn, Xn_ref) < 5e-3
    assert rel_err(ss2, Xn.float().pow(2).sum((1, 2))) < 1e-4


@pytest.mark.parametrize("T,rows", [(1, 48), (32, 48), (64, 16)])
def test_mhc_stats_small_matches_fp32(T, rows):
    """Decode-sized mHC statistics (CUDA-core kernel) against fp32 math on the same bf16 inputs."""
    K = 4 * 7168
    X = torch.randn(T, K).to(torch.bfloat16)
    fn = (torch.randn(rows, K) * 0.02).to(torch.bfloat16)
    out = torch.empty(T, rows, device=DEV)
    _ext().mhc_stats_small(X.to(DEV), fn.to(DEV), rows, out)
    assert rel_err(out, X.float() @ fn.float().t()) < 1e-5


# ----------------------------------------------------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("version", [1, 2, 3])
@pytest.mark.parametrize("lens,masked,qscale", [([128], False, 1.0), ([300, 77, 5], False, 1.0), ([513], True, 1.0),
                                                ([200, 260], True, 1.0), ([1000, 700], False, 4.0),
                                                ([1300], True, 3.0), ([256, 384, 129], False, 1.0)])
def test_attn_prefill(lens, masked, qscale, version):
    _check_attn_prefill(lens, masked, qscale, version, with_sink=False)


@pytest.mark.parametrize("version", [1, 2, 3])
@pytest.mark.parametrize("lens,masked", [([300, 77], False), ([513], True)])
def test_attn_prefill_with_sink(lens, masked, version):
    _check_attn_prefill(lens, masked, 1.0, version, with_sink=True)


def _check_attn_prefill(lens, masked, qscale, version, with_sink):
    from carbon_b200.ops.attention import prefill_attention

    torch.manual_seed(5)
    H = 4
    sink = torch.randn(H) * 2 if with_sink else None
    T = sum(lens)
    q = (torch.randn(T, H, 192) * qscale).to(torch.bfloat16)     # qscale > 1: row maxima keep growing (rescales)
    k = torch.randn(T, H, 192).to(torch.bfloat16)
    k[..., 128:] = torch.randn(T, 1, 64).to(torch.bfloat16)       # MLA: one RoPE key shared by all heads
    v = torch.randn(T, H, 128).to(torch.bfloat16)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    masks = None
    if masked:
        masks = [torch.rand(n, n) < 0.3 for n in lens]
        for m in masks:
            m.fill_diagonal_(True)
    out = prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), cu, 192 ** -0.5,
                            [m.to(DEV) for m in masks] if masks else None, version=version,
                            sink=sink.to(DEV) if with_sink else None)
    torch.cuda.synchronize()
    for b in range(len(lens)):
        s, t = cu[b], cu[b + 1]
        pos = torch.arange(t - s)
        ref = R.causal_attention(q[s:t], k[s:t], v[s:t], 192 ** -0.5, pos, pos, masks[b] if masks else None,
                                 sink=sink)
        assert rel_err(out[s:t], ref) < 1e-2, (b, rel_err(out[s:t], ref))


@pytest.mark.parametrize("n,H", [(300, 64), (700, 32)])
def test_indexer_logits_gemm(n, H):
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


@pytest.mark.parametrize("n,k", [(100, 128), (300, 64), (1000, 256), (2000, 512)])
def test_topk_mask_exact(n, k):
    from carbon_b200.ops.attention import unpack_key_mask

    torch.manual_seed(7)
    logits = torch.randn(n, n)
    logits[:, ::7] = 0.5            # ties, resolved toward the lower key index
    W = (n + 31) // 32
    mask = torch.zeros(n, W, dtype=torch.int32, device=DEV)
    _ext().topk_mask(logits.to(DEV), n, k, mask, 0)
    got = unpack_key_mask(mask.cpu(), [0, n])[0]
    pos = torch.arange(n)
    exp = R.topk_mask(logits, pos, pos, k)
    assert torch.equal(got, exp)


@pytest.mark.parametrize("T,H,K,S,splits_override", [(3, 128, 300, 1000, None), (16, 16, 64, 200, None),
                                                      (2, 128, 2048, 5000, None), (40, 64, 100, 300, None)])
@pytest.mark.parametrize("with_sink", [False, True])
def test_sparse_mla_decode(T, H, K, S, splits_override, with_sink):
    """with_sink: per-head attention-sink logits (single-split normalisation and the split combine)."""
    from carbon_b200.ops.attention import sparse_mla

    torch.manual_seed(8)
    sink = torch.randn(H) * 2 if with_sink else None
    q = (torch.randn(T, H, 576) * 0.5).to(torch.bfloat16)
    kv = torch.randn(S, 576).to(torch.bfloat16)
    idx = torch.randint(0, S, (T, K), dtype=torch.int32)
    idx[:, -7:] = -1                       # padding
    if T > 1:
        idx[1, 5:] = -1                    # a short row
    scale = 192 ** -0.5
    out = sparse_mla(q.to(DEV), kv.to(DEV), idx.to(DEV), scale, 512, sink=sink.to(DEV) if with_sink else None)
    torch.cuda.synchronize()
    ref = sparse_mla(q.float(), kv.float(), idx, scale, 512, sink=sink)
    assert rel_err(out, ref) < 1e-2, rel_err(out, ref)


@pytest.mark.parametrize("M,N,K,splits", [(32, 64, 28672, 0), (5, 48, 4096, 7), (130, 128, 8192, 4)])
def test_bf16_gemm_split_k(M, N, K, splits):
    from carbon_b200.ops.gemm import bf16_gemm

    torch.manual_seed(9)
    a = torch.randn(M, K).to(torch.bfloat16)
    b = torch.randn(N, K).to(torch.bfloat16)
    out = bf16_gemm(a.to(DEV), b.to(DEV), out_dtype=torch.float32, k_splits=splits)
    assert rel_err(out, a.float() @ b.float().t()) < 1e-5


@pytest.mark.parametrize("T,L,k", [(4, 300, 128), (3, 5000, 2048), (2, 100, 256)])
def test_indexer_topk_decode(T, L, k):
    from carbon_b200.ops.attention import indexer_topk

    torch.manual_seed(12)
    H, S = 64, 6000
    q = torch.randn(T, H, 128).to(torch.bfloat16)
    w = torch.randn(T, H) * 0.1
    kc = torch.randn(S, 128).to(torch.bfloat16)
    slots = torch.stack([torch.randperm(S)[:L] for _ in range(T)]).int()
    n = torch.tensor([L - 7 * i for i in range(T)], dtype=torch.int32)
    for i in range(T):
        slots[i, int(n[i]):] = -1
    got = indexer_topk(q.to(DEV), w.to(DEV), kc.to(DEV), slots.to(DEV), n.to(DEV), k).cpu()
    ref = indexer_topk(q, w, kc, slots, n, k)
    for i in range(T):
        assert set(got[i][got[i] >= 0].tolist()) == set(ref[i][ref[i] >= 0].tolist()), i


@pytest.mark.parametrize("T,L,H", [(3, 700, 64), (2, 129, 16), (5, 4100, 32), (1, 300, 128)])
def test_indexer_decode_logits_tcgen05(T, L, H):
    """tcgen05 decode indexer: Σ_h w·relu(q·k) over gathered key rows vs fp32; -inf past n_keys and at slot -1."""
    torch.manual_seed(3)
    S = 9000
    q = torch.randn(T, H, 128).to(torch.bfloat16)
    w = torch.randn(T, H) * 0.1
    kc = torch.randn(S, 128).to(torch.bfloat16)
    slots = torch.stack([torch.randperm(S)[:L] for _ in range(T)]).int()
    n = torch.tensor([max(1, L - 131 * i) for i in range(T)], dtype=torch.int32)
    slots[:, 5] = -1                                        # a hole inside the valid range
    out = torch.empty(T, L, device=DEV)
    _ext().indexer_decode_logits(q.to(DEV), w.to(DEV), kc.to(DEV), slots.to(DEV), n.to(DEV), out)
    out = out.cpu()
    for t in range(T):
        nt = int(n[t])
        s = slots[t, :nt].clamp(min=0).long()
        ref = ((q[t].float() @ kc[s].float().t()).clamp(min=0) * w[t][:, None]).sum(0)
        valid = slots[t, :nt] >= 0
        assert torch.isinf(out[t, :nt][~valid]).all() and torch.isinf(out[t, nt:]).all()
        assert rel_err(out[t, :nt][valid], ref[valid]) < 1e-5, t


@pytest.mark.parametrize("T", [1, 5, 32, 64])
@pytest.mark.parametrize("with_out", [False, True])
@pytest.mark.parametrize("D", [1024, 7168])
def test_mhc_boundary_fused_matches_separate_kernels(T, with_out, D):
    """The fused decode boundary (post-mix + statistics + coefficients + pre-norm, one cluster launch) against the
    four separate kernels it replaces."""
    from carbon_b200.models.deepseek import make_hc, mhc_mix
    from carbon_b200.ops.quant import empty_sf, unpack_sf

    e = _ext()
    torch.manual_seed(21 + T)
    hp = make_hc(torch.randn(24, 4 * D) * 0.02, torch.randn(24) * 0.5, torch.rand(3) + 0.5, torch.device(DEV))
    w = (torch.rand(D) + 0.5).to(DEV)
    X0 = torch.randn(T, 4, D).to(torch.bfloat16).to(DEV)
    out = torch.randn(T, D).to(torch.bfloat16).to(DEV) if with_out else None
    post_in = (torch.rand(T, 4) * 2).to(DEV)
    comb_in = torch.softmax(torch.randn(T, 4, 4), -1).to(DEV)
    iters, hc_eps, eps = 20, 1e-6, 1e-6
    # separate kernels
    Xa = X0.clone()
    if with_out:
        sumsq = torch.empty(T, device=DEV)
        e.mhc_post_mix(Xa, out, post_in, comb_in.view(-1, 16), Xa, sumsq)
    else:
        sumsq = Xa.float().pow(2).sum(dim=(1, 2))
    mix = mhc_mix(Xa.view(T, 4 * D), hp.fn)
    pre_a, post_a, comb_a = torch.empty(T, 4, device=DEV), torch.empty(T, 4, device=DEV), torch.empty(T, 4, 4, device=DEV)
    e.mhc_coeffs(mix, sumsq, hp.base, hp.scale, 4 * D, iters, hc_eps, eps, pre_a, post_a, comb_a)
    ya = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    qa = torch.empty(T, D, dtype=torch.float8_e4m3fn, device=DEV)
    sfa = empty_sf(T, D, DEV)
    e.mhc_pre_norm(Xa, pre_a, w, eps, ya, qa, sfa, None)
    # fused
    Xb = X0.clone()
    yb = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    qb = torch.empty(T, D, dtype=torch.float8_e4m3fn, device=DEV)
    sfb = empty_sf(T, D, DEV)
    pre_b, post_b, comb_b = torch.empty(T, 4, device=DEV), torch.empty(T, 4, device=DEV), torch.empty(T, 4, 4, device=DEV)
    e.mhc_boundary_small(Xb, out, post_in if with_out else None, comb_in if with_out else None, hp.fn, hp.base,
                         hp.scale, iters, hc_eps, eps, w, yb, qb, sfb, pre_b, post_b, comb_b)
    torch.cuda.synchronize()
    # the same post-mix arithmetic: equal up to a rare last-bit difference from FMA contraction
    assert (Xa != Xb).float().mean().item() < 1e-3
    assert rel_err(Xb, Xa) < 1e-3
    for a, b in ((pre_a, pre_b), (post_a, post_b), (comb_a, comb_b)):
        assert torch.allclose(a, b, rtol=1e-4, atol=1e-6), (a - b).abs().max().item()
    assert rel_err(yb, ya) < 2e-3, rel_err(yb, ya)
    da = qa.float().cpu() * unpack_sf(sfa.cpu(), T, D).repeat_interleave(128, 1)
    db = qb.float().cpu() * unpack_sf(sfb.cpu(), T, D).repeat_interleave(128, 1)
    assert rel_err(db, da) < 2e-2, rel_err(db, da)



@pytest.mark.parametrize("T", [1, 32, 300])
def test_indexer_kw_post_vs_torch(T):
    """Indexer key LayerNorm + RoPE and scaled head weights in one kernel, against the separate torch / RoPE ops."""
    import torch.nn.functional as F

    from carbon_b200.ops import core as C

    torch.manual_seed(41)
    Di, Hi, dr = 128, 64, 64
    kw = (torch.randn(T, Di + Hi) * 3).to(DEV)
    lw, lb = (torch.rand(Di) + 0.5).to(DEV), (torch.randn(Di) * 0.1).to(DEV)
    table = C.rope_table(4096, dr, 10000.0, DEV)
    pos = torch.randint(0, 4096, (T,), dtype=torch.int32, device=DEV)
    k = torch.empty(T, Di, dtype=torch.bfloat16, device=DEV)
    w = torch.empty(T, Hi, device=DEV)
    _ext().indexer_kw_post(kw, Di, lw, lb, 1e-6, table, pos, dr, 0.01, k, w)
    ref_k = F.layer_norm(kw[:, :Di], (Di,), lw, lb, 1e-6).to(torch.bfloat16).view(T, 1, Di)
    C.rope_(ref_k, 0, dr, table, pos)
    torch.cuda.synchronize()
    assert torch.allclose(w, kw[:, Di:] * 0.01)
    assert rel_err(k, ref_k.view(T, Di)) < 5e-3, rel_err(k, ref_k.view(T, Di))


# ----------------------------------------------------------------------------------------------------------------------
# per-head matmul of decode batches (swap-AB tcgen05)
# ----------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("T,H,N,K,xw,tail,odt", [
    (32, 128, 512, 128, 192, 64, torch.float16),     # MLA query absorption: q [T, H, 192] -> [q_nope W_uk | q_rope]
    (32, 128, 512, 128, 192, 64, torch.bfloat16),
    (32, 128, 128, 512, 512, 0, torch.bfloat16),     # value un-absorption: o_lat [T, H, 512] -> [T, H, 128]
    (1, 16, 512, 128, 192, 64, torch.bfloat16),
    (200, 16, 512, 128, 192, 64, torch.float16),
    (256, 16, 128, 512, 512, 0, torch.bfloat16),
    (7, 8, 256, 192, 256, 0, torch.bfloat16),
])
def test_head_bmm_decode_vs_fp32(T, H, N, K, xw, tail, odt):
    from carbon_b200.models.deepseek import _head_bmm_direct, head_bmm

    torch.manual_seed(0)
    x = torch.randn(T, H, xw, device=DEV).to(torch.bfloat16)
    w = (torch.randn(H, N, K, device=DEV) * 0.05).to(torch.bfloat16)
    assert _head_bmm_direct(x, w, tail, odt)
    launches = _ext().launch_count()
    out = head_bmm(x, w, tail=tail, out_dtype=odt)
    torch.cuda.synchronize()
    assert _ext().launch_count() == launches + 1                   # one launch, no staging copies
    ref = torch.einsum("thk,hnk->thn", x[..., :K].float(), w.float())
    assert out.shape == (T, H, N + tail) and out.dtype == odt
    assert rel_err(out[..., :N], ref) < 4e-3
    if tail:
        assert torch.equal(out[..., N:].float().cpu(), x[..., K:K + tail].to(odt).float().cpu())


# ----------------------------------------------------------------------------------------------------------------------
# EP receive-buffer layout (the count matrix of every source rank -> offsets and this rank's expert blocks)
# ----------------------------------------------------------------------------------------------------------------------
def _layout_ref(cnt, world, my_rank, max_blocks, align):
    E = cnt.shape[1]
    El = E // world
    my_off = [0] * E
    mbe = [-1] * max_blocks
    total = 0
    for o in range(world):
        acc = b = 0
        for el in range(El):
            e = o * El + el
            n = int(cnt[:, e].sum())
            my_off[e] = acc + int(cnt[:my_rank, e].sum())
            nb = (n + align - 1) // align * (align // 128)
            if o == my_rank:
                for _ in range(nb):
                    if b < max_blocks:
                        mbe[b] = el
                        b += 1
            acc += nb * 128
        if o == my_rank:
            total = b
    return my_off, mbe, total


@pytest.mark.parametrize("world,E,align,max_blocks", [(2, 256, 128, 300), (8, 256, 128, 64), (8, 256, 256, 40),
                                                      (4, 384, 128, 7)])
def test_moe_layout_vs_python(world, E, align, max_blocks):
    torch.manual_seed(world * 7 + E)
    cnt = torch.randint(0, 40, (world, E), dtype=torch.int32)
    cnt[cnt < 12] = 0                                              # experts nobody routes to
    for my_rank in range(world):
        off = torch.empty(E, dtype=torch.int32, device=DEV)
        mbe = torch.empty(max_blocks, dtype=torch.int32, device=DEV)
        nb = torch.empty(1, dtype=torch.int32, device=DEV)
        _ext().moe_layout(cnt.to(DEV), world, my_rank, off, mbe, nb, align)
        r_off, r_mbe, r_total = _layout_ref(cnt, world, my_rank, max_blocks, align)
        assert off.cpu().tolist() == r_off
        assert mbe.cpu().tolist() == r_mbe
        assert int(nb.item()) == r_total
