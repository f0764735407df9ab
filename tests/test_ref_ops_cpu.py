"""Unit tests of the fp32 oracle's ops (the numerics source of truth for every GPU kernel): each checks a
mathematical property of the op on its own, independent of any kernel."""
import math

import torch

from carbon_b200.config import tiny_v4_config
from carbon_b200.ref import ops as R


def test_sinkhorn_is_doubly_stochastic_and_mhc_ranges():
    g = torch.Generator().manual_seed(0)
    c = R.sinkhorn(torch.randn(64, 4, 4, generator=g), 20, 1e-6)      # unit-scale logits, as mHC produces
    assert torch.allclose(c.sum(-2), torch.ones(64, 4), atol=1e-4)     # the last pass normalises columns exactly
    assert torch.allclose(c.sum(-1), torch.ones(64, 4), atol=1e-3)     # rows converge within 20 passes
    assert (c > 0).all()
    X = torch.randn(16, 4, 256, generator=g)
    fn = torch.randn(24, 4 * 256, generator=g) * 0.02
    pre, post, comb = R.mhc_coeffs(X, fn, torch.randn(24, generator=g), torch.ones(3), 4, 20, 1e-6, 1e-6)
    assert (pre > 0).all() and (pre < 1 + 1e-5).all()
    assert (post > 0).all() and (post < 2).all()
    assert torch.allclose(comb.sum(-2), torch.ones(16, 4), atol=1e-4)


def test_rope_inverse_and_relative_position():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(10, 3, 64, generator=g)
    pos = torch.arange(10) * 7
    y = R.apply_rope(x, pos, 10000.0)
    assert torch.allclose(R.apply_rope(y, pos, 10000.0, inverse=True), x, atol=1e-5)
    # pairs are rotated: norms of (x0, x1) pairs unchanged
    assert torch.allclose(y.view(10, 3, 32, 2).norm(dim=-1), x.view(10, 3, 32, 2).norm(dim=-1), atol=1e-5)
    # <rope(q, i), rope(k, j)> depends on i - j only
    q, k = torch.randn(1, 1, 64, generator=g), torch.randn(1, 1, 64, generator=g)
    s = lambda i, j: float((R.apply_rope(q, torch.tensor([i]), 1e4) * R.apply_rope(k, torch.tensor([j]), 1e4)).sum())
    assert abs(s(5, 2) - s(103, 100)) < 1e-4 and abs(s(5, 2) - s(2, 5)) > 1e-3


def test_fp8_quantisers_bounds_and_scales():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(40, 384, generator=g) * torch.logspace(-4, 3, 40)[:, None]
    q, s = R.quant_fp8_rows(x)
    d = R.dequant_fp8_rows(q, s)
    blk = x.view(40, 3, 128)
    err = (d - x).view(40, 3, 128).abs().amax(-1) / blk.abs().amax(-1)
    assert (err <= 1 / 16 + 1e-6).all()                             # e4m3: 3 mantissa bits, round to nearest
    assert torch.equal(torch.log2(s), torch.round(torch.log2(s)))  # UE8M0: powers of two
    assert (blk.abs().amax(-1) / s <= R.FP8_MAX + 1e-3).all()
    w = torch.randn(300, 260, generator=g)
    qb, sb = R.quant_fp8_blocks(w)
    assert sb.shape == (3, 3) and ((R.dequant_fp8_blocks(qb, sb) - w).abs() <= w.abs().max() / 16).all()
    q32, s32 = R.quant_fp8_rows32(w[:, :256])
    assert s32.dtype == torch.uint8 and s32.shape == (300, 8)
    assert ((R.dequant_fp8_rows32(q32, s32) - w[:, :256]).view(300, 8, 32).abs().amax(-1)
            <= w[:, :256].view(300, 8, 32).abs().amax(-1) / 16 + 1e-6).all()


def test_mxfp4_codec():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(32, 128, generator=g)
    packed, scale = R.quant_mxfp4(w)
    assert packed.shape == (32, 64) and scale.shape == (32, 4)
    d = R.dequant_mxfp4(packed, scale)
    grid = torch.tensor(R.E2M1_VALUES)
    mags = (d / torch.pow(2.0, scale.float() - 127).repeat_interleave(32, 1)).abs()
    assert ((mags[..., None] - grid).abs().min(-1).values < 1e-6).all()          # every value on the e2m1 grid
    assert torch.equal(R.dequant_mxfp4(*R.quant_mxfp4(d)), d)                      # values round-trip exactly


def test_topk_mask_and_router():
    g = torch.Generator().manual_seed(4)
    T = 50
    logits = torch.randn(T, T, generator=g)
    logits[:, 3] = logits[:, 4] = 10.0                                               # a tie
    pos = torch.arange(T)
    m = R.topk_mask(logits, pos, pos, 8)
    assert not (m & ~(pos[None, :] <= pos[:, None])).any()                         # causal only
    assert torch.equal(m.sum(1), torch.clamp(pos + 1, max=8))                      # exactly min(k, #causal) keys
    m1 = R.topk_mask(logits, pos, pos, 1)
    assert m1[10, 3] and not m1[10, 4]                                             # ties go to the lower index
    for sf in ("sigmoid", "sqrtsoftplus", "softmax"):
        w, ids = R.router_topk(torch.randn(20, 16, generator=g), torch.randn(16, generator=g), 4, sf, 2.5, True)
        assert torch.allclose(w.sum(1), torch.full((20,), 2.5), atol=1e-5)
        assert all(len(set(r.tolist())) == 4 for r in ids)


def test_attention_sink_and_indexer_logits():
    g = torch.Generator().manual_seed(5)
    q, k, v = torch.randn(6, 2, 8, generator=g), torch.randn(6, 2, 8, generator=g), torch.randn(6, 2, 8, generator=g)
    pos = torch.arange(6)
    base = R.causal_attention(q, k, v, 0.3, pos, pos)
    assert torch.allclose(R.causal_attention(q, k, v, 0.3, pos, pos, sink=torch.full((2,), -1e30)), base, atol=1e-6)
    with_sink = R.causal_attention(q, k, v, 0.3, pos, pos, sink=torch.zeros(2))
    # a sink only adds denominator mass: the output is the sink-free output scaled by Σp / (Σp + e^sink)
    s = torch.einsum("qhd,khd->hqk", q, k) * 0.3
    s = s.masked_fill(~(pos[None, :] <= pos[:, None])[None], float("-inf"))
    z = torch.logsumexp(s, -1)                                                     # [h, q]
    frac = (torch.exp(z) / (torch.exp(z) + 1.0)).t()[..., None]
    assert torch.allclose(with_sink, base * frac, atol=1e-5)
    qi, ki, wi = torch.randn(5, 3, 16, generator=g), torch.randn(7, 16, generator=g), torch.randn(5, 3, generator=g)
    ref = torch.zeros(5, 7)
    for t in range(5):
        for j in range(7):
            ref[t, j] = sum(wi[t, h] * max(float(qi[t, h] @ ki[j]), 0.0) for h in range(3))
    assert torch.allclose(R.indexer_logits(qi, ki, wi), ref, atol=1e-5)


def test_engram_hash_rows_stay_in_their_columns():
    cfg = tiny_v4_config()
    g = torch.Generator().manual_seed(6)
    window = torch.randint(0, cfg.vocab_size, (200, max(cfg.engram_orders)), generator=g)
    window[:3, 1:] = -1                                                            # sequence start padding
    rows = R.engram_hash_ids(window, cfg.engram_orders, cfg.engram_heads, cfg.engram_primes, cfg.vocab_size)
    lo = 0
    for c, p in enumerate(cfg.engram_primes):
        assert ((rows[:, c] >= lo) & (rows[:, c] < lo + p)).all()
        lo += p
    assert torch.equal(rows, R.engram_hash_ids(window, cfg.engram_orders, cfg.engram_heads, cfg.engram_primes,
                                               cfg.vocab_size))                    # deterministic
    assert rows[:, 0].unique().numel() > 50                                         # spreads over the column
    X = torch.randn(4, 4, 32, generator=g)
    kv = torch.zeros(4, 5 * 32)
    assert torch.allclose(R.engram_gate(X, kv, torch.ones(32), torch.ones(32), 1e-6, 10.0), X)   # zero value: no-op
    assert math.isfinite(float(R.engram_gate(X, torch.randn(4, 160, generator=g), torch.ones(32), torch.ones(32),
                                             1e-6, 10.0).sum()))


def test_yarn_rope_and_group_limited_router():
    from carbon_b200.config import ModelConfig

    base = R.rope_inv_freq(64, 10000.0)
    y = R.rope_inv_freq(64, (10000.0, 40.0, 4096, 32.0, 1.0))
    ratio = y / base
    assert torch.allclose(ratio[:8], torch.ones(8, dtype=ratio.dtype))                # fast dims kept
    assert torch.allclose(ratio[-4:], torch.full((4,), 1 / 40, dtype=ratio.dtype))    # slow dims interpolated
    assert (ratio[1:] <= ratio[:-1] + 1e-12).all()                                     # monotone ramp
    cos, sin = R.rope_cos_sin(torch.arange(5), 64, 10000.0)
    assert torch.allclose(cos ** 2 + sin ** 2, torch.ones_like(cos), atol=1e-6)
    g = torch.Generator().manual_seed(7)
    logits = torch.randn(64, 32, generator=g)
    bias = torch.randn(32, generator=g) * 0.1
    w, ids = R.router_topk(logits, bias, 6, "sigmoid", 2.5, True, n_groups=8, topk_groups=3)
    assert all(len({int(e) // 4 for e in row}) <= 3 for row in ids)                    # experts from <= 3 groups
    assert torch.allclose(w.sum(1), torch.full((64,), 2.5), atol=1e-5)
    hf = {"vocab_size": 129280, "hidden_size": 7168, "intermediate_size": 18432, "moe_intermediate_size": 2048,
          "num_hidden_layers": 61, "num_attention_heads": 128, "n_shared_experts": 1, "n_routed_experts": 256,
          "routed_scaling_factor": 2.5, "kv_lora_rank": 512, "q_lora_rank": 1536, "qk_rope_head_dim": 64,
          "v_head_dim": 128, "qk_nope_head_dim": 128, "n_group": 8, "topk_group": 4, "num_experts_per_tok": 8,
          "first_k_dense_replace": 3, "norm_topk_prob": True, "scoring_func": "sigmoid", "rms_norm_eps": 1e-6,
          "rope_theta": 10000, "max_position_embeddings": 163840,
          "rope_scaling": {"beta_fast": 32, "beta_slow": 1, "factor": 40, "mscale": 1.0, "mscale_all_dim": 1.0,
                           "original_max_position_embeddings": 4096, "type": "yarn"}}
    c = ModelConfig.from_hf(hf)
    assert c.plain_residual and c.n_groups == 8 and c.topk_groups == 4 and c.n_dense_layers == 3
    assert abs(c.softmax_scale - 192 ** -0.5 * (0.1 * math.log(40) + 1) ** 2) < 1e-12
    assert c.index_topk == 0 and c.rope[1] == 40.0
