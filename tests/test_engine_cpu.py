"""The tiny model served by the engine (paged latent cache, absorbed decode, DSA top-k) matches
the naive full-recompute fp32 oracle within 1e-4 on every prefill and greedy-decode step."""
import torch

from carbon_b200.config import tiny_config, tiny_v4_config
from carbon_b200.engine.engine import Engine
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref.model import RefModel, init_weights


import pytest


@pytest.mark.parametrize("variant", ["v3", "v3_plain", "v3_hf", "v41_features", "v4_latent", "v4_latent_nodsa", "v4_image",
                                     "v4_late", "v3_sparse_prefill", "v41_sparse_prefill"])
def test_tiny_engine_matches_oracle(variant):
    """v41_features: DSA selection computed by index-source layers 1 and 3 only (layer 0 dense, layer 2 reuses
    layer 1's selection) and per-head attention sinks.  v4_latent: the V4 attention layout (latent MQA with output
    RoPE rotated back, grouped low-rank output projection, sliding window 16 + top-16 over older keys, sinks,
    sqrt-softplus router, Engram on layer 1); v4_latent_nodsa: the same without the indexer (window-only attention);
    v4_image: image tokens (every 5th prompt token) rank experts with the image bias and skip the Engram update;
    v4_late: bounded late-layer replay (layer 2 runs only each prompt's last 24 tokens, window-only); v3_plain: no
    hyper-connections (one residual stream, x + f(norm(x)), as in DeepSeek-V3 / V3.2 checkpoints); *_sparse_prefill:
    the 64-token prompts run the long-prompt MLA prefill (absorbed sparse attention over each query's top-k cached
    rows) instead of the dense masked kernel."""
    cfg = tiny_config()
    if variant == "v3_plain":
        cfg = cfg.replace(hc_mult=0, n_layers=3, n_dense_layers=1)
    elif variant == "v3_hf":                # + group-limited routing and YaRN RoPE (DeepSeek-V3's config.json)
        cfg = cfg.replace(hc_mult=0, n_groups=4, topk_groups=2, rope_factor=8.0, rope_orig_max=32)
    elif variant == "v41_features":
        cfg = cfg.replace(n_layers=4, index_sources=(1, 3), attn_sink=True)
    elif variant == "v4_latent":
        cfg = tiny_v4_config().replace(n_layers=3, index_sources=(1,))
    elif variant == "v4_latent_nodsa":
        cfg = tiny_v4_config().replace(index_n_heads=0)
    elif variant == "v4_image":
        cfg = tiny_v4_config().replace(image_token_id=7)
    elif variant == "v4_late":
        cfg = tiny_v4_config().replace(n_layers=3, late_layer_start=2, late_replay=24)
    elif variant == "v3_sparse_prefill":
        cfg = cfg.replace(sparse_prefill_min=40)
    elif variant == "v41_sparse_prefill":
        cfg = cfg.replace(n_layers=4, index_sources=(1, 3), attn_sink=True, sparse_prefill_min=40)
    w = init_weights(cfg, seed=0)
    ref = RefModel(cfg, w)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (64,), generator=g) for _ in range(2)]
    if cfg.image_token_id >= 0:
        for p in prompts:
            p[::5] = cfg.image_token_id
    eng = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=16, page_size=16)
    outs, hist = eng.generate([p.tolist() for p in prompts], max_new_tokens=16, return_logits=True)
    for b, p in enumerate(prompts):
        toks, ref_logits = ref.greedy(p, 16)
        assert outs[b] == toks
        for step in range(16):
            got = hist[step][b]
            exp = ref_logits[step]
            err = (got - exp).abs().max().item()
            assert err < 1e-4, (b, step, err)
    assert eng.cache.alloc.num_free() == 16 - 1   # all request pages returned (page 0 is the scratch page)


def test_fake_quant_mxfp4_matches_codec():
    """The indexer's arithmetic fp4 rounding equals the MXFP4 encode/decode pair (scales, ties, signs, zeros)."""
    from carbon_b200.ref import ops as R

    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 128, generator=g) * torch.logspace(-3, 3, 64)[:, None]
    x[0, :32] = 0.0
    x[1, :8] = torch.tensor([0.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.75, -5.0])
    assert torch.equal(R.fake_quant_mxfp4(x), R.dequant_mxfp4(*R.quant_mxfp4(x)))


@pytest.mark.parametrize("variant", ["v3", "v4_latent"])
def test_chunked_prefill_matches_oracle(variant):
    """Chunked prefill (17 tokens per step, every token attending to its request's cached keys) followed by greedy
    decode gives the oracle's tokens and logits; so does continuing a request whose prompt was partly prefilled."""
    cfg = tiny_config() if variant == "v3" else tiny_v4_config().replace(n_layers=3, index_sources=(1,))
    w = init_weights(cfg, seed=0)
    ref = RefModel(cfg, w)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (60, 23)]
    eng = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=16, page_size=16)
    reqs = [eng.add_request(p.tolist()) for p in prompts]
    logits = eng.prefill_chunked(reqs, chunk=17)
    for b, p in enumerate(prompts):
        toks, ref_logits = ref.greedy(p, 4)
        assert (logits[b] - ref_logits[0]).abs().max() < 1e-4
        cur = int(torch.argmax(logits[b]))
        got = [cur]
        r = reqs[b]
        for step in range(3):
            lg = eng.decode([r], [cur])[0]
            assert (lg - ref_logits[step + 1]).abs().max() < 1e-4, (b, step)
            cur = int(torch.argmax(lg))
            got.append(cur)
        assert got == toks[:4]


def test_head_bmm_decode_kernel_eligibility():
    """The decode shapes of the absorbed MLA take the swap-AB per-head kernel (query absorption with its RoPE tail,
    value un-absorption, V4's grouped wo_a); shapes its tensor maps cannot serve fall back to the grouped GEMM."""
    from carbon_b200.models.deepseek import _head_bmm_direct

    bf = torch.bfloat16
    q = torch.zeros(32, 128, 192, dtype=bf)
    w_uk = torch.zeros(128, 512, 128, dtype=bf)
    assert _head_bmm_direct(q, w_uk, 64, torch.float16)
    assert _head_bmm_direct(torch.zeros(32, 128, 512, dtype=bf), torch.zeros(128, 128, 512, dtype=bf), 0, bf)
    assert _head_bmm_direct(torch.zeros(256, 8, 512, dtype=bf), torch.zeros(8, 1024, 512, dtype=bf), 0, bf)
    assert not _head_bmm_direct(torch.zeros(257, 128, 192, dtype=bf), w_uk, 64, bf)        # more than 256 tokens
    assert not _head_bmm_direct(q, torch.zeros(128, 500, 128, dtype=bf), 64, bf)           # N not a multiple of 128
    assert not _head_bmm_direct(q.float(), w_uk, 64, bf)                                   # fp32 operand
    assert not _head_bmm_direct(q[:, :, 1:], w_uk, 60, bf)                                 # unaligned rows / tail
    assert not _head_bmm_direct(q, w_uk, 64, torch.float32)                                # fp32 output
