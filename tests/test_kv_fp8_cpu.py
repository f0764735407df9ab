"""fp8 latent KV cache format and its use by the engine, on CPU (fp32 oracle path)."""
import torch

from carbon_b200.config import tiny_config, tiny_v4_config
from carbon_b200.engine.engine import Engine
from carbon_b200.engine.kv_cache import PagedLatentCache
from carbon_b200.models.weights import WeightSource
from carbon_b200.ops.attention import sparse_mla
from carbon_b200.ref import ops as R
from carbon_b200.ref.model import init_weights


def test_latent_fp8_format():
    torch.manual_seed(0)
    x = torch.randn(6, 576) * torch.tensor([0.0, 1e-3, 1.0, 3.0, 100.0, 1e-20])[:, None]
    q = R.quant_latent_fp8(x, 512, 64, True)
    assert q.shape == (6, 656) and R.latent_fp8_row_bytes(512, 64, True) == 656
    assert R.latent_fp8_row_bytes(512, 64, False) == 528
    # layout: values of dims 0..255 | 8 scale bytes + 8 zero | values of dims 256..511 | fp16 RoPE key
    assert bool((q[:, 264:272] == 0).all())                    # scale padding
    assert bool((q[0, 256:264] == 127).all())                  # all-zero atoms: scale 2^0
    y = R.dequant_latent_fp8(q, 512, 64, True)
    assert torch.equal(y[:, 512:], x[:, 512:].half().float())  # RoPE key kept in fp16
    # per atom: |error| <= half an e4m3 step at the atom's scale (3 mantissa bits), relative to the atom's amax
    xa, ya = x[:, :512].reshape(6, 8, 64), y[:, :512].reshape(6, 8, 64)
    amax = xa.abs().amax(-1, keepdim=True)
    big = amax[..., 0] > 1e-10
    assert bool(((ya - xa).abs() <= amax * 2.0 ** -4 + 1e-30)[big].all())
    # a scale byte is the smallest power of two that keeps the atom's amax within 448
    e = q[:, 256:264].float() - 127
    assert bool((amax[..., 0][big] <= 448 * torch.pow(2.0, e[big])).all())
    assert bool((amax[..., 0][big] > 224 * torch.pow(2.0, e[big])).all())


def test_sparse_mla_reads_fp8_rows():
    torch.manual_seed(1)
    q = torch.randn(3, 4, 576)
    kv8 = R.quant_latent_fp8(torch.randn(50, 576), 512, 64, True)
    idx = torch.randint(0, 50, (3, 20), dtype=torch.int32)
    idx[0, 10:] = -1
    a = sparse_mla(q, kv8, idx, 0.1, 512)
    b = sparse_mla(q, R.dequant_latent_fp8(kv8, 512, 64, True), idx, 0.1, 512)
    assert torch.allclose(a, b)


def test_cache_bytes_per_token():
    cfg = tiny_config().replace(kv_lora_rank=512, qk_rope_head_dim=64, n_layers=3)
    bf = PagedLatentCache.bytes_per_token(cfg, 3)
    f8 = PagedLatentCache.bytes_per_token(cfg.replace(kv_fp8=True), 3)
    n_idx = sum(1 for l in range(3) if cfg.has_indexer(l))
    assert bf - f8 == (1152 - 656) * 3
    assert f8 == 656 * 3 + cfg.index_head_dim * 2 * n_idx


def _generate(cfg, w, prompts, n):
    eng = Engine(cfg, device="cpu", source=WeightSource(cfg, state=w), num_pages=16, page_size=16)
    return eng.generate(prompts, max_new_tokens=n, return_logits=True)


def test_engine_fp8_cache_close_to_full_precision():
    """Decode over the fp8 cache stays within fp8 rounding of the full-precision cache (MLA, and latent MQA without
    the indexer: with it, the small hidden-state differences can flip a near-tie of its top-16 in this tiny model,
    which is a different selection, not a numerics error)."""
    for cfg in (tiny_config(), tiny_v4_config().replace(index_n_heads=0)):
        w = init_weights(cfg, seed=0)
        g = torch.Generator().manual_seed(1)
        prompts = [torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist() for _ in range(2)]
        _, h32 = _generate(cfg, w, prompts, 4)
        eng8 = Engine(cfg.replace(kv_fp8=True), device="cpu", source=WeightSource(cfg, state=w), num_pages=16,
                      page_size=16)
        assert eng8.cache.latent[0].dtype == torch.uint8
        # teacher-forced: feed the full-precision run's tokens so both decode the same sequence
        reqs = [eng8.add_request(p) for p in prompts]
        eng8.prefill(reqs)
        toks = [int(h32[0][b].argmax()) for b in range(2)]
        for step in range(1, 4):
            got = eng8.decode(reqs, toks).float()
            exp = h32[step].float()
            rel = ((got - exp).norm() / exp.norm()).item()
            assert rel < 0.05, (cfg.attn_kind, step, rel)
            toks = [int(h32[step][b].argmax()) for b in range(2)]
