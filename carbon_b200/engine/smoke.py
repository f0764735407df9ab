"""One tiny serving step on cuda:0.

First three of the hot kernels run once on small inputs and are checked against fp32 PyTorch math: the CTA-pair
block-scaled fp8 GEMM, the MLA prefill attention and the absorbed sparse decode attention.  They run before the
model's weight init (which issues hundreds of small PyTorch launches), so a launch trace of the smoke run lists this
package's kernels first.  Then a 2-layer (dense + MoE) model at the reduced-width "small" shape, which keeps every
full-size kernel constraint, prefills a dense and a DSA-sparse prompt and decodes with CUDA graphs.
"""
from __future__ import annotations

import torch

from ..config import small_gpu_config
from ..models.weights import WeightSource
from .engine import Engine


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-9)).item()


def kernel_checks(dev="cuda") -> dict:
    """fp8 GEMM, prefill attention and sparse decode attention vs fp32 math (relative Frobenius error)."""
    from ..ops.attention import mla_prefill, sparse_mla
    from ..ops.gemm import fp8_gemm
    from ..ops.quant import dequant_act, quant_act, quantize_weight

    g = torch.Generator(device=dev).manual_seed(0)
    res = {}
    # CTA-pair GEMM (M >= 512 takes the 256x256 pair tiles)
    x = torch.randn(512, 1024, device=dev, generator=g).to(torch.bfloat16)
    w = quantize_weight(torch.randn(512, 1024, device=dev, generator=g) * 0.02)
    xq, xsf = quant_act(x)
    y = fp8_gemm(xq, xsf, w)
    res["gemm"] = _rel(y, dequant_act(xq, xsf).to(dev) @ w.dequant().to(dev).t())
    # MLA prefill attention, one 256-token causal sequence, 4 heads (192 / 128 dims)
    T, H = 256, 4
    q = torch.randn(T, H, 192, device=dev, generator=g).to(torch.bfloat16)
    kvb = torch.randn(T, H, 256, device=dev, generator=g).to(torch.bfloat16)
    kpe = torch.randn(T, 64, device=dev, generator=g).to(torch.bfloat16)
    o = mla_prefill(q, kvb, kpe, [0, T], 192 ** -0.5)
    k = torch.cat([kvb[..., :128].float(), kpe.float()[:, None].expand(T, H, 64)], -1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k) * 192 ** -0.5
    s = s.masked_fill(torch.ones(T, T, device=dev, dtype=torch.bool).triu(1), float("-inf"))
    res["prefill_attn"] = _rel(o, torch.einsum("hqk,khd->qhd", s.softmax(-1), kvb[..., 128:].float()))
    # absorbed sparse decode attention, 4 tokens x 128 heads x 256 selected latent rows
    qd = (torch.randn(4, 128, 576, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    kv = torch.randn(1024, 576, device=dev, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, 1024, (4, 256), device=dev, dtype=torch.int32, generator=g)
    od = sparse_mla(qd, kv, idx, 192 ** -0.5, 512)
    rows = kv.float()[idx.long()]                                           # [4, 256, 576]
    p = (torch.einsum("thd,tkd->thk", qd.float(), rows) * 192 ** -0.5).softmax(-1)
    res["sparse_mla"] = _rel(od, torch.einsum("thk,tkd->thd", p, rows[..., :512]))
    bad = {k: v for k, v in res.items() if not v < 2e-2}
    assert not bad, f"kernel check failed: {bad}"
    return res


def run_smoke(n_layers: int = 2) -> dict:
    assert torch.cuda.is_available(), "smoke() needs a GPU"
    from ..ops._ext import ext

    ext()  # fail loudly if the extension is missing
    checks = kernel_checks()
    cfg = small_gpu_config().replace(n_layers=n_layers)
    eng = Engine(cfg, device="cuda", source=WeightSource(cfg, seed=0), num_pages=64, page_size=64, cuda_graphs=True,
                 graph_buckets=(2, 4))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (300, 40)]
    outs, hist = eng.generate(prompts, max_new_tokens=4, return_logits=True)
    torch.cuda.synchronize()
    for h in hist:
        assert torch.isfinite(h).all(), "non-finite logits"
    info = {"kernel_checks": checks, "tokens": outs, "logit_absmax": float(max(h.abs().max() for h in hist))}
    print("smoke ok", info)
    return info
