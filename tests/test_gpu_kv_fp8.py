"""fp8 latent KV cache on the GPU: the store kernel writes exactly the oracle's bytes, and the fp8 path of the sparse
attention kernel (TMA gathers of the raw row pieces, fp16 expansion in shared memory, fp16 tcgen05 MMAs) matches
fp32 attention over the same dequantised rows."""
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
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


@pytest.mark.parametrize("D", [576, 512])
def test_latent_store_fp8_bitwise(D):
    torch.manual_seed(3)
    n, S, off = 37, 100, 1536
    mla = D == 576
    rb = R.latent_fp8_row_bytes(512, 64, mla)
    rows = (torch.randn(n, D) * torch.rand(n, 1) * 4).to(torch.bfloat16)
    rows[3] = 0
    rows[4, :64] *= 1e-3                           # one atom far smaller than the rest of its row
    big = torch.zeros(n, off + D, dtype=torch.bfloat16)
    big[:, off:] = rows                            # a strided view, like the projection output's latent columns
    slots = torch.randperm(S)[:n].int()
    slots[5] = -1                                  # skipped
    cache = torch.full((S, rb), 0xAB, dtype=torch.uint8, device=DEV)
    _ext().latent_store_fp8(big.to(DEV)[:, off:], slots.to(DEV), cache)
    got = cache.cpu()
    exp = R.quant_latent_fp8(rows.float(), 512, 64, mla)
    written = torch.zeros(S, dtype=torch.bool)
    for i in range(n):
        if slots[i] >= 0:
            assert torch.equal(got[slots[i]], exp[i]), i
            written[slots[i]] = True
    assert bool((got[~written] == 0xAB).all())


@pytest.mark.parametrize("D", [576, 512])
@pytest.mark.parametrize("T,H,K,S", [(3, 128, 300, 1000), (2, 128, 2048, 5000), (40, 64, 100, 300), (16, 16, 64, 200)])
@pytest.mark.parametrize("with_sink", [False, True])
def test_sparse_mla_fp8_rows(D, T, H, K, S, with_sink):
    from carbon_b200.ops.attention import sparse_mla

    torch.manual_seed(8)
    mla = D == 576
    sink = torch.randn(H) * 2 if with_sink else None
    q = (torch.randn(T, H, D) * 0.5).to(torch.bfloat16)
    rows = torch.randn(S, D) * (1 + torch.rand(S, 1) * 3)
    kv8 = R.quant_latent_fp8(rows, 512, 64, mla)
    idx = torch.randint(0, S, (T, K), dtype=torch.int32)
    idx[:, -7:] = -1
    if T > 1:
        idx[1, 5:] = -1
    scale = 192 ** -0.5
    out = sparse_mla(q.to(DEV), kv8.to(DEV), idx.to(DEV), scale, 512, sink=sink.to(DEV) if with_sink else None)
    torch.cuda.synchronize()
    # the kernel takes q in fp16; the oracle dequantises the same cache rows
    ref = sparse_mla(q.half().float(), kv8, idx, scale, 512, sink=sink)
    assert rel_err(out, ref) < 1e-2, rel_err(out, ref)


def test_sparse_mla_fp8_matches_bf16_rows():
    """fp8 rows vs the bf16 kernel on the dequantised rows (bf16-exact where the dequantised value fits bf16)."""
    from carbon_b200.ops.attention import sparse_mla

    torch.manual_seed(9)
    T, H, K, S = 8, 128, 1024, 4000
    q = (torch.randn(T, H, 576) * 0.5).to(torch.bfloat16)
    kv8 = R.quant_latent_fp8(torch.randn(S, 576), 512, 64, True)
    rows = R.dequant_latent_fp8(kv8, 512, 64, True).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(S)[:K] for _ in range(T)]).int()
    a = sparse_mla(q.to(DEV), kv8.to(DEV), idx.to(DEV), 0.07, 512)
    b = sparse_mla(q.to(DEV), rows.to(DEV), idx.to(DEV), 0.07, 512)
    assert rel_err(a, b) < 5e-3, rel_err(a, b)
