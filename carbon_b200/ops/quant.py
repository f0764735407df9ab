"""fp8 e4m3 quantisation with UE8M0 (power-of-two) block scales.

Formats (shared by every kernel):

* Activations: 1×128 blocks per row.  Weights: 128×128 blocks.
* Scales are stored as **SF tiles**: for each 512-wide K group ``kg`` and each 128-row block ``rb``, 128 int32
  words; word ``l*4 + j`` packs the four UE8M0 bytes (one per 128-wide K block, byte = k-block % 4) of row
  ``32*j + l`` of the block.  This is the order in which ``tcgen05.cp 32x128b.warpx4`` moves 128 rows of
  scale factors into tensor memory, so the GEMM copies tiles without reshuffling them.

The reference keeps its scales as column-major UE8M0 words and runs a 128×4 swizzle kernel before every
block-scaled MMA (``king_v10/bundle_v9/cuda_swizzle.py:15``); producing the MMA order directly removes that pass.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from ..ref import ops as R
from ._ext import ext


def sf_words(rows: int, k: int) -> int:
    return ((k + 511) // 512) * ((rows + 127) // 128) * 128


def empty_sf(rows: int, k: int, device) -> torch.Tensor:
    return torch.empty(sf_words(rows, k), dtype=torch.int32, device=device)


# ---------------------------------------------------------------------------------------------------------------------
# SF tile <-> plain fp32 scale matrices (host-side helpers; also used by tests)
# ---------------------------------------------------------------------------------------------------------------------
def _exp_bytes(scale: torch.Tensor) -> torch.Tensor:
    """fp32 power-of-two scales -> UE8M0 biased exponent bytes (uint8)."""
    e = torch.log2(scale.float()).round().to(torch.int32) + 127
    return e.clamp(0, 254).to(torch.uint8)


def pack_sf(scale_rows: torch.Tensor) -> torch.Tensor:
    """scale_rows: fp32 [rows, kblocks] (one scale per row and 128-wide K block) -> SF tiles (int32)."""
    rows, kblocks = scale_rows.shape
    rb = (rows + 127) // 128
    kg = (kblocks + 3) // 4
    b = torch.full((rb * 128, kg * 4), 127, dtype=torch.uint8, device=scale_rows.device)
    b[:rows, :kblocks] = _exp_bytes(scale_rows)
    # [rb, j(4), l(32), kg, byte(4)] -> [kg, rb, l, j, byte]
    t = b.view(rb, 4, 32, kg, 4).permute(3, 0, 2, 1, 4).contiguous()
    return t.view(torch.int32).reshape(-1)


def unpack_sf(sf: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """SF tiles -> fp32 [rows, ceil(k/128)]."""
    rb = (rows + 127) // 128
    kg = (k + 511) // 512
    kblocks = (k + 127) // 128
    b = sf[: kg * rb * 128].contiguous().view(torch.uint8).view(kg, rb, 32, 4, 4)  # kg, rb, l, j, byte
    b = b.permute(1, 3, 2, 0, 4).reshape(rb * 128, kg * 4)                       # rows, kblocks
    return torch.exp2(b[:rows, :kblocks].float() - 127.0)


@dataclass
class Fp8Weight:
    """A block-scaled fp8 weight [N, K] with its SF tiles (per-row copies of the 128×128 block scales)."""

    q: torch.Tensor          # float8_e4m3fn [N, K]
    sf: torch.Tensor         # int32 SF tiles for N rows
    scale: torch.Tensor      # fp32 [ceil(N/128), ceil(K/128)] (checkpoint form, `weight_scale_inv`)

    @property
    def shape(self):
        return self.q.shape

    def dequant(self) -> torch.Tensor:
        return R.dequant_fp8_blocks(self.q.float().to(torch.float8_e4m3fn) if self.q.dtype != torch.float8_e4m3fn
                                    else self.q, self.scale)

    @staticmethod
    def from_float(w: torch.Tensor) -> "Fp8Weight":
        q, s = R.quant_fp8_blocks(w.float())
        return Fp8Weight.from_quantized(q.to(w.device), s.to(w.device))

    @staticmethod
    def from_quantized(q: torch.Tensor, scale: torch.Tensor) -> "Fp8Weight":
        N, K = q.shape
        rows = scale.repeat_interleave(128, dim=0)[:N]          # [N, kblocks]
        return Fp8Weight(q.contiguous(), pack_sf(rows), scale)


def quant_act(x: torch.Tensor, src_rows: Optional[torch.Tensor] = None, M: Optional[int] = None,
              n_blocks: Optional[torch.Tensor] = None):
    """bf16 [T, K] -> (fp8 [M, K], SF tiles). With ``src_rows`` ([M] int32, -1 = zero row) rows are gathered;
    ``n_blocks`` (device int32) limits the work to the first n_blocks * 128 rows (the rest is left unwritten)."""
    if not x.is_cuda:
        xs = x.float() if src_rows is None else torch.where(
            (src_rows >= 0)[:, None], x.float()[src_rows.clamp(min=0).long()], torch.zeros(()))
        q, s = R.quant_fp8_rows(xs)
        return q, pack_sf(s)
    M = x.shape[0] if M is None else M
    if src_rows is not None:
        M = src_rows.numel()
    K = x.shape[1]
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    sf = empty_sf(M, K, x.device)
    ext().act_quant(x, q, sf, src_rows, M, n_blocks)
    return q, sf


def gather_rows_fp8(q: torch.Tensor, sf: torch.Tensor, src_rows: torch.Tensor,
                    n_blocks: Optional[torch.Tensor] = None):
    """Rows of an already-quantised matrix (fp8 + SF tiles) gathered by ``src_rows`` (-1 = zero row)."""
    M, K = src_rows.numel(), q.shape[1]
    if not q.is_cuda:
        s = unpack_sf(sf, q.shape[0], K)
        ok = src_rows >= 0
        idx = src_rows.clamp(min=0).long()
        qd = torch.where(ok[:, None], q.view(torch.uint8)[idx], torch.zeros((), dtype=torch.uint8)).view(q.dtype)
        sd = torch.where(ok[:, None], s[idx], torch.ones(()))
        return qd, pack_sf(sd)
    out = torch.empty(M, K, dtype=q.dtype, device=q.device)
    out_sf = empty_sf(M, K, q.device)
    ext().gather_fp8_rows(q, sf, src_rows, out, out_sf, n_blocks)
    return out, out_sf


def dequant_act(q: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    M, K = q.shape
    s = unpack_sf(sf.cpu(), M, K)
    return R.dequant_fp8_rows(q.cpu(), s)


def quantize_weight(w: torch.Tensor) -> Fp8Weight:
    """128×128 block quantisation on the tensor's own device (same math as ``ref.ops.quant_fp8_blocks``)."""
    N, K = w.shape
    nb, kb = (N + 127) // 128, (K + 127) // 128
    wp = torch.nn.functional.pad(w.float(), (0, kb * 128 - K, 0, nb * 128 - N))
    blocks = wp.view(nb, 128, kb, 128)
    s = R.ue8m0_scale(blocks.abs().amax(dim=(1, 3)))
    q = (blocks / s[:, None, :, None]).clamp(-R.FP8_MAX, R.FP8_MAX).to(torch.float8_e4m3fn)
    q = q.view(nb * 128, kb * 128)[:N, :K].contiguous()
    return Fp8Weight(q, pack_sf(s.repeat_interleave(128, dim=0)[:N]), s)


def stack_weights(ws) -> Fp8Weight:
    """Concatenate per-expert weights (each N rows, N % 128 == 0) into one [E*N, K] weight with SF tiles."""
    q = torch.cat([w.q for w in ws]).contiguous()
    rows = torch.cat([w.scale.repeat_interleave(128, dim=0)[: w.q.shape[0]] for w in ws])
    return Fp8Weight(q, pack_sf(rows), torch.cat([w.scale for w in ws]))
