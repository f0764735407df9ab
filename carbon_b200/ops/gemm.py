"""GEMM entry points (tcgen05 kernels in ``csrc/gemm.cuh``).

* ``fp8_gemm``      D = A·Bᵀ with block-scaled fp8 operands (kind::mxf8f6f4, UE8M0 scales), bf16/fp32 out.
* ``fp8_gemm_swiglu`` same GEMM whose epilogue applies SwiGLU to interleaved (gate|up) 128-column halves and
  re-quantises the result to fp8 + SF tiles (the input of the down projection).
* ``bf16_gemm``     kind::f16 bf16 GEMM, bf16/fp32 out.
* Grouped forms take ``m_block_expert`` (expert of each 128-row block, -1 = unused) for expert-sorted rows.

These replace the library GEMMs the reference dispatches per row band (FlashInfer CuTe-DSL / CUTLASS / cuBLASLt,
``king_v10/bundle_v9/prefill_gemm.py:15-72``; DeepGEMM fp8 GEMMs in ``dec/decode_gemm.py``).
"""
from __future__ import annotations

from typing import Optional

import torch

from ..ref import ops as R
from ._ext import ext
from .quant import Fp8Weight, dequant_act, empty_sf, quant_act, unpack_sf

OUT_BF16, OUT_SWIGLU_FP8, OUT_F32 = 0, 1, 2


def fp8_gemm(a_q: torch.Tensor, a_sf: torch.Tensor, w: Fp8Weight, out_dtype=torch.bfloat16,
             out: Optional[torch.Tensor] = None, m_block_expert=None, num_m_blocks=None, n_per_group: int = 0,
             status=None, pair: int = -1, row_valid=None) -> torch.Tensor:
    """pair: -1 = automatic (256x256 CTA-pair tiles for dense GEMMs with >= 512 rows), 1 = pair tiles (a grouped
    layout must then pad expert segments to 256 rows), 0 = 128-row tiles, 2 = weight streaming for grouped GEMMs
    with a few rows per expert (decode).  row_valid: rows < 0 are padding and are not written."""
    M = a_q.shape[0]
    N = n_per_group if m_block_expert is not None else w.q.shape[0]
    if not a_q.is_cuda:
        a = R.dequant_fp8_rows(a_q, unpack_sf(a_sf, M, a_q.shape[1]))
        return (a @ w.dequant().t()).to(out_dtype)
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a_q.device)
    epi = OUT_F32 if out.dtype == torch.float32 else OUT_BF16
    ext().gemm_fp8(a_q, a_sf, w.q, w.sf, out, epi, None, 0.0, m_block_expert, num_m_blocks, n_per_group, status,
                   pair, row_valid)
    return out


def fp8_gemm_swiglu(a_q, a_sf, w13: Fp8Weight, limit: float = 0.0, m_block_expert=None, num_m_blocks=None,
                    n_per_group: int = 0, status=None, pair: int = -1, row_valid=None):
    """w13 rows are interleaved in 128-row chunks: [gate 0:128, up 0:128, gate 128:256, up 128:256, ...].
    Returns (act fp8 [M, N/2], act SF tiles)."""
    M = a_q.shape[0]
    N = n_per_group if m_block_expert is not None else w13.q.shape[0]
    out = torch.empty(M, N // 2, dtype=torch.float8_e4m3fn, device=a_q.device)
    out_sf = empty_sf(M, N // 2, a_q.device)
    ext().gemm_fp8(a_q, a_sf, w13.q, w13.sf, out, OUT_SWIGLU_FP8, out_sf, float(limit), m_block_expert, num_m_blocks,
                   n_per_group, status, pair, row_valid)
    return out, out_sf


def bf16_gemm(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16, out: Optional[torch.Tensor] = None,
              m_block_expert=None, num_m_blocks=None, n_per_group: int = 0, status=None,
              k_splits: int = 0) -> torch.Tensor:
    """a [M, K] bf16, b [N, K] bf16 -> a @ b.T.  fp32 output with few rows and long K is split over K across
    CTAs (k_splits=0: automatic) so that a 1-tile problem still uses many SMs."""
    if not a.is_cuda:
        return (a.float() @ b.float().t()).to(out_dtype)
    M = a.shape[0]
    N = n_per_group if m_block_expert is not None else b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    epi = OUT_F32 if out.dtype == torch.float32 else OUT_BF16
    if k_splits == 0:
        k_splits = 1
        if epi == OUT_F32 and m_block_expert is None:
            # decode-sized rows: split K until the tiles x splits work items fill the SMs once (whole 4-block
            # k-groups per split); the weight stream is then read by one CTA per SM instead of a handful
            tiles = ((M + 127) // 128) * ((N + 127) // 128)
            kblocks = (a.shape[1] + 63) // 64
            if tiles < 32 and kblocks >= 64:
                k_splits = max(1, min(kblocks // 4, _num_sms(a.device) // tiles))
    ext().gemm_bf16(a, b, out, epi, m_block_expert, num_m_blocks, n_per_group, status, k_splits)
    return out


_SMS = {}


def _num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def interleave_gate_up(w1: torch.Tensor, w3: torch.Tensor, chunk: int = 128) -> torch.Tensor:
    """[I, K] gate and up -> [2I, K] with alternating 128-row chunks (gate, up, gate, up, ...)."""
    I, K = w1.shape
    assert I % chunk == 0
    g = w1.reshape(I // chunk, chunk, K)
    u = w3.reshape(I // chunk, chunk, K)
    return torch.stack([g, u], dim=1).reshape(2 * I, K)


def linear_fp8(x: torch.Tensor, w: Fp8Weight, out_dtype=torch.bfloat16, out=None) -> torch.Tensor:
    """x bf16 [M, K] -> quantise (1x128) -> block-scaled GEMM -> [M, N]."""
    q, sf = quant_act(x)
    return fp8_gemm(q, sf, w, out_dtype=out_dtype, out=out)
