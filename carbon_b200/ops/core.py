"""Wrappers of the CUDA-core kernels (``csrc/small_ops.cu``). CPU tensors run the fp32 oracle instead."""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ..ref import ops as R
from ._ext import ext
from .quant import empty_sf, pack_sf

SCORE_FUNCS = {"sigmoid": 0, "sqrtsoftplus": 1, "softmax": 2}


def rms_norm_(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """In-place RMSNorm of the rows of x (a bf16 [M, D] view with unit column stride, e.g. a column slice of a
    wider projection output).  The kernel reads each element before it writes it, with one thread per element in both
    passes, so the output may alias the input."""
    if not x.is_cuda:
        x.copy_(R.rms_norm(x, w, eps).to(x.dtype))
        return x
    ext().rms_norm(x, w, x, None, None, float(eps))
    return x


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, want_bf16: bool = True, want_fp8: bool = False):
    """Returns y (bf16) and/or (q fp8, sf)."""
    if not x.is_cuda:
        y = R.rms_norm(x, w, eps)
        outs = []
        if want_bf16:
            outs.append(y.to(x.dtype))
        if want_fp8:
            q, s = R.quant_fp8_rows(y)
            outs.append((q, pack_sf(s)))
        return outs[0] if len(outs) == 1 else tuple(outs)
    M, D = x.shape
    y = torch.empty(M, D, dtype=torch.bfloat16, device=x.device) if want_bf16 else None
    q = torch.empty(M, D, dtype=torch.float8_e4m3fn, device=x.device) if want_fp8 else None
    sf = empty_sf(M, D, x.device) if want_fp8 else None
    ext().rms_norm(x, w, y, q, sf, float(eps))
    if want_bf16 and want_fp8:
        return y, (q, sf)
    return y if want_bf16 else (q, sf)


def rope_table(max_pos: int, dim: int, theta: float, device) -> torch.Tensor:
    """fp32 [max_pos, dim] interleaved (cos_j, sin_j) pairs computed in fp64."""
    cos, sin = R.rope_cos_sin(torch.arange(max_pos), dim, theta)     # theta: a float or a YaRN spec
    return torch.stack([cos, sin], dim=-1).reshape(max_pos, dim).contiguous().to(device)


def rope_(x: torch.Tensor, off: int, dim: int, table: torch.Tensor, pos: torch.Tensor, inverse: bool = False):
    """In-place RoPE on x[T, H, off:off+dim] (interleaved pairs)."""
    if not x.is_cuda:
        cs = table[pos.long()].view(x.shape[0], dim // 2, 2)
        cos, sin = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
        if inverse:
            sin = -sin
        seg = x[..., off:off + dim].float()
        a, b = seg[..., 0::2], seg[..., 1::2]
        out = torch.empty_like(seg)
        out[..., 0::2] = a * cos - b * sin
        out[..., 1::2] = a * sin + b * cos
        x[..., off:off + dim] = out.to(x.dtype)
        return x
    ext().rope(x, off, dim, table, pos, inverse)
    return x


def router_topk(logits: torch.Tensor, bias: Optional[torch.Tensor], k: int, score_func: str, route_scale: float,
                norm: bool, bias_img: Optional[torch.Tensor] = None, tok: Optional[torch.Tensor] = None,
                img_id: int = -1, n_groups: int = 1, topk_groups: int = 1) -> Tuple[torch.Tensor, torch.Tensor]:
    """Biased top-k router; with ``bias_img``, tokens whose id (``tok``) is ``img_id`` rank with that bias.
    Group-limited routing (``n_groups`` > 1: experts only from the ``topk_groups`` groups with the best top-2 key
    sums, ties toward the lower group) runs in the same kernel."""
    if not logits.is_cuda:
        if bias_img is not None and tok is not None:
            is_img = (tok.long() == img_id)[:, None]
            b = bias if bias is not None else torch.zeros_like(bias_img)
            bias = torch.where(is_img, bias_img.float()[None, :], b.float()[None, :])
        w, ids = R.router_topk(logits, bias, k, score_func, route_scale, norm, n_groups, topk_groups)
        return w.contiguous(), ids.contiguous()          # the expert kernels read dense [T, k] rows
    T = logits.shape[0]
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    ext().router_topk(logits.float().contiguous(), bias, k, SCORE_FUNCS[score_func], norm, float(route_scale), w, ids,
                      bias_img, tok.to(torch.int32).contiguous() if tok is not None else None, int(img_id),
                      int(n_groups), int(topk_groups))
    return w, ids


_ALIGN_FLAG = None


def moe_align(rows: int, n_experts: int) -> int:
    """Row alignment of expert segments: 256 (CTA-pair GEMM tiles) once experts average enough rows that the extra
    padding costs less than the pair tiles save, else 128.  ``CARBON_MOE_ALIGN`` (KernelFlags.moe_align) pins it."""
    global _ALIGN_FLAG
    if _ALIGN_FLAG is None:
        from ..config import KernelFlags

        _ALIGN_FLAG = KernelFlags.from_env().moe_align
    if _ALIGN_FLAG in (128, 256):
        return _ALIGN_FLAG
    return 256 if rows >= 384 * n_experts else 128


class MoeLayout:
    """Expert-sorted row layout of one MoE call: every expert segment padded to `align` rows (128 or 256), blocks
    of 128 rows tagged with their expert."""

    def __init__(self, ids: torch.Tensor, n_experts: int, max_blocks: Optional[int] = None, align: int = 0):
        T, k = ids.shape
        dev = ids.device
        if align == 0:
            align = moe_align(T * k, n_experts)
        self.align = align
        if max_blocks is None:
            max_blocks = (T * k + 127) // 128 + n_experts * (align // 128)
            max_blocks += max_blocks & 1
        self.T, self.k, self.E, self.max_blocks = T, k, n_experts, max_blocks
        self.slot_pos = torch.empty(T, k, dtype=torch.int32, device=dev)
        self.row_src = torch.empty(max_blocks * 128, dtype=torch.int32, device=dev)
        self.m_block_expert = torch.empty(max_blocks, dtype=torch.int32, device=dev)
        self.num_blocks = torch.empty(1, dtype=torch.int32, device=dev)
        self.counts = torch.empty(n_experts, dtype=torch.int32, device=dev)
        if ids.is_cuda:
            scratch = torch.empty(2 * n_experts, dtype=torch.int32, device=dev)
            ext().moe_layout(ids.contiguous(), n_experts, self.slot_pos, self.row_src, self.m_block_expert,
                             self.num_blocks, self.counts, align, scratch)
        else:
            self._cpu(ids)

    def _cpu(self, ids):
        T, k, E = self.T, self.k, self.E
        flat = ids.reshape(-1).long()
        counts = torch.bincount(flat, minlength=E)
        start = torch.zeros(E, dtype=torch.long)
        acc = 0
        mbe = []
        for e in range(E):
            start[e] = acc
            nb = (int(counts[e]) + self.align - 1) // self.align * (self.align // 128)
            mbe += [e] * nb
            acc += nb * 128
        self.num_blocks[0] = len(mbe)
        self.m_block_expert.fill_(-1)
        self.m_block_expert[: len(mbe)] = torch.tensor(mbe, dtype=torch.int32)
        self.row_src.fill_(-1)
        fill = torch.zeros(E, dtype=torch.long)
        for i in range(T * k):
            e = int(flat[i])
            pos = int(start[e] + fill[e])
            fill[e] += 1
            self.slot_pos.view(-1)[i] = pos
            self.row_src[pos] = i // k
        self.counts.copy_(counts.to(torch.int32))

    @property
    def rows(self) -> int:
        return self.max_blocks * 128

    @property
    def pair(self) -> int:
        """GEMM tile mode for this layout: 1 = CTA-pair tiles, 2 = weight streaming (a few rows per expert, decode),
        0 = 128-row tiles."""
        if self.align == 256:
            return 1
        return 2 if self.T * self.k <= 32 * self.E else 0


def moe_combine(Y: torch.Tensor, w: torch.Tensor, slot_pos: torch.Tensor, add: Optional[torch.Tensor],
                T: int) -> torch.Tensor:
    if not Y.is_cuda:
        out = torch.zeros(T, Y.shape[1], dtype=torch.float32)
        for j in range(slot_pos.shape[1]):
            pos = slot_pos[:, j].long()
            ok = pos >= 0
            out[ok] += w[ok, j:j + 1].float() * Y[pos[ok]].float()
        if add is not None:
            out += add.float()
        return out.to(Y.dtype)
    out = torch.empty(T, Y.shape[1], dtype=torch.bfloat16, device=Y.device)
    ext().moe_combine(Y, w, slot_pos, add, out)
    return out


def split_hi_lo(fn: torch.Tensor) -> torch.Tensor:
    """fp32 [n, K] -> bf16 [2n, K] = [hi; lo] with hi = bf16(fn), lo = bf16(fn - hi): x·fn ≈ x·hi + x·lo."""
    hi = fn.float().to(torch.bfloat16)
    lo = (fn.float() - hi.float()).to(torch.bfloat16)
    return torch.cat([hi, lo], dim=0).contiguous()
