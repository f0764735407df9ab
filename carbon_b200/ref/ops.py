"""Plain fp32 PyTorch restatements of every op. These are the numerics oracle for the CUDA kernels.

Each function states the math the corresponding kernel must reproduce.  The reference has no unit oracle (its checks
compare a new kernel with the sealed engine's bytes, ``king_v10/bundle_v9/moe_front.py:200-295``); here the oracle
is this file, written from the definitions:

* mHC stats / Sinkhorn / boundary: reconstructed from ``king_v10/bundle_v9/cuda_sinkhorn.py:150-190`` and
  ``cuda_mhc_packed.py:60-170`` (pre = σ(·)+eps, post = 2σ(·), comb = Sinkhorn of a 4×4 logit block).
* Router: sigmoid / sqrt-softplus / softmax score, bias only in the ranking key, ties to the lower expert id,
  renormalise, × routed scale (``cuda_moe_front.py:262-346`` for the sqrt-softplus form).
* fp8 quantisers: e4m3 with power-of-two (UE8M0) block scales, 1×128 for activations and 128×128 for weights.
* DSA lightning indexer: ``logit[t,s] = Σ_h w[t,h]·relu(q[t,h]·k[s])`` (``dec/cuda_paged_logits.py:35-37``).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

FP8_MAX = 448.0


# ----------------------------------------------------------------------------------------------------------------------
# norms / activations
# ----------------------------------------------------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y * w.float() if w is not None else y


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    return F.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(), eps)


def swiglu(g: torch.Tensor, u: torch.Tensor, limit: float = 0.0) -> torch.Tensor:
    if limit > 0:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
    return F.silu(g) * u


def softplus(x: torch.Tensor) -> torch.Tensor:
    """log(1 + e^x) from its definition, with the large-x cutoff (x > 20 => x)."""
    return torch.where(x > 20.0, x, torch.log1p(torch.exp(torch.clamp(x, max=20.0))))


# ----------------------------------------------------------------------------------------------------------------------
# RoPE (interleaved pairs: (x[2i], x[2i+1]) rotated by pos·θ^(-2i/d))
# ----------------------------------------------------------------------------------------------------------------------
def rope_inv_freq(dim: int, rope) -> torch.Tensor:
    """Inverse frequencies [dim/2] (fp64).  ``rope`` is theta, or (theta, factor, orig_max, beta_fast, beta_slow)
    for YaRN (Peng et al., 2023): dimensions that turn fewer than beta_slow times over the original context are
    interpolated (frequency / factor), those that turn more than beta_fast times are kept, with a linear ramp
    between the two correction dimensions."""
    theta = rope[0] if isinstance(rope, tuple) else rope
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    if not isinstance(rope, tuple):
        return inv
    _, factor, orig, beta_fast, beta_slow = rope

    def corr_dim(turns):                    # dimension index whose wavelength fits ``turns`` times in ``orig``
        return dim * math.log(orig / (turns * 2 * math.pi)) / (2 * math.log(theta))

    lo = max(math.floor(corr_dim(beta_fast)), 0)
    hi = min(math.ceil(corr_dim(beta_slow)), dim - 1)
    if lo == hi:
        hi += 0.001
    ramp = ((torch.arange(dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
    keep = 1.0 - ramp                       # 1: original frequency, 0: interpolated
    return inv / factor * (1 - keep) + inv * keep


def rope_cos_sin(positions: torch.Tensor, dim: int, theta) -> Tuple[torch.Tensor, torch.Tensor]:
    inv = rope_inv_freq(dim, theta)
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float, inverse: bool = False) -> torch.Tensor:
    """x: [T, ..., d] (d even); positions: [T]."""
    d = x.shape[-1]
    cos, sin = rope_cos_sin(positions, d, theta)
    if inverse:
        sin = -sin
    shape = [x.shape[0]] + [1] * (x.dim() - 2) + [d // 2]
    cos, sin = cos.view(shape), sin.view(shape)
    xf = x.float()
    x0, x1 = xf[..., 0::2], xf[..., 1::2]
    out = torch.empty_like(xf)
    out[..., 0::2] = x0 * cos - x1 * sin
    out[..., 1::2] = x0 * sin + x1 * cos
    return out


# ----------------------------------------------------------------------------------------------------------------------
# fp8 block quantisation with UE8M0 (power-of-two) scales
# ----------------------------------------------------------------------------------------------------------------------
def ue8m0_scale(amax: torch.Tensor) -> torch.Tensor:
    """Smallest power of two s with amax / s <= 448 (s = 2^ceil(log2(amax/448))); amax == 0 gives s = 1."""
    a = amax.float().clamp(min=1e-30)
    e = torch.ceil(torch.log2(a / FP8_MAX))
    s = torch.exp2(e)
    return torch.where(amax > 0, s, torch.ones_like(s))


def quant_fp8_rows(x: torch.Tensor, block: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-row 1×block quantisation. Returns (q fp8 e4m3 [M,K], scale fp32 [M, ceil(K/block)])."""
    M, K = x.shape
    nb = (K + block - 1) // block
    xp = F.pad(x.float(), (0, nb * block - K))
    blocks = xp.view(M, nb, block)
    s = ue8m0_scale(blocks.abs().amax(-1))
    q = (blocks / s[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(M, nb * block)[:, :K].contiguous(), s


def dequant_fp8_rows(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    M, K = q.shape
    sf = s.repeat_interleave(block, dim=1)[:, :K]
    return q.float() * sf


def fake_quant_fp8_rows(x: torch.Tensor) -> torch.Tensor:
    """Round the last dim (a multiple of 128) to e4m3 with one UE8M0 scale per 128 elements, in x's dtype (the
    values are exact in bf16)."""
    shp = x.shape
    q, s = quant_fp8_rows(x.reshape(-1, shp[-1]).float())
    return dequant_fp8_rows(q, s).reshape(shp).to(x.dtype)


def quant_fp8_blocks(w: torch.Tensor, block: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """128×128 weight quantisation. Returns (q [N,K], scale fp32 [ceil(N/128), ceil(K/128)])."""
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    wp = F.pad(w.float(), (0, kb * block - K, 0, nb * block - N))
    blocks = wp.view(nb, block, kb, block)
    s = ue8m0_scale(blocks.abs().amax(dim=(1, 3)))
    q = (blocks / s[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(nb * block, kb * block)[:N, :K].contiguous(), s


def dequant_fp8_blocks(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    sf = s.repeat_interleave(block, 0).repeat_interleave(block, 1)[:N, :K]
    return q.float() * sf


# ----------------------------------------------------------------------------------------------------------------------
# MXFP4 (OCP microscaling fp4): e2m1 elements, one UE8M0 power-of-two scale per 32 consecutive elements of a row.
# The reference's routed experts are stored this way (fp8 activations x MXFP4 weights, UE8M0/32; moe_prefill.py:14-16).
# ----------------------------------------------------------------------------------------------------------------------
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)      # magnitudes of codes 0..7; bit 3 is the sign


def quant_mxfp4(w: torch.Tensor, block: int = 32) -> Tuple[torch.Tensor, torch.Tensor]:
    """[N, K] -> (packed uint8 [N, K/2]: element 2i in the low nibble, 2i+1 in the high one; scale uint8 [N, K/32]:
    biased exponent e+127 of the block scale 2^e, the smallest power of two with amax / 2^e <= 6).  Elements round
    to the nearest e2m1 value (ties to the smaller magnitude)."""
    N, K = w.shape
    assert K % block == 0 and block % 2 == 0
    wb = w.float().reshape(N, K // block, block)
    amax = wb.abs().amax(-1)
    m, ex = torch.frexp(amax / 6.0)                          # amax/6 = m * 2^ex, m in [0.5, 1)
    e = torch.where(amax > 0, ex - (m == 0.5).to(ex.dtype), torch.zeros_like(ex)).clamp(-127, 127)
    x = wb / torch.pow(2.0, e.float())[..., None]
    grid = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=w.device)
    code = (x.abs()[..., None] - grid).abs().argmin(-1)      # first minimum: the smaller magnitude on a tie
    nib = code | (((x < 0) & (code > 0)).long() << 3)
    nib = nib.reshape(N, K)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).to(torch.uint8)
    return packed.contiguous(), (e + 127).to(torch.uint8).contiguous()


def dequant_mxfp4(packed: torch.Tensor, scale: torch.Tensor, block: int = 32) -> torch.Tensor:
    """Inverse of ``quant_mxfp4``: -> fp32 [N, K]."""
    N = packed.shape[0]
    K = packed.shape[1] * 2
    p = packed.long()
    nib = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(N, K)
    grid = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=packed.device)
    v = grid[nib & 7] * torch.where((nib & 8) != 0, -1.0, 1.0)
    s = torch.pow(2.0, scale.float() - 127.0).repeat_interleave(block, dim=1)
    return v * s


def quant_fp8_rows32(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """[R, K] -> (e4m3 [R, K], UE8M0 biased exponents uint8 [R, K/32]): one power-of-two scale per 32 elements,
    the smallest with amax / 2^e <= 448 (the Engram table row format: 256 e4m3 + UE8M0/32)."""
    R_, K = w.shape
    wb = w.float().reshape(R_, K // 32, 32)
    amax = wb.abs().amax(-1)
    m, ex = torch.frexp(amax / FP8_MAX)
    e = torch.where(amax > 0, ex - (m == 0.5).to(ex.dtype), torch.full_like(ex, -127)).clamp(-127, 127)
    q = (wb / torch.pow(2.0, e.float())[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(R_, K).contiguous(), (e + 127).to(torch.uint8).contiguous()


def dequant_fp8_rows32(q: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    return q.float() * torch.pow(2.0, sf.float() - 127.0).repeat_interleave(32, dim=1)


# ----------------------------------------------------------------------------------------------------------------------
# fp8 latent KV rows (the paged cache's quantised format)
# ----------------------------------------------------------------------------------------------------------------------
LATENT_ATOM = 64


def latent_fp8_row_bytes(r: int, dr: int, mla: bool) -> int:
    """Bytes of one cached token row in the fp8 format: r e4m3 latent values (one UE8M0 scale per 64-dim atom),
    the scale bytes padded to 16, then (MLA) the dr RoPE-key dims as fp16.  r = 512, dr = 64: 656 bytes for MLA
    (1152 in bf16), 528 for latent MQA (1024 in bf16; its RoPE dims are the last atom of the latent)."""
    na = r // LATENT_ATOM
    return r + (na + 15) // 16 * 16 + (2 * dr if mla else 0)


def _latent_fp8_offsets(r: int, dr: int, mla: bool):
    """Byte layout of an fp8 row: [values of the first r/2 dims | scale bytes (padded to 16) | values of the last
    r/2 dims | fp16 RoPE key (MLA)].  Each half of the decode kernel's CTA pair then reads one contiguous piece:
    [0, r/2 + 16) and [r/2, end)."""
    na = r // LATENT_ATOM
    h = r // 2
    sc = (na + 15) // 16 * 16
    return h, h + sc, r + sc          # scales at h, second half of the values at h + sc, RoPE at r + sc


def quant_latent_fp8(rows: torch.Tensor, r: int, dr: int, mla: bool) -> torch.Tensor:
    """[n, r (+ dr)] latent rows -> [n, row_bytes] uint8 in the fp8 cache format.  Each 64-dim atom gets the
    smallest power-of-two scale 2^e with amax / 2^e <= 448 (e clamped to [-126, 127]; 2^0 for an all-zero atom)
    and its values are rounded to nearest-even e4m3."""
    n = rows.shape[0]
    na = r // LATENT_ATOM
    rb = latent_fp8_row_bytes(r, dr, mla)
    s_off, v2_off, pe_off = _latent_fp8_offsets(r, dr, mla)
    h = r // 2
    x = rows[:, :r].float().reshape(n, na, LATENT_ATOM)
    amax = x.abs().amax(-1)
    m, ex = torch.frexp(amax / FP8_MAX)
    e = torch.where(amax > 0, ex - (m == 0.5).to(ex.dtype), torch.zeros_like(ex)).clamp(-126, 127)
    q = (x / torch.pow(2.0, e.float())[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    qb = q.reshape(n, r).view(torch.uint8)
    out = torch.zeros(n, rb, dtype=torch.uint8, device=rows.device)
    out[:, :h] = qb[:, :h]
    out[:, s_off:s_off + na] = (e + 127).to(torch.uint8)
    out[:, v2_off:v2_off + r - h] = qb[:, h:]
    if mla:
        out[:, pe_off:pe_off + 2 * dr] = rows[:, r:r + dr].to(torch.float16).contiguous().view(torch.uint8)
    return out


def dequant_latent_fp8(rows8: torch.Tensor, r: int, dr: int, mla: bool) -> torch.Tensor:
    """Inverse of ``quant_latent_fp8``: [n, row_bytes] uint8 -> [n, r (+ dr)] float32."""
    n = rows8.shape[0]
    na = r // LATENT_ATOM
    s_off, v2_off, pe_off = _latent_fp8_offsets(r, dr, mla)
    h = r // 2
    qb = torch.cat([rows8[:, :h], rows8[:, v2_off:v2_off + r - h]], dim=1).contiguous()
    q = qb.view(torch.float8_e4m3fn).float().reshape(n, na, LATENT_ATOM)
    s = torch.pow(2.0, rows8[:, s_off:s_off + na].float() - 127.0)
    x = (q * s[..., None]).reshape(n, r)
    if mla:
        x = torch.cat([x, rows8[:, pe_off:pe_off + 2 * dr].contiguous().view(torch.float16).float()], dim=1)
    return x


def fake_quant_mxfp4(x: torch.Tensor, block: int = 32) -> torch.Tensor:
    """Round x (any shape, last dim a multiple of 32) to MXFP4 values in its own dtype: per 32-element block the
    scale of ``quant_mxfp4`` and the nearest e2m1 value, ties to the smaller magnitude (identical to
    dequant_mxfp4(quant_mxfp4(x))).  Arithmetic only, so it runs on any device without large temporaries."""
    shp = x.shape
    xb = x.float().reshape(-1, shp[-1] // block, block)
    amax = xb.abs().amax(-1, keepdim=True)
    m, ex = torch.frexp(amax / 6.0)
    e = torch.where(amax > 0, ex - (m == 0.5).to(ex.dtype), torch.zeros_like(ex)).clamp(-127, 127)
    sc = torch.pow(2.0, e.float())
    mag = xb.abs() / sc
    step = torch.where(mag < 2.0, 0.5, torch.where(mag < 4.0, 1.0, 2.0))
    r = (torch.ceil(mag / step - 0.5) * step).clamp(max=6.0)
    return (torch.sign(xb) * r * sc).reshape(shp).to(x.dtype)


def fp8_gemm(a_q, a_s, b_q, b_s) -> torch.Tensor:
    """Block-scaled fp8 GEMM oracle: dequantise both operands and multiply in fp32. Returns [M, N] fp32."""
    return dequant_fp8_rows(a_q, a_s) @ dequant_fp8_blocks(b_q, b_s).t()


# ----------------------------------------------------------------------------------------------------------------------
# mHC
# ----------------------------------------------------------------------------------------------------------------------
def sinkhorn(logits: torch.Tensor, iters: int, eps: float) -> torch.Tensor:
    """logits [..., n, n] -> doubly-stochastic comb. Row softmax + eps, column normalise, then iters-1 more
    (row, column) normalisation passes, each dividing by (sum + eps)."""
    c = torch.softmax(logits.float(), dim=-1) + eps
    c = c / (c.sum(-2, keepdim=True) + eps)
    for _ in range(iters - 1):
        c = c / (c.sum(-1, keepdim=True) + eps)
        c = c / (c.sum(-2, keepdim=True) + eps)
    return c


def mhc_coeffs(X: torch.Tensor, fn: torch.Tensor, base: torch.Tensor, scale: torch.Tensor, hc: int,
               iters: int, hc_eps: float, rms_eps: float):
    """X [T, hc, D]; fn [hc*(2+hc), hc*D]; base [hc*(2+hc)]; scale [3].
    Returns pre [T,hc], post [T,hc], comb [T,hc,hc]."""
    T = X.shape[0]
    xf = X.reshape(T, X.shape[1] * X.shape[2]).float()
    rsq = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + rms_eps)
    m = (xf @ fn.float().t()) * rsq
    pre = torch.sigmoid(m[:, :hc] * scale[0] + base[:hc]) + hc_eps
    post = 2.0 * torch.sigmoid(m[:, hc:2 * hc] * scale[1] + base[hc:2 * hc])
    comb = sinkhorn((m[:, 2 * hc:] * scale[2] + base[2 * hc:]).view(T, hc, hc), iters, hc_eps)
    return pre, post, comb


def mhc_head_coeffs(X, fn, base, scale, hc_eps, rms_eps):
    T = X.shape[0]
    xf = X.reshape(T, X.shape[1] * X.shape[2]).float()
    rsq = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + rms_eps)
    m = (xf @ fn.float().t()) * rsq
    return torch.sigmoid(m * scale[0] + base) + hc_eps


def mhc_pre_mix(X: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    """y = Σ_i pre_i · X_i  -> [T, D]."""
    return (X.float() * pre[:, :, None]).sum(1)


def mhc_post_mix(X: torch.Tensor, out: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
    """X'_o = post_o · out + Σ_i comb[i][o] · X_i  -> [T, hc, D]."""
    return post[:, :, None] * out.float()[:, None, :] + torch.einsum("tio,tid->tod", comb, X.float())


# ----------------------------------------------------------------------------------------------------------------------
# router
# ----------------------------------------------------------------------------------------------------------------------
def router_topk(logits: torch.Tensor, bias: Optional[torch.Tensor], k: int, score_func: str, route_scale: float,
                norm: bool, n_groups: int = 1, topk_groups: int = 1):
    """logits [T, E] fp32. Returns (weights [T,k] fp32, ids [T,k] int32). Ties go to the lower expert id."""
    lf = logits.float()
    if score_func == "sigmoid":
        act = torch.sigmoid(lf)
    elif score_func == "sqrtsoftplus":
        act = torch.sqrt(softplus(lf))
    elif score_func == "softmax":
        act = torch.softmax(lf, dim=-1)
    else:
        raise ValueError(score_func)
    if bias is None:
        key = act.clone()
    else:                                   # [E] shared, or [T, E] per token (multimodal bias switch)
        key = act + (bias.float()[None, :] if bias.dim() == 1 else bias.float())
    T, E = key.shape
    if n_groups > 1:
        g = key.view(T, n_groups, E // n_groups)
        gscore = g.topk(2, dim=-1).values.sum(-1)
        keep = _stable_topk(gscore, topk_groups)
        mask = torch.zeros(T, n_groups, dtype=torch.bool, device=key.device)
        mask.scatter_(1, keep, True)
        key = key.masked_fill(~mask.repeat_interleave(E // n_groups, dim=1), float("-inf"))
    ids = _stable_topk(key, k)
    w = act.gather(1, ids)
    if norm:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return w * route_scale, ids.to(torch.int32)


def _stable_topk(key: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k by value with ties broken toward the lower index (deterministic)."""
    E = key.shape[-1]
    # sort by (-value, index): stable sort on -value keeps index order for ties
    order = torch.sort(-key, dim=-1, stable=True).indices
    return order[..., :k]


# ----------------------------------------------------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------------------------------------------------
def causal_attention(q, k, v, scale: float, q_pos: torch.Tensor, k_pos: torch.Tensor,
                     allowed: Optional[torch.Tensor] = None, sink: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q [Tq,H,dq], k [Tk,H,dq] or [Tk,1,dq], v [Tk,H,dv] or [Tk,1,dv].
    Mask: k_pos <= q_pos, and (if given) allowed[Tq, Tk] bool.  sink [H]: one extra logit per head in the softmax
    denominator (it takes probability mass but has no value row).  Returns [Tq, H, dv] fp32."""
    qf, kf, vf = q.float(), k.float(), v.float()
    if kf.shape[1] == 1:
        kf = kf.expand(-1, qf.shape[1], -1)
    if vf.shape[1] == 1:
        vf = vf.expand(-1, qf.shape[1], -1)
    s = torch.einsum("qhd,khd->hqk", qf, kf) * scale
    mask = k_pos[None, :] <= q_pos[:, None]
    if allowed is not None:
        mask = mask & allowed
    s = s.masked_fill(~mask[None], float("-inf"))
    if sink is not None:
        s = torch.cat([s, sink.float()[:, None, None].expand(-1, s.shape[1], 1)], dim=-1)
        p = torch.softmax(s, dim=-1)[..., :-1]
    else:
        p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vf)


def indexer_logits(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """q [Tq, Hi, d], k [Tk, d], w [Tq, Hi] -> logits [Tq, Tk] = Σ_h w[t,h]·relu(q[t,h]·k[s])."""
    s = torch.einsum("qhd,kd->qhk", q.float(), k.float()).clamp(min=0)
    return torch.einsum("qhk,qh->qk", s, w.float())


def topk_mask(logits: torch.Tensor, q_pos: torch.Tensor, k_pos: torch.Tensor, topk: int) -> torch.Tensor:
    """Boolean [Tq, Tk]: the top-k causal keys of each query (all causal keys when fewer than topk exist)."""
    causal = k_pos[None, :] <= q_pos[:, None]
    l = logits.masked_fill(~causal, float("-inf"))
    k = min(topk, l.shape[1])
    idx = _stable_topk(l, k)
    m = torch.zeros_like(causal)
    m.scatter_(1, idx, True)
    return m & causal


# ----------------------------------------------------------------------------------------------------------------------
# Engram: hashed n-gram memory
# ----------------------------------------------------------------------------------------------------------------------
ENGRAM_MULT = 1000003          # hash multiplier (odd, < 2^20 so every step fits int64)


def engram_hash_ids(window: torch.Tensor, orders, heads: int, primes, vocab_size: int) -> torch.Tensor:
    """window [T, nmax] int64: column i = the token i positions back (i = 0: the token itself), -1 before the
    sequence start.  Column c = (order orders[c // heads], head c % heads) hashes the `order` most recent tokens:
    h = 0; for each token u (most recent first): h = ((h * MULT) ^ (u' + 7919 * (c + 1))) & (2^31 - 1), with
    u' = u + 1 (0 for the padding before the sequence start); row = h % primes[c] + (rows of earlier columns).
    Returns int64 [T, n_cols] global table rows."""
    T = window.shape[0]
    cols = []
    base = 0
    w = torch.where(window >= 0, window + 1, torch.zeros_like(window)).long()
    for c in range(len(orders) * heads):
        n = orders[c // heads]
        h = torch.zeros(T, dtype=torch.long, device=window.device)
        for i in range(n):
            h = ((h * ENGRAM_MULT) ^ (w[:, i] + 7919 * (c + 1))) & 0x7FFFFFFF
        cols.append(h % primes[c] + base)
        base += primes[c]
    return torch.stack(cols, dim=1)


def engram_gate(X: torch.Tensor, kv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor, eps: float,
                clamp: float) -> torch.Tensor:
    """X [T, hc, D] residual streams, kv [T, (hc + 1) * D] = per-stream keys then the shared value.
    X_c + sigmoid(clamp(<rms(X_c) * q_w, rms(k_c) * k_w> / sqrt(D), +-clamp)) * value."""
    T, hc, D = X.shape
    Xf = X.float()
    k = kv[:, :hc * D].float().view(T, hc, D)
    v = kv[:, hc * D:].float()
    xn = Xf * torch.rsqrt(Xf.pow(2).mean(-1, keepdim=True) + eps) * q_w.float()
    kn = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + eps) * k_w.float()
    s = (xn * kn).sum(-1) / math.sqrt(D)
    g = torch.sigmoid(s.clamp(-clamp, clamp))                                  # [T, hc]
    return Xf + g[..., None] * v[:, None, :]
