"""Weight sources: a checkpoint/state dict, or seeded random init generated directly on the target device.

Random init is deterministic per tensor name (the seed is derived from the name), so any rank can materialise any
shard without generating the others, and a run with tied layer sets (``layer_sets``) reuses the tensors of layer
``i % layer_sets`` for layer ``i``.  The checkpoint naming follows ``ref.model.param_shapes``; fp8 checkpoints
carry ``<name>`` (float8_e4m3fn) plus ``<name>_scale_inv`` (fp32 128×128 block scales, the DeepSeek format).
"""
from __future__ import annotations

import hashlib
import re
from typing import Dict, Optional

import torch

from ..config import ModelConfig
from ..ref.model import param_shapes

_LAYER_RE = re.compile(r"^layers\.(\d+)\.")


def _seed_of(name: str, base: int) -> int:
    h = hashlib.sha256(f"{base}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & 0x7FFFFFFFFFFFFFFF


class WeightSource:
    def __init__(self, cfg: ModelConfig, state: Optional[Dict[str, torch.Tensor]] = None, seed: int = 0,
                 layer_sets: Optional[int] = None):
        self.cfg = cfg
        self.state = state
        self.seed = seed
        self.layer_sets = layer_sets
        self.shapes = param_shapes(cfg)

    def canonical(self, name: str) -> str:
        if self.layer_sets:
            m = _LAYER_RE.match(name)
            if m:
                i = int(m.group(1))
                # keep dense/MoE kind: tie within the same layer kind
                nd = self.cfg.n_dense_layers
                if i < nd:
                    j = i % min(self.layer_sets, nd)
                else:
                    j = nd + (i - nd) % self.layer_sets
                name = f"layers.{j}." + name[m.end():]
        return name

    def get(self, name: str, device, rows: Optional[slice] = None) -> torch.Tensor:
        """fp32 tensor (optionally a slice of rows of dim 0) on `device`."""
        cname = self.canonical(name)
        if self.state is not None:
            t = self.state[cname]
            if rows is not None:
                t = t[rows]
            return t.to(device=device, dtype=torch.float32)
        shape, kind = self.shapes[name]
        if rows is not None:
            start, stop = rows.start or 0, rows.stop if rows.stop is not None else shape[0]
            shape = (stop - start,) + tuple(shape[1:])
        if kind == "ones":
            return torch.ones(shape, device=device)
        if kind == "zeros":
            return torch.zeros(shape, device=device)
        g = torch.Generator(device=device)
        g.manual_seed(_seed_of(cname + (f"[{rows.start}:{rows.stop}]" if rows is not None else ""), self.seed))
        return torch.randn(shape, generator=g, device=device) * self.cfg.init_std
