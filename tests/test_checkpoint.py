"""fp8 block-scaled safetensors checkpoints: save -> load round trip; the engine served from a checkpoint equals
the engine served from the same (fp8-rounded) weights in memory."""
import torch

from carbon_b200.config import tiny_config
from carbon_b200.engine.engine import Engine
from carbon_b200.models.checkpoint import CheckpointSource, is_fp8_name, save_checkpoint
from carbon_b200.models.weights import WeightSource
from carbon_b200.ref import ops as R
from carbon_b200.ref.model import init_weights


def _fp8_rounded(w):
    out = {}
    for k, v in w.items():
        if is_fp8_name(k):
            out[k] = torch.stack([R.dequant_fp8_blocks(*R.quant_fp8_blocks(x)) for x in v]) if v.dim() == 3 else \
                R.dequant_fp8_blocks(*R.quant_fp8_blocks(v))
        else:
            out[k] = v
    return out


def test_checkpoint_roundtrip_and_engine(tmp_path):
    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    for per_expert in (False, True):
        d = tmp_path / f"ckpt{int(per_expert)}"
        save_checkpoint(w, str(d), per_expert=per_expert)
        src = CheckpointSource(cfg, str(d))
        ref = _fp8_rounded(w)
        for name in ("layers.0.attn.wq_b.weight", "layers.1.ffn.experts.w2", "layers.0.attn_hc.fn"):
            got = src.get(name, "cpu")
            exp = ref[name] if is_fp8_name(name) else ref[name].to(torch.bfloat16).float() \
                if ref[name].numel() > 4096 else ref[name]
            assert torch.allclose(got, exp, atol=1e-6), name
    prompts = [[1, 2, 3, 4, 5, 6, 7, 8] * 4]
    e1 = Engine(cfg, "cpu", source=CheckpointSource(cfg, str(tmp_path / "ckpt0")), num_pages=8, page_size=16)
    st = {n: CheckpointSource(cfg, str(tmp_path / "ckpt0")).get(n, "cpu") for n in w}
    e2 = Engine(cfg, "cpu", source=WeightSource(cfg, state=st), num_pages=8, page_size=16)
    assert e1.generate(prompts, 4) == e2.generate(prompts, 4)


def test_mxfp4_experts_checkpoint(tmp_path):
    """Routed experts stored as MXFP4 (e2m1 + UE8M0 per 32) load as their exact values, for stacked and per-expert
    storage, and the engine served from that checkpoint equals the engine over the same values in memory; the V4
    layout's grouped output projection (wo_b) is stored in fp8."""
    from carbon_b200.config import tiny_v4_config

    cfg = tiny_v4_config()
    w = init_weights(cfg, seed=0)
    for per_expert in (False, True):
        d = tmp_path / f"mx{int(per_expert)}"
        save_checkpoint(w, str(d), per_expert=per_expert, mxfp4_experts=True)
        src = CheckpointSource(cfg, str(d))
        for name in ("layers.0.ffn.experts.w1", "layers.1.ffn.experts.w2"):
            exp = torch.stack([R.dequant_mxfp4(*R.quant_mxfp4(x)) for x in w[name]])
            assert torch.equal(src.get(name, "cpu"), exp), name
        got = src.get("layers.0.attn.wo_b.weight", "cpu")
        assert torch.equal(got, R.dequant_fp8_blocks(*R.quant_fp8_blocks(w["layers.0.attn.wo_b.weight"])))
        tab = w["layers.1.engram.table"]           # Engram rows: e4m3 + UE8M0 per 32
        assert torch.equal(src.get("layers.1.engram.table", "cpu"), R.dequant_fp8_rows32(*R.quant_fp8_rows32(tab)))
    st = {n: CheckpointSource(cfg, str(tmp_path / "mx0")).get(n, "cpu") for n in w}
    prompts = [[5, 6, 7, 8, 9] * 8]
    e1 = Engine(cfg, "cpu", source=CheckpointSource(cfg, str(tmp_path / "mx0")), num_pages=8, page_size=16)
    e2 = Engine(cfg, "cpu", source=WeightSource(cfg, state=st), num_pages=8, page_size=16)
    assert e1.generate(prompts, 4) == e2.generate(prompts, 4)
