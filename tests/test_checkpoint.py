"""fp8 block-scaled safetensors checkpoints: save -> load round trip; the engine served from a checkpoint equals
the engine served from the same (fp8-rounded) weights in memory."""
import os

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


def _to_hf(name):
    """This test's own spelling of Hugging Face DeepSeek names (written out independently of the loader's table)."""
    import re

    top = {"embed.weight": "model.embed_tokens.weight", "norm.weight": "model.norm.weight",
           "head.weight": "lm_head.weight"}
    if name in top:
        return top[name]
    m = re.match(r"^layers\.(\d+)\.(.+)$", name)
    if m is None:
        return name
    i, rest = m.group(1), m.group(2)
    sub = [("attn_norm.weight", "input_layernorm.weight"), ("ffn_norm.weight", "post_attention_layernorm.weight"),
           ("attn.wq_a.", "self_attn.q_a_proj."), ("attn.wq_b.", "self_attn.q_b_proj."),
           ("attn.wkv_a.", "self_attn.kv_a_proj_with_mqa."), ("attn.wkv_b.", "self_attn.kv_b_proj."),
           ("attn.wo.", "self_attn.o_proj."), ("attn.q_norm.", "self_attn.q_a_layernorm."),
           ("attn.kv_norm.", "self_attn.kv_a_layernorm."), ("attn.indexer.wq.", "self_attn.indexer.wq_b."),
           ("attn.indexer.", "self_attn.indexer."), ("ffn.gate.weight", "mlp.gate.weight"),
           ("ffn.gate.bias", "mlp.gate.e_score_correction_bias")]
    for a, b in sub:
        if rest.startswith(a):
            return f"model.layers.{i}.{b}{rest[len(a):]}"
    m = re.match(r"^ffn\.(experts\.\d+\.|shared\.|)(w[123])(_scale_inv)?$", rest)
    if m:
        grp = {"": "", "shared.": "shared_experts."}.get(m.group(1), m.group(1))
        proj = {"w1": "gate_proj", "w2": "down_proj", "w3": "up_proj"}[m.group(2)]
        return f"model.layers.{i}.mlp.{grp}{proj}.weight{m.group(3) or ''}"
    return name                                           # mHC parameters keep this loader's names


def test_hugging_face_names_load(tmp_path):
    from safetensors.torch import load_file, save_file

    cfg = tiny_config()
    w = init_weights(cfg, seed=0)
    d = tmp_path / "ours"
    save_checkpoint(w, str(d), per_expert=True)
    tensors = {}
    for fn in sorted(os.listdir(d)):
        if fn.endswith(".safetensors"):
            tensors.update(load_file(str(d / fn)))
    hf = {_to_hf(k): v for k, v in tensors.items()}
    assert any(k.startswith("model.layers.0.mlp.experts.1.up_proj.weight_scale_inv") for k in hf)
    hf[f"model.layers.{cfg.n_layers}.eh_proj.weight"] = torch.zeros(4, 4)   # an MTP layer: ignored
    h = tmp_path / "hf"
    h.mkdir()
    save_file(hf, str(h / "model.safetensors"))
    a, b = CheckpointSource(cfg, str(d)), CheckpointSource(cfg, str(h))
    for k in w:
        assert torch.equal(a.get(k, "cpu"), b.get(k, "cpu")), k
    ref = Engine(cfg, "cpu", source=a, num_pages=16, page_size=16).generate([list(range(20))], 4)
    got = Engine(cfg, "cpu", source=b, num_pages=16, page_size=16).generate([list(range(20))], 4)
    assert got == ref
