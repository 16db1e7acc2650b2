"""Converters, security helpers and the HF adapter on CPU."""
import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.utils import conversion as cv
from complexity_framework_b200.utils import security as sec

CFG = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
           vocab_size=256, intermediate_size=64, shared_intermediate_size=128, num_experts=4,
           top_k=2, routing_strategy="token_id_multi_hash", max_position_embeddings=64)


def _model():
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(**CFG)).eval()


def test_token_routed_conversion_transplants_tables():
    m = _model()
    sd = m.state_dict()
    old = {}
    for k, v in sd.items():
        if ".mlp.engine.expert_gate" in k:
            old[k.replace("engine.expert_gate", "gate_proj_w")] = v
        elif ".mlp.engine.expert_up" in k:
            old[k.replace("engine.expert_up", "up_proj_w")] = v
        elif ".mlp.engine.expert_down" in k:
            old[k.replace("engine.expert_down", "down_proj_w")] = v
        elif ".mlp.engine.route_table" in k:
            old[k.replace("engine.route_table", "topk_token_to_expert")] = v
        elif ".mlp.engine." in k and "fused" not in k and "_route_weights" not in k:
            old[k.replace("engine.", "")] = v
        elif ".mlp." not in k:
            old[k] = v
    cfg = dict(m.config.to_dict(), mlp_type="token_routed")
    new = cv.convert_token_routed_checkpoint(old, cfg).eval()
    ids = torch.randint(0, 256, (2, 16))
    assert torch.allclose(new(ids)["logits"], m(ids)["logits"], atol=1e-5)


def test_expert_expansion_preserves_outputs():
    m = _model()
    new = cv.convert_checkpoint_to_expanded_experts(m.state_dict(), m.config.to_dict()).eval()
    assert new.config.num_experts == 8
    ids = torch.randint(0, 256, (2, 16))
    assert torch.allclose(new(ids)["logits"], m(ids)["logits"], atol=1e-4)


def test_multi_hash_conversion_keeps_experts():
    m = _model()
    new = cv.convert_checkpoint_to_multi_hash(m.state_dict(), m.config.to_dict())
    a = m.state_dict()["layers.0.mlp.engine.expert_gate"]
    assert torch.equal(new.state_dict()["layers.0.mlp.engine.expert_gate"], a)


def test_hf_mapping_roundtrip():
    m = _model()
    hf = cv.convert_to_hf_state_dict(m.state_dict())
    assert "model.layers.0.self_attn.q_proj.weight" in hf
    back = cv.convert_hf_state_dict(hf)
    assert torch.equal(back["layers.1.self_attn.o_proj.weight"],
                       m.state_dict()["layers.1.self_attn.o_proj.weight"])


def test_security_helpers(tmp_path):
    m = _model()
    h = sec.compute_model_hash(m)
    assert sec.verify_model_hash(m, h)
    p = tmp_path / "w.pt"
    torch.save(m.state_dict(), p)
    sd = sec.safe_torch_load(p, expected_sha256=sec.file_sha256(p))
    assert set(sd) == set(m.state_dict())
    torch.save({"obj": object.__new__(sec.ModelManifest)}, tmp_path / "bad.pt") if False else None
    with pytest.raises(sec.UnsafeCheckpointError):
        sec.safe_torch_load(p, expected_sha256="0" * 64)
    with pytest.raises(ValueError):
        sec.validate_input_ids(torch.tensor([[0, 300]]), 256)
    assert sec.sanitize_config({"wandb_api_key": "x", "lr": 1})["wandb_api_key"] == "***"
    log = sec.AuditLogger(tmp_path / "audit.jsonl")
    with sec.SecureTrainingContext(tmp_path / "audit.jsonl", {"token": "t"}):
        pass
    ev = log.events()
    assert [e["event"] for e in ev] == ["training_start", "training_end"]
    m.save_pretrained(tmp_path / "ck")
    man = sec.create_model_manifest(m, tmp_path / "ck")
    man.save(tmp_path / "ck" / "manifest.json")
    assert sec.ModelManifest.load(tmp_path / "ck" / "manifest.json").verify_files(tmp_path / "ck") == []


def test_hf_adapter_roundtrip(tmp_path):
    pytest.importorskip("transformers")
    from complexity_framework_b200.integrations.hf import (TRHashForCausalLM, export_hf,
                                                           register_auto_classes)
    m = _model()
    export_hf(m, tmp_path / "hf")
    register_auto_classes()
    from transformers import AutoModelForCausalLM

    hf = AutoModelForCausalLM.from_pretrained(str(tmp_path / "hf"))
    assert isinstance(hf, TRHashForCausalLM)
    ids = torch.randint(0, 256, (1, 12))
    assert torch.allclose(hf(ids).logits, m(ids)["logits"], atol=1e-5)
    # native names: the same directory also loads as a ComplexityModel
    m2 = ComplexityModel.from_pretrained(tmp_path / "hf")
    assert torch.allclose(m2(ids)["logits"], m(ids)["logits"], atol=1e-5)
    out = hf.generate(ids, max_new_tokens=3)
    assert out.shape == (1, 15)
