"""Released-format DSV4 checkpoints: FP8/FP4 codecs, write + load round trip, and loading with the
reference loader for parity."""

import os
import shutil

import pytest
import torch

from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM
from tiny_dsv41_b200.models.dsv4.checkpoint import load_dsv41_backbone_prefix, write_released_checkpoint
from tiny_dsv41_b200.utils import quant

from ref_oracle import import_reference, reference_available

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_fp4_fp8_codecs_roundtrip():
    torch.manual_seed(0)
    w = torch.randn(64, 128) * 0.02
    packed, scale = quant.quantize_fp4_rows(w)
    assert packed.shape == (64, 64) and scale.shape == (64, 4)
    back = quant.dequantize_fp4_rows(packed, scale, dtype=torch.float32)
    # E2M1 keeps ~1 significant bit: error bounded by half the largest code gap relative to amax
    blocks = w.view(64, 4, 32).abs().amax(-1, keepdim=True)
    assert ((back - w).view(64, 4, 32).abs() <= blocks / 3 + 1e-12).all()
    exact = torch.tensor(quant.E2M1_VALUES[:8]).repeat(4).view(1, 32) * 0.25
    p2, s2 = quant.quantize_fp4_rows(exact)
    assert torch.equal(quant.dequantize_fp4_rows(p2, s2, dtype=torch.float32), exact)
    q, s = quant.quantize_fp8_blocks(w)
    assert (quant.dequantize_fp8_blocks(q, s, dtype=torch.float32) - w).abs().max() < 0.1 * w.abs().max()


def test_released_checkpoint_roundtrip(tmp_path):
    torch.manual_seed(0)
    model = DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny())
    write_released_checkpoint(model, tmp_path)
    loaded = load_dsv41_backbone_prefix(tmp_path, num_layers=6, dtype=torch.float32)
    ids = torch.randint(0, 32, (1, 24))
    with torch.no_grad():
        a, b = model(ids, labels=ids).loss, loaded(ids, labels=ids).loss
    assert abs(a.item() - b.item()) < 0.05 * a.item()
    prefix = load_dsv41_backbone_prefix(tmp_path, num_layers=3, dtype=torch.float32)
    assert len(prefix.model.layers) == 3 and prefix.config.candidate_source_layer_id == -1


@pytest.mark.skipif(not reference_available(), reason="reference not installed under baseline/_ref")
def test_loader_parity_with_reference(tmp_path):
    import_reference()
    from dsv41_train.models.dsv4.checkpoint import load_dsv41_backbone_prefix as ref_load

    import json
    import shutil

    from tiny_dsv41_b200.models.dsv4.model import build_compressed_token_map

    torch.manual_seed(0)
    write_released_checkpoint(DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny()), tmp_path)
    # the reference derives the Engram token map from the checkpoint tokenizer
    shutil.copy(os.path.join(ROOT, "examples", "tiny-dsv41", "tokenizer.json"), tmp_path / "tokenizer.json")
    _, compressed = build_compressed_token_map(tmp_path / "tokenizer.json")
    config = json.loads((tmp_path / "config.json").read_text())
    config["engram_compressed_vocab_size"] = compressed
    (tmp_path / "config.json").write_text(json.dumps(config))
    mine = load_dsv41_backbone_prefix(tmp_path, num_layers=6, dtype=torch.float32)
    ref = ref_load(tmp_path, num_layers=6, dtype=torch.float32)
    ref_state = ref.state_dict()
    for name, value in mine.state_dict().items():
        assert torch.equal(value, ref_state[name]), name


def test_frozen_fp4_experts_match_dequantised(tmp_path):
    """Experts kept as MXFP4 codes give the same forward and input gradient as experts dequantised
    at load (the same FP4 values either way)."""
    from tiny_dsv41_b200.models.dsv4.checkpoint import load_dsv41_backbone_prefix
    from tiny_dsv41_b200.ops.fp4 import dequantize_fp4

    torch.manual_seed(0)
    write_released_checkpoint(DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny()), tmp_path)
    shutil.copy(os.path.join(ROOT, "examples", "tiny-dsv41", "tokenizer.json"), tmp_path / "tokenizer.json")
    dense = load_dsv41_backbone_prefix(tmp_path, num_layers=3, dtype=torch.float32)
    packed = load_dsv41_backbone_prefix(tmp_path, num_layers=3, dtype=torch.float32, fp4_experts=True)
    routed = packed.model.layers[1].moe.routed
    assert routed.frozen_fp4 and not any("routed" in n for n, _ in packed.named_parameters())
    expanded = dequantize_fp4(routed.gate_up_fp4, routed.gate_up_scale).float()
    assert torch.equal(expanded, dense.model.layers[1].moe.routed.gate_up.detach().to(torch.bfloat16).float())
    ids = torch.randint(0, 32, (1, 24))
    emb = [m.model.embedding.weight for m in (dense, packed)]
    for e in emb:
        e.requires_grad_(True)
    a = dense(ids, labels=ids)
    b = packed(ids, labels=ids)
    assert torch.allclose(a.loss, b.loss, rtol=2e-2), (a.loss, b.loss)
    a.loss.backward()
    b.loss.backward()
    rel = (emb[0].grad - emb[1].grad).norm() / emb[0].grad.norm()
    assert rel < 5e-2, rel
