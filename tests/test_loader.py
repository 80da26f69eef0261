"""Checkpoint loader: role split, q/k/v and gate/up merging, TP sharding with GQA replication,
EP partition with zero padding, block-FP8 expert weights and scales."""
import dataclasses

import pytest
import torch

from fastafd_b200.config import PRESETS
from fastafd_b200.models.loader import load_attention_stage, load_expert_stage, normalize_key, save_checkpoint
from fastafd_b200.models.transformer import AttentionStage, ExpertStage, shard_attention_param
from fastafd_b200.reference import ops_ref as ref

CFG = dataclasses.replace(PRESETS["tiny-qwen3-moe"], num_layers=2, num_experts=6)


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    attn = AttentionStage(CFG, "cpu", torch.float32).init_random(3)
    exp = ExpertStage(CFG, "cpu", torch.float32).init_random(3)
    save_checkpoint(CFG, attn, [exp], str(d / "bf16"), shard_mb=1)
    save_checkpoint(CFG, attn, [exp], str(d / "fp8"), fp8_experts=True, shard_mb=1)
    return d, attn, exp


def test_key_normalisation():
    assert normalize_key("model.language_model.layers.0.self_attn.q_proj.weight") == "model.layers.0.self_attn.q_proj.weight"
    assert normalize_key("model.layers.1.self_attn.k_scale") is None
    assert normalize_key("model.layers.1.block_sparse_moe.gate.weight") == "model.layers.1.mlp.gate.weight"
    assert normalize_key("visual.blocks.0.attn.qkv.weight") is None


def test_attention_stage_roundtrip_and_role_split(ckpt):
    d, attn, _ = ckpt
    got = AttentionStage(CFG, "cpu", torch.float32)
    load_attention_stage(got, str(d / "bf16"))
    assert set(got.w) == set(attn.w)
    for k in attn.w:
        assert torch.equal(got.w[k], attn.w[k]), k
    assert not any("experts" in k for k in got.w)


@pytest.mark.parametrize("tp", [2, 4])
def test_tp_shards_reassemble(ckpt, tp):
    d, attn, _ = ckpt
    D, Hq, Hkv = CFG.head_dim, CFG.num_q_heads, CFG.num_kv_heads
    shards = []
    for r in range(tp):
        s = AttentionStage(CFG, "cpu", torch.float32, r, tp)
        load_attention_stage(s, str(d / "bf16"))
        shards.append(s)
    name = "model.layers.0.self_attn.qkv_proj.weight"
    full = attn.w[name]
    hq, hkv = Hq // tp, max(1, Hkv // tp)
    q = torch.cat([s.w[name][:hq * D] for s in shards], 0)
    assert torch.equal(q, full[:Hq * D])
    for r, s in enumerate(shards):
        kv_rank = r * Hkv // tp if Hkv < tp else r          # kv heads replicate when tp > kv heads
        k = s.w[name][hq * D:(hq + hkv) * D]
        assert torch.equal(k, full[Hq * D + kv_rank * hkv * D: Hq * D + (kv_rank + 1) * hkv * D])
    o = torch.cat([s.w["model.layers.0.self_attn.o_proj.weight"] for s in shards], 1)
    assert torch.equal(o, attn.w["model.layers.0.self_attn.o_proj.weight"])
    emb = torch.cat([s.w["model.embed_tokens.weight"] for s in shards], 0)
    assert torch.equal(emb, attn.w["model.embed_tokens.weight"])


def test_expert_partition_with_zero_padding(ckpt):
    d, _, exp = ckpt
    parts = []
    for r in range(4):                              # 6 experts over 4 ranks: 2,2,2,0(padding)
        s = ExpertStage(CFG, "cpu", torch.float32, r, 4)
        load_expert_stage(s, str(d / "bf16"))
        parts.append(s)
    assert parts[0].experts_local == 2
    for layer in exp.moe_layers:
        got = torch.cat([p.gate_up[layer] for p in parts], 0)
        assert torch.equal(got[:6], exp.gate_up[layer])
        assert float(got[6:].abs().sum()) == 0.0
        assert torch.equal(torch.cat([p.down[layer] for p in parts], 0)[:6], exp.down[layer])


def test_fp8_checkpoint_keeps_exact_block_scales(ckpt):
    d, _, exp = ckpt
    s = ExpertStage(CFG, "cpu", torch.float32)
    load_expert_stage(s, str(d / "fp8"))
    layer = exp.moe_layers[0]
    I = CFG.moe_intermediate_size
    q, sc = ref.block_quant_fp8(exp.gate_up[layer][1, :I])
    torch.testing.assert_close(s.gate_up[layer][1, :I], ref.block_dequant_fp8(q, sc))     # CPU stage dequantises
    torch.testing.assert_close(s.gate_up[layer], exp.gate_up[layer], atol=0.02, rtol=0.08)


def test_missing_tensor_is_reported(ckpt, tmp_path):
    import shutil, glob, os
    d, _, _ = ckpt
    dst = tmp_path / "broken"
    shutil.copytree(d / "bf16", dst)
    os.remove(sorted(glob.glob(str(dst / "*.safetensors")))[0])
    with pytest.raises(KeyError):
        load_attention_stage(AttentionStage(CFG, "cpu", torch.float32), str(dst))
